/*
 * lancius_types.h -- tensor dtype / ownership / runtime-state types shared by
 * the IR, the planner and the CUDA executor.
 *
 * ABI-compatible with the reference's bleeding/v11A1/include/lancius/lancius_types.h:9-60
 * (same enum values, same lancius_runtime_state field order) so that a graph
 * built against either header can be handed to this library.
 */
#ifndef LANCIUS_TYPES_H
#define LANCIUS_TYPES_H

#include <stddef.h>
#include <stdint.h>

typedef enum {
    LANCIUS_DTYPE_FP64 = 0,
    LANCIUS_DTYPE_INT8 = 1,
    LANCIUS_DTYPE_FP32 = 2,
    LANCIUS_DTYPE_INT32 = 3
} lancius_dtype;

static inline size_t lancius_dtype_size(lancius_dtype dt) {
    return dt == LANCIUS_DTYPE_FP32 ? 4u : dt == LANCIUS_DTYPE_INT8 ? 1u
         : dt == LANCIUS_DTYPE_INT32 ? 4u : 8u;
}

static inline const char* lancius_dtype_name(lancius_dtype dt) {
    return dt == LANCIUS_DTYPE_FP64 ? "fp64" : dt == LANCIUS_DTYPE_FP32 ? "fp32"
         : dt == LANCIUS_DTYPE_INT8 ? "int8" : dt == LANCIUS_DTYPE_INT32 ? "int32" : "unknown";
}

static inline int lancius_dtype_is_valid(uint8_t code) { return code <= (uint8_t)LANCIUS_DTYPE_INT32; }

typedef enum {
    LANCIUS_MEMORY_EXTERNAL = 0,
    LANCIUS_MEMORY_ARENA = 1,
    LANCIUS_MEMORY_POOL = 2,
    LANCIUS_MEMORY_OWNED_HEAP = 3
} lancius_memory_owner;

/* Mutable per-node execution state; `offset` is the node's byte offset inside
 * the pooled buffer (host pool for the CPU executor, the per-GPU device pool
 * for lancius_schedule_execute_cuda). */
typedef struct lancius_runtime_state {
    void* buffer;
    int8_t* buffer_int8;
    lancius_dtype dtype;
    double scale;
    lancius_memory_owner owner;
    lancius_memory_owner buffer_owner;
    lancius_memory_owner int8_owner;
    size_t offset;
    uint32_t flags;
} lancius_runtime_state;

#define LANCIUS_RT_FLAG_AUTOFREE_BUFFER (1u << 0)
#define LANCIUS_RT_FLAG_AUTOFREE_INT8   (1u << 1)

#endif

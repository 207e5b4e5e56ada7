/*
 * lancius_scheduler.h -- wave (level-set) schedule of a graph.
 * Struct layout and entry points follow the reference's
 * bleeding/v11A1/include/lancius/lancius_scheduler.h:10-29. The CPU executors
 * (lancius_schedule_execute*) are not part of this library: execution goes through
 * lancius_schedule_execute_cuda (lancius_cuda.h).
 */
#ifndef LANCIUS_SCHEDULER_H
#define LANCIUS_SCHEDULER_H
#include "lancius/lancius_ir.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct { lancius_node** nodes; uint32_t node_count; } lancius_wave;
struct lancius_memory_plan;
typedef struct { lancius_wave* waves; uint32_t wave_count; struct lancius_memory_plan* plan; void* static_pool; } lancius_schedule;

lancius_schedule* lancius_ir_schedule(lancius_graph* g);
void lancius_schedule_destroy(lancius_schedule* schedule);
size_t lancius_schedule_peak_memory(lancius_schedule* schedule);

typedef struct {
    size_t peak_memory_bytes;
    size_t total_allocs;
    size_t tensor_count;
} lancius_liveness_profile;

lancius_liveness_profile lancius_analyze_liveness(lancius_graph* g);
void lancius_schedule_attach_pool(lancius_schedule* schedule, void* flat_buffer, struct lancius_memory_plan* plan);

#ifdef __cplusplus
}
#endif
#endif

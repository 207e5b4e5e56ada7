/*
 * lancius_scheduler.h -- wave (level-set) schedule of a graph.
 * Struct layout and entry points follow the reference's
 * bleeding/v11A1/include/lancius/lancius_scheduler.h:10-29.
 *
 * The three executors keep the reference's names, arguments and host-side memory
 * contract (which node gets which runtime_data pointer), but run the math on a GPU
 * through an implicit per-thread device context (device LANCIUS_CUDA_DEVICE, default
 * 0; LANCIUS_CUDA_MODE=tf32 or bf16 selects a fast mode, default FP32-exact):
 * bound INPUT data is uploaded, the schedule runs on the device, and every node
 * that no other node reads (the graph's outputs) is copied back into its FP64
 * runtime_data before the call returns. LCU_DROPIN_DOWNLOAD_ALL=1 copies back every
 * computed node instead (the device then keeps each node's own value: no epilogue
 * folding). Errors: lancius_get_error(). lancius_dropin_release() frees the calling
 * thread's device context. Direct control of the device (pinned buffers, streams,
 * graph replay) is lancius_cuda.h.
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

struct lancius_arena;
struct lancius_pool;

lancius_schedule* lancius_ir_schedule(lancius_graph* g);
/* reference: lancius_scheduler.c:311-362 (nodes without runtime_data get it from
 * `scratch`, or from the attached pool when the plan pools them) */
void lancius_schedule_execute(lancius_schedule* schedule, struct lancius_arena* scratch);
/* reference: lancius_scheduler.c:364-413; `pool` must be non-NULL as there, but the
 * wave's nodes are run concurrently by the device, not by the pool's threads */
void lancius_schedule_execute_parallel(lancius_schedule* schedule, struct lancius_arena* scratch,
                                       struct lancius_pool* pool);
/* reference: lancius_scheduler.c:475-520 (every computed node is bump-placed in
 * flat_buffer, 32-byte aligned, in wave order) */
void lancius_schedule_execute_static(lancius_schedule* schedule, void* flat_buffer);
/* No reference counterpart: frees the calling thread's implicit device context. */
void lancius_dropin_release(void);
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

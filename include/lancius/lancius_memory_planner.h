/*
 * lancius_memory_planner.h -- liveness-based offset planner for one flat pool.
 *
 * The plan struct and lancius_build_memory_plan() signature match the reference
 * (bleeding/v11A1/include/lancius/lancius_memory_planner.h:13-23). This
 * implementation keeps each live interval's own offset while scanning, so two
 * tensors alive in the same wave never share bytes (the reference writes the
 * chosen offset only into plan->offsets and frees blocks at offset 0,
 * lancius_memory_planner.c:122-127,140,162). lancius_memory_plan_validate()
 * checks that property for any plan, including one produced elsewhere.
 */
#ifndef LANCIUS_MEMORY_PLANNER_H
#define LANCIUS_MEMORY_PLANNER_H
#include "lancius/lancius_ir.h"
#include "lancius/lancius_scheduler.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lancius_memory_plan {
    size_t peak_memory;   /* bytes of the flat pool */
    size_t* offsets;      /* [g->next_id] byte offset of each pooled node */
    uint8_t* is_pooled;   /* [g->next_id] 1 when the node lives in the pool */
} lancius_memory_plan;

/* Same contract as the reference: sizes come from lancius_node_bytes(), 32-B aligned. */
lancius_memory_plan* lancius_build_memory_plan(lancius_schedule* sched, lancius_graph* g);

/* Planner with an explicit element size (4 for the FP32 device pool) and slot
 * alignment; RESHAPE/FLATTEN nodes alias their source when alias_views != 0
 * (is_pooled = 2 marks an alias: offsets[id] is the source's offset). */
lancius_memory_plan* lancius_build_memory_plan_ex(lancius_schedule* sched, lancius_graph* g,
                                                  size_t elem_bytes, size_t align, int alias_views);

/* Returns LANCIUS_ERROR_OK when no two simultaneously live pooled tensors overlap
 * and every slot fits inside peak_memory; LANCIUS_ERROR_INVALID_MODEL otherwise. */
lancius_error lancius_memory_plan_validate(const lancius_memory_plan* plan, lancius_schedule* sched,
                                           lancius_graph* g, size_t elem_bytes);

void lancius_memory_plan_destroy(lancius_memory_plan* plan);

#ifdef __cplusplus
}
#endif
#endif

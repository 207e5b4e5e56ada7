/* Executor-side planner entry: plans with an explicit alias table (fused chains
 * and views share the bytes of their storage root). Not part of the public ABI. */
#ifndef LCU_PLANNER_INTERNAL_H
#define LCU_PLANNER_INTERNAL_H
#include "lancius/lancius_memory_planner.h"
#ifdef __cplusplus
extern "C" {
#endif
#define LCU_ALIAS_NONE   0xFFFFFFFFu
#define LCU_ALIAS_ELIDED 0xFFFFFFFEu
lancius_memory_plan* lcu_plan_aliased(lancius_schedule* s, lancius_graph* g, size_t elem_bytes, size_t align,
                                      const uint32_t* alias);
#ifdef __cplusplus
}
#endif
#endif

/*
 * Wave schedule: a node's wave is 0 when it has no inputs, else one more than the
 * latest wave among its inputs. This is the level set that the reference's
 * repeated ready-scan produces (bleeding/v11A1/src/runtime/lancius_scheduler.c:12-59),
 * with nodes inside a wave kept in graph order. A cycle is reported as
 * LANCIUS_ERROR_INVALID_MODEL and NULL instead of a truncated schedule.
 */
#include "lancius/lancius_scheduler.h"
#include "lancius/lancius_memory_planner.h"
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define UNSET 0xFFFFFFFFu

lancius_schedule* lancius_ir_schedule(lancius_graph* g) {
    if (!g || g->node_count == 0) return NULL;
    uint32_t* lvl = (uint32_t*)malloc(sizeof(uint32_t) * g->next_id);
    uint32_t* count = NULL;
    lancius_schedule* s = NULL;
    if (!lvl) goto oom;
    for (uint32_t i = 0; i < g->next_id; i++) lvl[i] = UNSET;

    uint32_t placed = 0, depth = 0;
    for (int changed = 1; changed && placed < g->node_count;) {
        changed = 0;
        for (uint32_t i = 0; i < g->node_count; i++) {
            const lancius_node* n = g->nodes[i];
            if (lvl[n->id] != UNSET) continue;
            uint32_t l = 0; int ready = 1;
            for (uint32_t j = 0; j < n->input_count; j++) {
                uint32_t li = n->inputs[j] ? lvl[n->inputs[j]->id] : UNSET;
                if (li == UNSET) { ready = 0; break; }
                if (li + 1 > l) l = li + 1;
            }
            if (!ready) continue;
            lvl[n->id] = l; placed++; changed = 1;
            if (l + 1 > depth) depth = l + 1;
        }
    }
    if (placed < g->node_count) {
        fprintf(stderr, "[LANCIUS SCHEDULE] cycle or dangling input: placed %u of %u nodes\n", placed, g->node_count);
        free(lvl);
        lancius_set_error(LANCIUS_ERROR_INVALID_MODEL);
        return NULL;
    }

    s = (lancius_schedule*)calloc(1, sizeof(*s));
    count = (uint32_t*)calloc(depth, sizeof(uint32_t));
    if (!s || !count) goto oom;
    s->waves = (lancius_wave*)calloc(depth, sizeof(lancius_wave));
    if (!s->waves) goto oom;
    s->wave_count = depth;
    for (uint32_t i = 0; i < g->node_count; i++) count[lvl[g->nodes[i]->id]]++;
    for (uint32_t w = 0; w < depth; w++) {
        s->waves[w].nodes = (lancius_node**)malloc(sizeof(lancius_node*) * count[w]);
        if (!s->waves[w].nodes) goto oom;
    }
    for (uint32_t i = 0; i < g->node_count; i++) {
        lancius_wave* w = &s->waves[lvl[g->nodes[i]->id]];
        w->nodes[w->node_count++] = g->nodes[i];
    }
    free(lvl); free(count);
    return s;
oom:
    free(lvl); free(count);
    lancius_schedule_destroy(s);
    lancius_set_error(LANCIUS_ERROR_OOM);
    return NULL;
}

void lancius_schedule_destroy(lancius_schedule* s) {
    if (!s) return;
    if (s->waves) for (uint32_t w = 0; w < s->wave_count; w++) free(s->waves[w].nodes);
    free(s->waves);
    free(s);
}

/* reference :428-443 -- largest sum of non-INPUT/CONST node bytes within one wave */
size_t lancius_schedule_peak_memory(lancius_schedule* s) {
    size_t peak = 0;
    if (!s) return 0;
    for (uint32_t w = 0; w < s->wave_count; w++) {
        size_t b = 0;
        for (uint32_t i = 0; i < s->waves[w].node_count; i++) {
            const lancius_node* n = s->waves[w].nodes[i];
            if (n->op != LANCIUS_OP_INPUT && n->op != LANCIUS_OP_CONST) b += lancius_node_bytes(n);
        }
        if (b > peak) peak = b;
    }
    return peak;
}

/* reference :448-470 (FP64 element size, as there) */
lancius_liveness_profile lancius_analyze_liveness(lancius_graph* g) {
    lancius_liveness_profile p = { 0, 0, 0 };
    lancius_schedule* s = lancius_ir_schedule(g);
    if (!s) return p;
    for (uint32_t w = 0; w < s->wave_count; w++) {
        size_t b = 0;
        for (uint32_t i = 0; i < s->waves[w].node_count; i++) {
            const lancius_node* n = s->waves[w].nodes[i];
            if (n->op != LANCIUS_OP_INPUT && n->op != LANCIUS_OP_CONST) {
                b += lancius_node_elements(n) * sizeof(double);
                p.tensor_count++;
            }
        }
        if (b > p.peak_memory_bytes) p.peak_memory_bytes = b;
        p.total_allocs += s->waves[w].node_count;
    }
    lancius_schedule_destroy(s);
    return p;
}

void lancius_schedule_attach_pool(lancius_schedule* s, void* flat_buffer, lancius_memory_plan* plan) {
    if (!s) return;
    s->static_pool = flat_buffer;
    s->plan = plan;
}

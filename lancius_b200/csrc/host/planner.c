/*
 * Liveness planner for one flat pool.
 *
 * Liveness follows the reference (bleeding/v11A1/src/runtime/lancius_memory_planner.c:33-92):
 * a non-INPUT/CONST node is born in its wave, dies in the last wave that reads it,
 * and a node no other node reads lives to the end (wave_count). Placement differs:
 * intervals are taken in birth order and each goes to the lowest offset that does
 * not overlap any interval still alive, using the live intervals' own offsets.
 * (The reference frees expired blocks at the offset recorded in its interval copy,
 * which is always 0, so it can hand live bytes to a new tensor.)
 */
#include "lancius/lancius_memory_planner.h"
#include "planner_internal.h"
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define NONE 0xFFFFFFFFu

typedef struct { uint32_t id, birth, death; size_t size, off; } span;

static size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static int is_view_op(const lancius_node* n) {
    return n->op == LANCIUS_OP_RESHAPE || n->op == LANCIUS_OP_FLATTEN;
}

/* Storage owner of a node. `alias` (optional, indexed by id) maps a node onto the
 * node whose bytes it shares (LCU_ALIAS_NONE = owns its bytes, LCU_ALIAS_ELIDED =
 * needs no bytes); without a table, alias_views makes RESHAPE/FLATTEN share
 * their source's bytes. */
typedef struct { const uint32_t* alias; const lancius_node** byid; int alias_views; } rootctx;

static const lancius_node* storage_root(const lancius_node* n, const rootctx* rc) {
    for (int hops = 0; hops < 1 << 20; hops++) {
        if (rc->alias) {
            uint32_t a = rc->alias[n->id];
            if (a == LCU_ALIAS_NONE || a == LCU_ALIAS_ELIDED || !rc->byid[a]) return n;
            n = rc->byid[a];
        } else if (rc->alias_views && is_view_op(n) && n->input_count == 1 && n->inputs[0]) {
            n = n->inputs[0];
        } else {
            return n;
        }
    }
    return n;
}

static int elided(const lancius_node* n, const rootctx* rc) {
    return rc->alias && rc->alias[n->id] == LCU_ALIAS_ELIDED;
}

static int pooled_op(const lancius_node* n) {
    return n->op != LANCIUS_OP_INPUT && n->op != LANCIUS_OP_CONST && n->op != LANCIUS_OP_NOP;
}

/* birth/death per storage root; returns number of waves or 0 on OOM */
static int liveness(lancius_schedule* s, lancius_graph* g, const rootctx* rc,
                    uint32_t* birth, uint32_t* death) {
    uint32_t ids = g->next_id;
    uint8_t* read = (uint8_t*)calloc(ids, 1);
    if (!read) return 0;
    for (uint32_t i = 0; i < ids; i++) { birth[i] = NONE; death[i] = 0; }
    for (uint32_t i = 0; i < g->node_count; i++)
        for (uint32_t j = 0; j < g->nodes[i]->input_count; j++)
            if (g->nodes[i]->inputs[j]) read[g->nodes[i]->inputs[j]->id] = 1;
    for (uint32_t w = 0; w < s->wave_count; w++) {
        for (uint32_t i = 0; i < s->waves[w].node_count; i++) {
            const lancius_node* n = s->waves[w].nodes[i];
            const lancius_node* r = storage_root(n, rc);
            if (r == n && pooled_op(n) && !elided(n, rc) && birth[n->id] == NONE) birth[n->id] = w;
            /* a node no one reads stays alive to the end of the schedule */
            if (!read[n->id]) {
                uint32_t rid = r->id;
                death[rid] = s->wave_count;
            }
            for (uint32_t j = 0; j < n->input_count; j++) {
                if (!n->inputs[j]) continue;
                uint32_t rid = storage_root(n->inputs[j], rc)->id;
                if (w > death[rid]) death[rid] = w;
            }
        }
    }
    for (uint32_t i = 0; i < ids; i++)
        if (birth[i] != NONE && death[i] < birth[i]) death[i] = birth[i];
    free(read);
    return 1;
}

static const lancius_node** id_index(lancius_graph* g) {
    const lancius_node** byid = (const lancius_node**)calloc(g->next_id ? g->next_id : 1, sizeof(lancius_node*));
    if (byid) for (uint32_t i = 0; i < g->node_count; i++) byid[g->nodes[i]->id] = g->nodes[i];
    return byid;
}

static lancius_memory_plan* plan_core(lancius_schedule* s, lancius_graph* g, size_t elem_bytes, size_t align,
                                      int alias_views, const uint32_t* alias) {
    if (!s || !g || s->wave_count == 0) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return NULL; }
    if (align == 0 || (align & (align - 1))) align = 32;
    uint32_t ids = g->next_id;
    const lancius_node** byid = id_index(g);
    rootctx rc = { alias, byid, alias_views };
    uint32_t* birth = (uint32_t*)malloc(sizeof(uint32_t) * ids);
    uint32_t* death = (uint32_t*)malloc(sizeof(uint32_t) * ids);
    span* sp = (span*)malloc(sizeof(span) * (ids ? ids : 1));
    span** live = (span**)malloc(sizeof(span*) * (ids ? ids : 1));
    lancius_memory_plan* plan = (lancius_memory_plan*)calloc(1, sizeof(*plan));
    if (plan) {
        plan->offsets = (size_t*)calloc(ids ? ids : 1, sizeof(size_t));
        plan->is_pooled = (uint8_t*)calloc(ids ? ids : 1, 1);
    }
    if (!birth || !death || !sp || !live || !plan || !plan->offsets || !plan->is_pooled || !byid ||
        !liveness(s, g, &rc, birth, death)) {
        free(birth); free(death); free(sp); free(live); free((void*)byid);
        lancius_memory_plan_destroy(plan);
        lancius_set_error(LANCIUS_ERROR_OOM);
        return NULL;
    }

    /* spans in (birth, graph order) -- a stable counting walk over waves */
    uint32_t n_sp = 0;
    for (uint32_t w = 0; w < s->wave_count; w++)
        for (uint32_t i = 0; i < s->waves[w].node_count; i++) {
            const lancius_node* n = s->waves[w].nodes[i];
            if (birth[n->id] != w) continue;
            size_t bytes = elem_bytes ? lancius_node_elements(n) * elem_bytes : lancius_node_bytes(n);
            sp[n_sp].id = n->id; sp[n_sp].birth = w; sp[n_sp].death = death[n->id];
            sp[n_sp].size = round_up(bytes ? bytes : 1, align); sp[n_sp].off = 0;
            n_sp++;
        }

    size_t peak = 0;
    uint32_t n_live = 0;
    for (uint32_t k = 0; k < n_sp; k++) {
        span* c = &sp[k];
        uint32_t keep = 0;
        for (uint32_t a = 0; a < n_live; a++)
            if (live[a]->death >= c->birth) live[keep++] = live[a];
        n_live = keep;
        /* live list sorted by offset: find the first gap that fits */
        size_t cand = 0;
        for (uint32_t a = 0; a < n_live; a++) {
            if (live[a]->off >= cand + c->size) break;
            size_t end = live[a]->off + live[a]->size;
            if (end > cand) cand = end;
        }
        c->off = cand;
        uint32_t pos = n_live;
        while (pos > 0 && live[pos - 1]->off > c->off) { live[pos] = live[pos - 1]; pos--; }
        live[pos] = c; n_live++;
        if (c->off + c->size > peak) peak = c->off + c->size;
        plan->offsets[c->id] = c->off;
        plan->is_pooled[c->id] = 1;
    }
    for (uint32_t i = 0; i < g->node_count; i++) {
        const lancius_node* n = g->nodes[i];
        const lancius_node* r = storage_root(n, &rc);
        if (r != n) { plan->is_pooled[n->id] = 2; plan->offsets[n->id] = plan->offsets[r->id]; }
    }
    plan->peak_memory = peak;
    free(birth); free(death); free(sp); free(live); free((void*)byid);
    return plan;
}

lancius_memory_plan* lancius_build_memory_plan_ex(lancius_schedule* s, lancius_graph* g,
                                                  size_t elem_bytes, size_t align, int alias_views) {
    return plan_core(s, g, elem_bytes, align, alias_views, NULL);
}

lancius_memory_plan* lcu_plan_aliased(lancius_schedule* s, lancius_graph* g, size_t elem_bytes, size_t align,
                                      const uint32_t* alias) {
    return plan_core(s, g, elem_bytes, align, 0, alias);
}

lancius_memory_plan* lancius_build_memory_plan(lancius_schedule* s, lancius_graph* g) {
    return lancius_build_memory_plan_ex(s, g, 0, 32, 0);
}

lancius_error lancius_memory_plan_validate(const lancius_memory_plan* plan, lancius_schedule* s,
                                           lancius_graph* g, size_t elem_bytes) {
    if (!plan || !s || !g || !plan->offsets || !plan->is_pooled) {
        lancius_set_error(LANCIUS_ERROR_NULL_PTR);
        return LANCIUS_ERROR_NULL_PTR;
    }
    int alias = 0;
    for (uint32_t i = 0; i < g->next_id; i++) alias |= plan->is_pooled[i] == 2;
    uint32_t ids = g->next_id;
    const lancius_node** byid0 = id_index(g);
    rootctx rc = { NULL, byid0, alias };
    uint32_t* birth = (uint32_t*)malloc(sizeof(uint32_t) * ids);
    uint32_t* death = (uint32_t*)malloc(sizeof(uint32_t) * ids);
    uint32_t* list = (uint32_t*)malloc(sizeof(uint32_t) * (ids ? ids : 1));
    const lancius_node** byid = (const lancius_node**)calloc(ids ? ids : 1, sizeof(lancius_node*));
    if (!birth || !death || !list || !byid || !byid0 || !liveness(s, g, &rc, birth, death)) {
        free(birth); free(death); free(list); free(byid); free((void*)byid0);
        lancius_set_error(LANCIUS_ERROR_OOM);
        return LANCIUS_ERROR_OOM;
    }
    lancius_error err = LANCIUS_ERROR_OK;
    uint32_t n = 0;
    for (uint32_t i = 0; i < g->node_count; i++) byid[g->nodes[i]->id] = g->nodes[i];
    for (uint32_t i = 0; i < g->node_count; i++) {
        const lancius_node* nd = g->nodes[i];
        if (birth[nd->id] == NONE) continue;              /* INPUT / CONST / NOP / alias */
        if (plan->is_pooled[nd->id] != 1) { err = LANCIUS_ERROR_INVALID_MODEL; break; }
        size_t bytes = elem_bytes ? lancius_node_elements(nd) * elem_bytes : lancius_node_bytes(nd);
        if (plan->offsets[nd->id] > plan->peak_memory || bytes > plan->peak_memory - plan->offsets[nd->id]) {
            err = LANCIUS_ERROR_INVALID_MODEL; break;
        }
        list[n++] = nd->id;
    }
    for (uint32_t a = 0; err == LANCIUS_ERROR_OK && a < n; a++) {
        const lancius_node* na = byid[list[a]];
        size_t sa = elem_bytes ? lancius_node_elements(na) * elem_bytes : lancius_node_bytes(na);
        size_t oa = plan->offsets[list[a]];
        for (uint32_t b = a + 1; b < n; b++) {
            uint32_t ia = list[a], ib = list[b];
            if (death[ia] < birth[ib] || death[ib] < birth[ia]) continue;   /* never alive together */
            const lancius_node* nb = byid[ib];
            size_t sb = elem_bytes ? lancius_node_elements(nb) * elem_bytes : lancius_node_bytes(nb);
            size_t ob = plan->offsets[ib];
            if (oa < ob + sb && ob < oa + sa) {
                fprintf(stderr, "[LANCIUS PLAN] nodes %u and %u are live together and overlap\n", ia, ib);
                err = LANCIUS_ERROR_INVALID_MODEL; break;
            }
        }
    }
    free(birth); free(death); free(list); free(byid); free((void*)byid0);
    if (err != LANCIUS_ERROR_OK) lancius_set_error(err);
    return err;
}

void lancius_memory_plan_destroy(lancius_memory_plan* plan) {
    if (!plan) return;
    free(plan->offsets); free(plan->is_pooled); free(plan);
}

/*
 * Conv2D+ReLU fusion pass, same rewrite as the reference
 * (bleeding/v11A1/src/compiler/lancius_optimizer.c:15-41): a RELU whose input is a
 * CONV2D with exactly one consumer becomes CONV2D_RELU_FUSED over the conv's
 * inputs and attributes; the conv becomes a NOP with no inputs.
 */
#include "lancius/lancius_ir.h"

static int consumers_of(const lancius_graph* g, const lancius_node* t) {
    int c = 0;
    for (uint32_t i = 0; i < g->node_count; i++)
        for (uint32_t j = 0; j < g->nodes[i]->input_count; j++)
            c += g->nodes[i]->inputs[j] == t;
    return c;
}

void lancius_optimize_fusion(lancius_graph* g) {
    if (!g) return;
    for (uint32_t k = g->node_count; k-- > 0;) {
        lancius_node* r = g->nodes[k];
        if (r->op != LANCIUS_OP_RELU || r->input_count == 0 || r->inputs[0]->op != LANCIUS_OP_CONV2D) continue;
        lancius_node* c = (lancius_node*)r->inputs[0];
        if (consumers_of(g, c) != 1) continue;
        r->op = LANCIUS_OP_CONV2D_RELU_FUSED;
        r->inputs = c->inputs; r->input_count = 2;
        r->kernel_h = c->kernel_h; r->kernel_w = c->kernel_w; r->stride = c->stride; r->pad = c->pad;
        for (int d = 0; d < 4; d++) r->shape[d] = c->shape[d];
        r->ndim = 4;
        c->op = LANCIUS_OP_NOP; c->input_count = 0; c->inputs = NULL;
    }
}

/*
 * BASIS stage-6 graph IR (the reference's src/basis/stage6_ir/graph.c:30-119 API) and
 * its lowering onto the Lancius IR, so BASIS-built MLP-shaped graphs run on the B200
 * executor. Builders follow the reference's shape rules and error behaviour (message on
 * stderr, NULL result); node ids are dense indices in creation order.
 */
#include "basis/stage6_ir/graph.h"
#include "lancius/lancius_ir.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static basis_node* push_node(basis_graph* g, basis_op_type op, size_t r, size_t c, const char* name) {
    if (!g) return NULL;
    if (g->node_count == g->node_cap) {
        size_t cap = g->node_cap ? 2 * g->node_cap : 16;
        basis_node* grown = (basis_node*)realloc(g->nodes, cap * sizeof(basis_node));
        if (!grown) return NULL;
        g->nodes = grown;
        g->node_cap = cap;
    }
    basis_node* n = &g->nodes[g->node_count];
    memset(n, 0, sizeof(*n));
    n->id = (int)g->node_count;
    n->op = op;
    n->input_ids[0] = n->input_ids[1] = -1;
    n->rows = r;
    n->cols = c;
    if (name) {
        size_t len = strlen(name);
        n->name = (char*)malloc(len + 1);
        if (n->name) memcpy(n->name, name, len + 1);
    }
    g->node_count++;
    return n;
}

basis_graph* basis_graph_new(void) { return (basis_graph*)calloc(1, sizeof(basis_graph)); }

basis_node* basis_graph_input(basis_graph* g, const char* name, size_t r, size_t c) {
    return push_node(g, BASIS_OP_INPUT, r, c, name);
}

/* a and b may point into g->nodes, which push_node can move: read them first */
static basis_node* binary(basis_graph* g, basis_op_type op, const basis_node* a, const basis_node* b, size_t r,
                          size_t c) {
    const int ia = a->id, ib = b->id;
    basis_node* n = push_node(g, op, r, c, NULL);
    if (n) { n->input_ids[0] = ia; n->input_ids[1] = ib; }
    return n;
}

basis_node* basis_graph_matmul(basis_graph* g, basis_node* a, basis_node* b) {
    if (!a || !b) return NULL;
    if (a->cols != b->rows) {
        fprintf(stderr, "[IR ERROR] MatMul shape mismatch: [%zux%zu] x [%zux%zu]\n", a->rows, a->cols, b->rows, b->cols);
        return NULL;
    }
    return binary(g, BASIS_OP_MATMUL, a, b, a->rows, b->cols);
}

basis_node* basis_graph_add(basis_graph* g, basis_node* a, basis_node* b) {
    if (!a || !b) return NULL;
    if (a->rows != b->rows || a->cols != b->cols) {
        fprintf(stderr, "[IR ERROR] Add shape mismatch\n");
        return NULL;
    }
    return binary(g, BASIS_OP_ADD, a, b, a->rows, a->cols);
}

basis_node* basis_graph_broadcast_add(basis_graph* g, basis_node* a, basis_node* bias) {
    if (!a || !bias) return NULL;
    if (bias->rows != 1 || bias->cols != a->cols) {
        fprintf(stderr, "[IR ERROR] Broadcast Add shape mismatch\n");
        return NULL;
    }
    return binary(g, BASIS_OP_BROADCAST_ADD, a, bias, a->rows, a->cols);
}

static basis_node* unary(basis_graph* g, basis_op_type op, const basis_node* a) {
    if (!a) return NULL;
    const int ia = a->id;
    const size_t r = a->rows, c = a->cols;
    basis_node* n = push_node(g, op, r, c, NULL);
    if (n) n->input_ids[0] = ia;
    return n;
}

basis_node* basis_graph_relu(basis_graph* g, basis_node* a) { return unary(g, BASIS_OP_RELU, a); }
basis_node* basis_graph_tanh(basis_graph* g, basis_node* a) { return unary(g, BASIS_OP_TANH, a); }

static const char* op_name(basis_op_type op) {
    static const char* names[] = {"INPUT", "MATMUL", "ADD", "RELU", "TANH", "BROADCAST_ADD"};
    return (unsigned)op < sizeof(names) / sizeof(names[0]) ? names[op] : "UNKNOWN";
}

void basis_graph_print(basis_graph* g) {
    if (!g) return;
    printf("=== BASIS Static Graph IR ===\n");
    for (size_t i = 0; i < g->node_count; i++) {
        const basis_node* n = &g->nodes[i];
        printf("Node %2d | %-15s | Shape: [%3zu x %3zu] | Inputs: ", n->id, op_name(n->op), n->rows, n->cols);
        if (n->op == BASIS_OP_INPUT) printf("None (Name: \"%s\")", n->name ? n->name : "(null)");
        else printf("[%d, %d]", n->input_ids[0], n->input_ids[1]);
        printf("\n");
    }
    printf("=============================\n");
}

void basis_graph_free(basis_graph* g) {
    if (!g) return;
    for (size_t i = 0; i < g->node_count; i++) free(g->nodes[i].name);
    free(g->nodes);
    free(g);
}

int basis_graph_lower(const basis_graph* bg, lancius_graph* lg, lancius_node** map) {
    if (!bg || !lg || !map) return -1;
    for (size_t i = 0; i < bg->node_count; i++) {
        const basis_node* n = &bg->nodes[i];
        const int i0 = n->input_ids[0], i1 = n->input_ids[1];
        const int arity = n->op == BASIS_OP_INPUT ? 0 : (n->op == BASIS_OP_RELU || n->op == BASIS_OP_TANH) ? 1 : 2;
        if ((arity >= 1 && (i0 < 0 || (size_t)i0 >= i)) || (arity == 2 && (i1 < 0 || (size_t)i1 >= i))) return -1;
        lancius_node* a = arity >= 1 ? map[i0] : NULL;
        lancius_node* b = arity == 2 ? map[i1] : NULL;
        lancius_node* out = NULL;
        switch (n->op) {
            case BASIS_OP_INPUT: out = lancius_input(lg, n->rows, n->cols); break;
            case BASIS_OP_MATMUL: out = lancius_matmul(lg, a, b); break;
            case BASIS_OP_ADD: out = lancius_add(lg, a, b); break;
            case BASIS_OP_RELU: out = lancius_relu(lg, a); break;
            case BASIS_OP_TANH: out = lancius_tanh(lg, a); break;
            case BASIS_OP_BROADCAST_ADD: out = lancius_add(lg, a, lancius_broadcast(lg, b, n->rows, n->cols)); break;
            default: return -1;
        }
        if (!out) return -1;
        map[i] = out;
    }
    return 0;
}

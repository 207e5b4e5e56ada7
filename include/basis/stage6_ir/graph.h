/*
 * BASIS stage-6 static graph IR: the reference's legacy 2-D graph-construction API
 * (include/basis/stage6_ir/graph.h, src/basis/stage6_ir/graph.c:30-119), kept
 * field-for-field and value-for-value compatible so code written against it builds
 * unchanged. The reference has no executor for it; here basis_graph_lower() turns it
 * into a Lancius graph (lancius_ir.h) that the B200 executor runs.
 */
#ifndef BASIS_STAGE6_IR_GRAPH_H
#define BASIS_STAGE6_IR_GRAPH_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    BASIS_OP_INPUT,
    BASIS_OP_MATMUL,
    BASIS_OP_ADD,
    BASIS_OP_RELU,
    BASIS_OP_TANH,
    BASIS_OP_BROADCAST_ADD
} basis_op_type;

typedef struct basis_node {
    int id;                 /* index in basis_graph.nodes */
    basis_op_type op;
    int input_ids[2];       /* -1 where unused */
    size_t rows;
    size_t cols;
    char* name;             /* INPUT nodes only (owned copy) */
} basis_node;

typedef struct basis_graph {
    basis_node* nodes;
    size_t node_count;
    size_t node_cap;
} basis_graph;

/* Builders: same shape rules as the reference (MATMUL a.cols == b.rows; ADD equal shapes;
 * BROADCAST_ADD bias is [1, a.cols]); a violated rule prints an error and returns NULL.
 * The returned pointer lives in g->nodes and moves when a later call grows the array. */
basis_graph* basis_graph_new(void);
basis_node* basis_graph_input(basis_graph* g, const char* name, size_t r, size_t c);
basis_node* basis_graph_matmul(basis_graph* g, basis_node* a, basis_node* b);
basis_node* basis_graph_add(basis_graph* g, basis_node* a, basis_node* b);
basis_node* basis_graph_broadcast_add(basis_graph* g, basis_node* a, basis_node* bias);
basis_node* basis_graph_relu(basis_graph* g, basis_node* a);
basis_node* basis_graph_tanh(basis_graph* g, basis_node* a);
void basis_graph_print(basis_graph* g);
void basis_graph_free(basis_graph* g);

/* Extension (no counterpart in the reference): lower `bg` onto the Lancius IR in `lg`.
 * map[i] receives the Lancius node computing basis node i (node_count entries); INPUT
 * becomes lancius_input, MATMUL/ADD/RELU map one to one, BROADCAST_ADD becomes
 * ADD(a, BROADCAST(bias)), TANH becomes LANCIUS_OP_TANH. Returns 0, or -1 on a NULL
 * argument or a node that refers to a later one. */
struct lancius_graph;
struct lancius_node;
int basis_graph_lower(const basis_graph* bg, struct lancius_graph* lg, struct lancius_node** map);

#ifdef __cplusplus
}
#endif
#endif

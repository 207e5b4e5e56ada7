/*
 * lancius_ir.h -- the Lancius static-graph IR: opcodes, node and graph structs,
 * and the shape-inferring node builders.
 *
 * Field order, opcode numbering and builder signatures are kept identical to the
 * reference (bleeding/v11A1/include/lancius/lancius_ir.h:16-148) so that code
 * written against Lancius builds unchanged against this library and graphs can be
 * exchanged between the two. Two additions, both outside the reference's numbering:
 *   - LANCIUS_OP_TANH (after LANCIUS_OP_GQA): needed to lower the legacy BASIS
 *     TANH node (reference src/basis/stage6_ir/graph.c:119-123);
 *   - lancius_attention_noncausal(): an ATTENTION node whose attr_val is 1.0,
 *     meaning "no mask" (the reference kernel is always causal,
 *     lancius_kernels.c:307; attr_val defaults to 0.0 = causal).
 */
#ifndef LANCIUS_IR_H
#define LANCIUS_IR_H
#include "lancius/lancius_arena.h"
#include "lancius/lancius_types.h"
#include "lancius/lancius_error.h"
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    LANCIUS_OP_NOP = 0, LANCIUS_OP_INPUT, LANCIUS_OP_CONST, LANCIUS_OP_ADD, LANCIUS_OP_SUB, LANCIUS_OP_MUL,
    LANCIUS_OP_MATMUL, LANCIUS_OP_RELU, LANCIUS_OP_SOFTMAX, LANCIUS_OP_SUM, LANCIUS_OP_BROADCAST,
    LANCIUS_OP_TRANSPOSE, LANCIUS_OP_RELU_BWD, LANCIUS_OP_SOFTMAX_BWD, LANCIUS_OP_SUM_AXIS0, LANCIUS_OP_SUM_AXIS1,
    LANCIUS_OP_CONV2D, LANCIUS_OP_MAXPOOL2D, LANCIUS_OP_FLATTEN, LANCIUS_OP_CONV2D_RELU_FUSED,
    LANCIUS_OP_CROSS_ENTROPY, LANCIUS_OP_CROSS_ENTROPY_BWD, LANCIUS_OP_PERMUTE, LANCIUS_OP_MATMUL_BATCHED,
    LANCIUS_OP_CONV2D_BWD, LANCIUS_OP_CONV2D_BWD_W, LANCIUS_OP_MAXPOOL2D_BWD, LANCIUS_OP_RESHAPE,
    LANCIUS_OP_EMBEDDING, LANCIUS_OP_LAYERNORM, LANCIUS_OP_GELU, LANCIUS_OP_ROPE,
    LANCIUS_OP_ATTENTION, LANCIUS_OP_KV_CACHE_READ, LANCIUS_OP_KV_CACHE_WRITE,
    LANCIUS_OP_RMSNORM,
    LANCIUS_OP_SWIGLU,
    LANCIUS_OP_GQA,
    LANCIUS_OP_TANH          /* extension: BASIS TANH lowering target */
} lancius_opcode;

typedef struct lancius_node {
    uint32_t id;
    lancius_opcode op;
    size_t shape[4];
    uint8_t ndim;
    uint32_t kernel_h, kernel_w, stride, pad;
    uint32_t axes[4];
    const struct lancius_node** inputs;
    uint32_t input_count;
    double attr_val;
    double* runtime_data;          /* host FP64 data (INPUT binding / CPU results) */
    lancius_dtype dtype;
    double scale;
    int8_t* runtime_data_int8;
    lancius_runtime_state* rt;
    uint8_t is_view;
    size_t strides[4];
    const struct lancius_node* view_source;
} lancius_node;

typedef struct lancius_graph {
    lancius_arena* arena;
    lancius_node** nodes;
    uint32_t node_count, node_cap, next_id;
    lancius_runtime_state* rt_states;
    size_t rt_cap;
} lancius_graph;

static inline size_t lancius_node_elements(const lancius_node* n) {
    size_t e = 1;
    for (uint8_t i = 0; i < n->ndim; i++) e *= n->shape[i];
    return e;
}
static inline size_t lancius_node_element_bytes(const lancius_node* n) {
    return lancius_dtype_size(n ? n->dtype : LANCIUS_DTYPE_FP64);
}
static inline size_t lancius_node_bytes(const lancius_node* n) {
    return n ? lancius_node_elements(n) * lancius_node_element_bytes(n) : 0;
}

lancius_graph* lancius_graph_create(void);
void lancius_graph_destroy(lancius_graph* g);

lancius_node* lancius_input(lancius_graph* g, size_t r, size_t c);
lancius_node* lancius_input_4d(lancius_graph* g, size_t n, size_t c, size_t h, size_t w);
lancius_node* lancius_const(lancius_graph* g, double val, size_t r, size_t c);
lancius_node* lancius_add(lancius_graph* g, const lancius_node* a, const lancius_node* b);
lancius_node* lancius_sub(lancius_graph* g, const lancius_node* a, const lancius_node* b);
lancius_node* lancius_mul(lancius_graph* g, const lancius_node* a, const lancius_node* b);
lancius_node* lancius_matmul(lancius_graph* g, const lancius_node* a, const lancius_node* b);
lancius_node* lancius_relu(lancius_graph* g, const lancius_node* a);
lancius_node* lancius_softmax(lancius_graph* g, const lancius_node* a);
lancius_node* lancius_sum(lancius_graph* g, const lancius_node* a);
lancius_node* lancius_broadcast_4d(lancius_graph* g, const lancius_node* a, size_t n, size_t c, size_t h, size_t w);
lancius_node* lancius_broadcast(lancius_graph* g, const lancius_node* a, size_t r, size_t c);
lancius_node* lancius_transpose(lancius_graph* g, const lancius_node* a);
lancius_node* lancius_conv2d(lancius_graph* g, const lancius_node* in, const lancius_node* w, uint32_t stride, uint32_t pad);
lancius_node* lancius_maxpool2d(lancius_graph* g, const lancius_node* in, uint32_t kernel, uint32_t stride);
lancius_node* lancius_flatten(lancius_graph* g, const lancius_node* in);
lancius_node* lancius_relu_bwd(lancius_graph* g, const lancius_node* grad, const lancius_node* fwd_a);
lancius_node* lancius_softmax_bwd(lancius_graph* g, const lancius_node* grad, const lancius_node* fwd_y);
lancius_node* lancius_sum_axis0(lancius_graph* g, const lancius_node* a);
lancius_node* lancius_sum_axis1(lancius_graph* g, const lancius_node* a);
lancius_node* lancius_cross_entropy(lancius_graph* g, const lancius_node* logits, const lancius_node* targets);
lancius_node* lancius_permute(lancius_graph* g, const lancius_node* in, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3);
lancius_node* lancius_matmul_batched(lancius_graph* g, const lancius_node* a, const lancius_node* b);
lancius_node* lancius_cross_entropy_bwd(lancius_graph* g, const lancius_node* logits, const lancius_node* targets, const lancius_node* grad_out);
lancius_node* lancius_conv2d_bwd(lancius_graph* g, const lancius_node* grad, const lancius_node* fwd_in, const lancius_node* fwd_w, uint32_t stride, uint32_t pad);
lancius_node* lancius_reshape(lancius_graph* g, const lancius_node* in, uint8_t ndim, size_t s0, size_t s1, size_t s2, size_t s3);
lancius_node* lancius_conv2d_bwd_w(lancius_graph* g, const lancius_node* grad, const lancius_node* fwd_in, uint32_t k_h, uint32_t k_w, uint32_t stride, uint32_t pad);
lancius_node* lancius_maxpool2d_bwd(lancius_graph* g, const lancius_node* grad, const lancius_node* fwd_in, uint32_t kernel, uint32_t stride);

void lancius_optimize_fusion(lancius_graph* g);

/* .lancius v1 files (reference lancius_serialize.c:13-259); the loader also reads the
 * older record layout without the is_view byte (stable/v9S files). */
void lancius_graph_save(lancius_graph* g, const char* path);
lancius_graph* lancius_graph_load(const char* path);

lancius_node* lancius_attention(lancius_graph* g, const lancius_node* q, const lancius_node* k, const lancius_node* v);
lancius_node* lancius_attention_noncausal(lancius_graph* g, const lancius_node* q, const lancius_node* k, const lancius_node* v);
lancius_node* lancius_layernorm(lancius_graph* g, const lancius_node* in, const lancius_node* gamma, const lancius_node* beta);
lancius_node* lancius_gelu(lancius_graph* g, const lancius_node* in);
lancius_node* lancius_tanh(lancius_graph* g, const lancius_node* in);
lancius_node* lancius_rmsnorm(lancius_graph* g, const lancius_node* in, const lancius_node* gamma);
lancius_node* lancius_swiglu(lancius_graph* g, const lancius_node* gate, const lancius_node* up);
lancius_node* lancius_gqa(lancius_graph* g, const lancius_node* q, const lancius_node* k, const lancius_node* v, uint32_t n_heads_q, uint32_t n_heads_kv);

lancius_runtime_state* lancius_graph_runtime(lancius_graph* g, uint32_t node_id);
lancius_runtime_state* lancius_node_rt(const lancius_node* n);
void lancius_runtime_sync_from_legacy(lancius_node* n);
void lancius_runtime_sync_to_legacy(lancius_node* n);
void lancius_graph_sync_runtime_to_legacy(lancius_graph* g);
void lancius_node_set_owner(lancius_node* n, lancius_memory_owner owner);
lancius_memory_owner lancius_node_get_owner(const lancius_node* n);
void lancius_node_bind_external(lancius_node* n, void* data);
void lancius_node_bind_external_int8(lancius_node* n, int8_t* data);
void lancius_node_bind_owned_heap(lancius_node* n, void* data);
void lancius_node_bind_owned_heap_int8(lancius_node* n, int8_t* data);
void lancius_node_release_owned(lancius_node* n);
void lancius_graph_release_owned(lancius_graph* g);

#ifdef __cplusplus
}
#endif
#endif

/*
 * Graph construction with shape inference. Every builder reproduces the output
 * shape, attribute placement and NULL-on-invalid behaviour of the reference
 * builder cited beside it (bleeding/v11A1/src/ir/lancius_ir.c), so graphs built
 * here and graphs built with the reference are structurally identical.
 */
#include "lancius/lancius_ir.h"
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define NODE_TABLE_INIT 1024u

static int grow_rt(lancius_graph* g, uint32_t id) {
    if (id < g->rt_cap) return 1;
    size_t cap = g->rt_cap ? g->rt_cap : NODE_TABLE_INIT;
    while (cap <= id) cap *= 2;
    lancius_runtime_state* t = (lancius_runtime_state*)realloc(g->rt_states, cap * sizeof(*t));
    if (!t) return 0;
    memset(t + g->rt_cap, 0, (cap - g->rt_cap) * sizeof(*t));
    /* existing nodes keep pointing into the table: re-point them */
    for (uint32_t i = 0; i < g->node_count; i++)
        if (g->nodes[i]->rt) g->nodes[i]->rt = &t[g->nodes[i]->id];
    g->rt_states = t; g->rt_cap = cap;
    return 1;
}

/* lancius_ir.c:107-143 */
static lancius_node* new_node(lancius_graph* g, lancius_opcode op, uint8_t ndim, uint32_t nin) {
    if (!g) { lancius_set_error(LANCIUS_ERROR_NULL_PTR); return NULL; }
    lancius_node* n = (lancius_node*)lancius_arena_alloc(g->arena, sizeof(lancius_node), 8);
    if (!n) { lancius_set_error(LANCIUS_ERROR_OOM); return NULL; }
    memset(n, 0, sizeof(*n));
    n->id = g->next_id++;
    n->op = op; n->ndim = ndim; n->input_count = nin;
    if (nin) {
        n->inputs = (const lancius_node**)lancius_arena_alloc(g->arena, nin * sizeof(lancius_node*), 8);
        if (!n->inputs) { lancius_set_error(LANCIUS_ERROR_OOM); return NULL; }
    }
    if (grow_rt(g, n->id)) {
        lancius_runtime_state* rt = &g->rt_states[n->id];
        memset(rt, 0, sizeof(*rt));
        rt->dtype = LANCIUS_DTYPE_FP64; rt->scale = 1.0;
        n->rt = rt;
    }
    if (g->node_count == g->node_cap) {
        uint32_t cap = g->node_cap ? g->node_cap * 2 : NODE_TABLE_INIT;
        lancius_node** t = (lancius_node**)realloc(g->nodes, cap * sizeof(*t));
        if (!t) { lancius_set_error(LANCIUS_ERROR_OOM); return NULL; }
        g->nodes = t; g->node_cap = cap;
    }
    g->nodes[g->node_count++] = n;
    return n;
}

static void same_shape(lancius_node* n, const lancius_node* like) {
    memcpy(n->shape, like->shape, sizeof(size_t) * like->ndim);
}

lancius_graph* lancius_graph_create(void) {
    lancius_graph* g = (lancius_graph*)calloc(1, sizeof(*g));
    if (!g) goto oom;
    g->arena = lancius_arena_create((size_t)16 << 20);
    g->node_cap = NODE_TABLE_INIT;
    g->nodes = (lancius_node**)malloc(g->node_cap * sizeof(lancius_node*));
    g->rt_cap = NODE_TABLE_INIT;
    g->rt_states = (lancius_runtime_state*)calloc(g->rt_cap, sizeof(lancius_runtime_state));
    if (!g->arena || !g->nodes || !g->rt_states) { lancius_graph_destroy(g); goto oom; }
    return g;
oom:
    lancius_set_error(LANCIUS_ERROR_OOM);
    return NULL;
}

void lancius_graph_destroy(lancius_graph* g) {
    if (!g) return;
    free(g->nodes); free(g->rt_states);
    lancius_arena_destroy(g->arena);
    free(g);
}

/* :145-156 */
lancius_node* lancius_input(lancius_graph* g, size_t r, size_t c) {
    lancius_node* n = new_node(g, LANCIUS_OP_INPUT, 2, 0);
    if (n) { n->shape[0] = r; n->shape[1] = c; }
    return n;
}
lancius_node* lancius_input_4d(lancius_graph* g, size_t nb, size_t c, size_t h, size_t w) {
    lancius_node* n = new_node(g, LANCIUS_OP_INPUT, 4, 0);
    if (n) { n->shape[0] = nb; n->shape[1] = c; n->shape[2] = h; n->shape[3] = w; }
    return n;
}
lancius_node* lancius_const(lancius_graph* g, double val, size_t r, size_t c) {
    lancius_node* n = new_node(g, LANCIUS_OP_CONST, 2, 0);
    if (n) { n->shape[0] = r; n->shape[1] = c; n->attr_val = val; }
    return n;
}

/* elementwise binaries take a's shape, no broadcasting checks (:157-177) */
static lancius_node* binary(lancius_graph* g, lancius_opcode op, const lancius_node* a, const lancius_node* b) {
    if (!a || !b) { fprintf(stderr, "[LANCIUS IR] binary op with NULL input\n"); return NULL; }
    lancius_node* n = new_node(g, op, a->ndim, 2);
    if (n) { same_shape(n, a); n->inputs[0] = a; n->inputs[1] = b; }
    return n;
}
lancius_node* lancius_add(lancius_graph* g, const lancius_node* a, const lancius_node* b) { return binary(g, LANCIUS_OP_ADD, a, b); }
lancius_node* lancius_sub(lancius_graph* g, const lancius_node* a, const lancius_node* b) { return binary(g, LANCIUS_OP_SUB, a, b); }
lancius_node* lancius_mul(lancius_graph* g, const lancius_node* a, const lancius_node* b) { return binary(g, LANCIUS_OP_MUL, a, b); }

static lancius_node* unary(lancius_graph* g, lancius_opcode op, const lancius_node* a) {
    if (!a) return NULL;
    lancius_node* n = new_node(g, op, a->ndim, 1);
    if (n) { same_shape(n, a); n->inputs[0] = a; }
    return n;
}

/* :178-196: the last two dims of each operand are the matrix */
lancius_node* lancius_matmul(lancius_graph* g, const lancius_node* a, const lancius_node* b) {
    if (!a || !b || a->ndim < 2 || b->ndim < 2) {
        fprintf(stderr, "[LANCIUS IR] MATMUL needs two operands of rank >= 2\n");
        return NULL;
    }
    size_t m = a->shape[a->ndim - 2], k = a->shape[a->ndim - 1];
    size_t kb = b->shape[b->ndim - 2], nn = b->shape[b->ndim - 1];
    if (k != kb) {
        fprintf(stderr, "[LANCIUS IR] MATMUL inner dims differ: [%zux%zu] x [%zux%zu]\n", m, k, kb, nn);
        return NULL;
    }
    lancius_node* n = new_node(g, LANCIUS_OP_MATMUL, 2, 2);
    if (n) { n->shape[0] = m; n->shape[1] = nn; n->inputs[0] = a; n->inputs[1] = b; }
    return n;
}
lancius_node* lancius_relu(lancius_graph* g, const lancius_node* a) { return unary(g, LANCIUS_OP_RELU, a); }
lancius_node* lancius_gelu(lancius_graph* g, const lancius_node* a) { return unary(g, LANCIUS_OP_GELU, a); }
lancius_node* lancius_tanh(lancius_graph* g, const lancius_node* a) { return unary(g, LANCIUS_OP_TANH, a); }
lancius_node* lancius_softmax(lancius_graph* g, const lancius_node* a) {
    if (!a || a->ndim != 2) return NULL;
    return unary(g, LANCIUS_OP_SOFTMAX, a);
}
lancius_node* lancius_sum(lancius_graph* g, const lancius_node* a) {
    if (!a) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_SUM, 2, 1);
    if (n) { n->shape[0] = 1; n->shape[1] = 1; n->inputs[0] = a; }
    return n;
}
lancius_node* lancius_broadcast(lancius_graph* g, const lancius_node* a, size_t r, size_t c) {
    if (!a) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_BROADCAST, 2, 1);
    if (n) { n->shape[0] = r; n->shape[1] = c; n->inputs[0] = a; }
    return n;
}
lancius_node* lancius_broadcast_4d(lancius_graph* g, const lancius_node* a, size_t nb, size_t c, size_t h, size_t w) {
    if (!a) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_BROADCAST, 4, 1);
    if (n) { n->shape[0] = nb; n->shape[1] = c; n->shape[2] = h; n->shape[3] = w; n->inputs[0] = a; }
    return n;
}
lancius_node* lancius_transpose(lancius_graph* g, const lancius_node* a) {
    if (!a || a->ndim != 2) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_TRANSPOSE, 2, 1);
    if (n) { n->shape[0] = a->shape[1]; n->shape[1] = a->shape[0]; n->inputs[0] = a; }
    return n;
}
lancius_node* lancius_relu_bwd(lancius_graph* g, const lancius_node* grad, const lancius_node* fwd) {
    if (!grad || !fwd) return NULL;
    return binary(g, LANCIUS_OP_RELU_BWD, grad, fwd);
}
lancius_node* lancius_softmax_bwd(lancius_graph* g, const lancius_node* grad, const lancius_node* fwd_y) {
    if (!grad || !fwd_y) return NULL;
    return binary(g, LANCIUS_OP_SOFTMAX_BWD, grad, fwd_y);
}
lancius_node* lancius_sum_axis0(lancius_graph* g, const lancius_node* a) {
    if (!a || a->ndim != 2) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_SUM_AXIS0, 2, 1);
    if (n) { n->shape[0] = 1; n->shape[1] = a->shape[1]; n->inputs[0] = a; }
    return n;
}
lancius_node* lancius_sum_axis1(lancius_graph* g, const lancius_node* a) {
    if (!a || a->ndim != 2) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_SUM_AXIS1, 2, 1);
    if (n) { n->shape[0] = a->shape[0]; n->shape[1] = 1; n->inputs[0] = a; }
    return n;
}

/* :243-261: out = [N, C_out, (H+2p-Kh)/s+1, (W+2p-Kw)/s+1] */
lancius_node* lancius_conv2d(lancius_graph* g, const lancius_node* in, const lancius_node* w, uint32_t stride, uint32_t pad) {
    if (!in || !w || in->ndim != 4 || w->ndim != 4) { fprintf(stderr, "[LANCIUS IR] CONV2D needs rank-4 input and weight\n"); return NULL; }
    if (in->shape[1] != w->shape[1]) { fprintf(stderr, "[LANCIUS IR] CONV2D channel mismatch %zu vs %zu\n", in->shape[1], w->shape[1]); return NULL; }
    size_t kh = w->shape[2], kw = w->shape[3];
    if (in->shape[2] + 2 * (size_t)pad < kh || in->shape[3] + 2 * (size_t)pad < kw || stride == 0) {
        fprintf(stderr, "[LANCIUS IR] CONV2D window larger than padded input\n"); return NULL;
    }
    lancius_node* n = new_node(g, LANCIUS_OP_CONV2D, 4, 2);
    if (!n) return NULL;
    n->shape[0] = in->shape[0]; n->shape[1] = w->shape[0];
    n->shape[2] = (in->shape[2] + 2 * (size_t)pad - kh) / stride + 1;
    n->shape[3] = (in->shape[3] + 2 * (size_t)pad - kw) / stride + 1;
    n->kernel_h = (uint32_t)kh; n->kernel_w = (uint32_t)kw; n->stride = stride; n->pad = pad;
    n->inputs[0] = in; n->inputs[1] = w;
    return n;
}

/* :263-279 */
lancius_node* lancius_maxpool2d(lancius_graph* g, const lancius_node* in, uint32_t kernel, uint32_t stride) {
    if (!in || in->ndim != 4) return NULL;
    if (in->shape[2] < kernel || in->shape[3] < kernel || stride == 0) {
        fprintf(stderr, "[LANCIUS IR] MAXPOOL2D window larger than input\n"); return NULL;
    }
    lancius_node* n = new_node(g, LANCIUS_OP_MAXPOOL2D, 4, 1);
    if (!n) return NULL;
    n->shape[0] = in->shape[0]; n->shape[1] = in->shape[1];
    n->shape[2] = (in->shape[2] - kernel) / stride + 1;
    n->shape[3] = (in->shape[3] - kernel) / stride + 1;
    n->kernel_h = n->kernel_w = kernel; n->stride = stride;
    n->inputs[0] = in;
    return n;
}

lancius_node* lancius_flatten(lancius_graph* g, const lancius_node* in) {
    if (!in || in->ndim != 4) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_FLATTEN, 2, 1);
    if (n) { n->shape[0] = in->shape[0]; n->shape[1] = in->shape[1] * in->shape[2] * in->shape[3]; n->inputs[0] = in; }
    return n;
}

/* :291-299 */
lancius_node* lancius_reshape(lancius_graph* g, const lancius_node* in, uint8_t ndim, size_t s0, size_t s1, size_t s2, size_t s3) {
    if (!in) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_RESHAPE, ndim, 1);
    if (!n) return NULL;
    size_t s[4] = { s0, s1, s2, s3 };
    for (uint8_t i = 0; i < ndim && i < 4; i++) n->shape[i] = s[i];
    n->inputs[0] = in;
    return n;
}

lancius_node* lancius_conv2d_bwd_w(lancius_graph* g, const lancius_node* grad, const lancius_node* fwd_in, uint32_t k_h, uint32_t k_w, uint32_t stride, uint32_t pad) {
    if (!grad || !fwd_in) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_CONV2D_BWD_W, 4, 2);
    if (!n) return NULL;
    n->shape[0] = grad->shape[1]; n->shape[1] = fwd_in->shape[1]; n->shape[2] = k_h; n->shape[3] = k_w;
    n->kernel_h = k_h; n->kernel_w = k_w; n->stride = stride; n->pad = pad;
    n->inputs[0] = grad; n->inputs[1] = fwd_in;
    return n;
}

lancius_node* lancius_permute(lancius_graph* g, const lancius_node* in, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3) {
    if (!in || in->ndim != 4 || a0 > 3 || a1 > 3 || a2 > 3 || a3 > 3) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_PERMUTE, 4, 1);
    if (!n) return NULL;
    uint32_t ax[4] = { a0, a1, a2, a3 };
    for (int i = 0; i < 4; i++) { n->axes[i] = ax[i]; n->shape[i] = in->shape[ax[i]]; }
    n->inputs[0] = in;
    return n;
}

lancius_node* lancius_matmul_batched(lancius_graph* g, const lancius_node* a, const lancius_node* b) {
    if (!a || !b || a->ndim != 3 || b->ndim != 3) return NULL;
    if (a->shape[0] != b->shape[0] || a->shape[2] != b->shape[1]) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_MATMUL_BATCHED, 3, 2);
    if (n) { n->shape[0] = a->shape[0]; n->shape[1] = a->shape[1]; n->shape[2] = b->shape[2]; n->inputs[0] = a; n->inputs[1] = b; }
    return n;
}

lancius_node* lancius_cross_entropy(lancius_graph* g, const lancius_node* logits, const lancius_node* targets) {
    if (!logits || !targets || logits->ndim != 2 || targets->ndim != 2) return NULL;
    if (logits->shape[0] != targets->shape[0] || logits->shape[1] != targets->shape[1]) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_CROSS_ENTROPY, 2, 2);
    if (n) { n->shape[0] = 1; n->shape[1] = 1; n->inputs[0] = logits; n->inputs[1] = targets; }
    return n;
}

lancius_node* lancius_cross_entropy_bwd(lancius_graph* g, const lancius_node* logits, const lancius_node* targets, const lancius_node* grad_out) {
    if (!logits || !targets || !grad_out) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_CROSS_ENTROPY_BWD, logits->ndim, 3);
    if (n) { same_shape(n, logits); n->inputs[0] = logits; n->inputs[1] = targets; n->inputs[2] = grad_out; }
    return n;
}

lancius_node* lancius_conv2d_bwd(lancius_graph* g, const lancius_node* grad, const lancius_node* fwd_in, const lancius_node* fwd_w, uint32_t stride, uint32_t pad) {
    if (!grad || !fwd_in || !fwd_w) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_CONV2D_BWD, 4, 3);
    if (!n) return NULL;
    memcpy(n->shape, fwd_in->shape, sizeof(size_t) * 4);
    n->stride = stride; n->pad = pad;
    n->inputs[0] = grad; n->inputs[1] = fwd_in; n->inputs[2] = fwd_w;
    return n;
}

lancius_node* lancius_maxpool2d_bwd(lancius_graph* g, const lancius_node* grad, const lancius_node* fwd_in, uint32_t kernel, uint32_t stride) {
    if (!grad || !fwd_in) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_MAXPOOL2D_BWD, 4, 2);
    if (!n) return NULL;
    memcpy(n->shape, fwd_in->shape, sizeof(size_t) * 4);
    n->kernel_h = n->kernel_w = kernel; n->stride = stride;
    n->inputs[0] = grad; n->inputs[1] = fwd_in;
    return n;
}

/* :72-77: node shape = q's [S, H, D]; attr_val 0 = causal (reference behaviour) */
lancius_node* lancius_attention(lancius_graph* g, const lancius_node* q, const lancius_node* k, const lancius_node* v) {
    if (!q || !k || !v) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_ATTENTION, 3, 3);
    if (n) { memcpy(n->shape, q->shape, sizeof(size_t) * 3); n->inputs[0] = q; n->inputs[1] = k; n->inputs[2] = v; }
    return n;
}
lancius_node* lancius_attention_noncausal(lancius_graph* g, const lancius_node* q, const lancius_node* k, const lancius_node* v) {
    lancius_node* n = lancius_attention(g, q, k, v);
    if (n) n->attr_val = 1.0;
    return n;
}

lancius_node* lancius_layernorm(lancius_graph* g, const lancius_node* in, const lancius_node* gamma, const lancius_node* beta) {
    if (!in || !gamma || !beta) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_LAYERNORM, in->ndim, 3);
    if (n) { same_shape(n, in); n->inputs[0] = in; n->inputs[1] = gamma; n->inputs[2] = beta; }
    return n;
}

lancius_node* lancius_rmsnorm(lancius_graph* g, const lancius_node* in, const lancius_node* gamma) {
    if (!in || !gamma) return NULL;
    return binary(g, LANCIUS_OP_RMSNORM, in, gamma);
}
lancius_node* lancius_swiglu(lancius_graph* g, const lancius_node* gate, const lancius_node* up) {
    if (!gate || !up) return NULL;
    return binary(g, LANCIUS_OP_SWIGLU, gate, up);
}
lancius_node* lancius_gqa(lancius_graph* g, const lancius_node* q, const lancius_node* k, const lancius_node* v, uint32_t hq, uint32_t hkv) {
    if (!q || !k || !v) return NULL;
    lancius_node* n = new_node(g, LANCIUS_OP_GQA, q->ndim, 3);
    if (n) { same_shape(n, q); n->kernel_h = hq; n->kernel_w = hkv; n->inputs[0] = q; n->inputs[1] = k; n->inputs[2] = v; }
    return n;
}

/* runtime-state / ownership helpers (:402-545) */
lancius_runtime_state* lancius_graph_runtime(lancius_graph* g, uint32_t id) {
    return (g && g->rt_states && id < g->rt_cap) ? &g->rt_states[id] : NULL;
}
lancius_runtime_state* lancius_node_rt(const lancius_node* n) { return n ? n->rt : NULL; }

void lancius_runtime_sync_from_legacy(lancius_node* n) {
    if (!n || !n->rt) return;
    n->rt->buffer = n->runtime_data; n->rt->buffer_int8 = n->runtime_data_int8;
    n->rt->dtype = n->dtype; n->rt->scale = n->scale;
}
void lancius_runtime_sync_to_legacy(lancius_node* n) {
    if (!n || !n->rt) return;
    n->runtime_data = (double*)n->rt->buffer; n->runtime_data_int8 = n->rt->buffer_int8;
    n->dtype = n->rt->dtype; n->scale = n->rt->scale;
}
void lancius_graph_sync_runtime_to_legacy(lancius_graph* g) {
    if (!g) return;
    for (uint32_t i = 0; i < g->node_count; i++) lancius_runtime_sync_to_legacy(g->nodes[i]);
}
void lancius_node_set_owner(lancius_node* n, lancius_memory_owner o) {
    if (!n || !n->rt) return;
    n->rt->owner = n->rt->buffer_owner = n->rt->int8_owner = o;
}
lancius_memory_owner lancius_node_get_owner(const lancius_node* n) {
    return (n && n->rt) ? n->rt->buffer_owner : LANCIUS_MEMORY_EXTERNAL;
}
void lancius_node_bind_external(lancius_node* n, void* data) {
    if (!n) return;
    n->runtime_data = (double*)data;
    if (n->rt) { n->rt->buffer = data; n->rt->buffer_owner = n->rt->owner = LANCIUS_MEMORY_EXTERNAL; n->rt->dtype = n->dtype; }
}
void lancius_node_bind_external_int8(lancius_node* n, int8_t* data) {
    if (!n) return;
    n->runtime_data_int8 = data;
    if (n->rt) { n->rt->buffer_int8 = data; n->rt->int8_owner = LANCIUS_MEMORY_EXTERNAL; }
}
void lancius_node_bind_owned_heap(lancius_node* n, void* data) {
    if (!n) return;
    if (!data) { lancius_node_bind_external(n, NULL); return; }
    n->runtime_data = (double*)data;
    if (n->rt) { n->rt->buffer = data; n->rt->buffer_owner = n->rt->owner = LANCIUS_MEMORY_OWNED_HEAP; n->rt->dtype = n->dtype; }
}
void lancius_node_bind_owned_heap_int8(lancius_node* n, int8_t* data) {
    if (!n) return;
    if (!data) { lancius_node_bind_external_int8(n, NULL); return; }
    n->runtime_data_int8 = data;
    if (n->rt) {
        n->rt->buffer_int8 = data; n->rt->int8_owner = LANCIUS_MEMORY_OWNED_HEAP;
        if (n->dtype == LANCIUS_DTYPE_INT8) n->rt->dtype = LANCIUS_DTYPE_INT8;
    }
}
void lancius_node_release_owned(lancius_node* n) {
    if (!n || !n->rt) return;
    if (n->rt->buffer_owner == LANCIUS_MEMORY_OWNED_HEAP && n->runtime_data) {
        free(n->runtime_data); n->runtime_data = NULL; n->rt->buffer = NULL;
        n->rt->buffer_owner = LANCIUS_MEMORY_EXTERNAL;
    }
    if (n->rt->int8_owner == LANCIUS_MEMORY_OWNED_HEAP && n->runtime_data_int8) {
        free(n->runtime_data_int8); n->runtime_data_int8 = NULL; n->rt->buffer_int8 = NULL;
        n->rt->int8_owner = LANCIUS_MEMORY_EXTERNAL;
    }
    if (n->rt->buffer_owner == LANCIUS_MEMORY_EXTERNAL && n->rt->int8_owner == LANCIUS_MEMORY_EXTERNAL)
        n->rt->owner = LANCIUS_MEMORY_EXTERNAL;
}
void lancius_graph_release_owned(lancius_graph* g) {
    if (!g) return;
    for (uint32_t i = 0; i < g->node_count; i++) lancius_node_release_owned(g->nodes[i]);
}

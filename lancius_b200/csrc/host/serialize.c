/*
 * .lancius model files (format v1 of the reference, bleeding/v11A1/src/core/lancius_serialize.c:13-63):
 *   u32 magic 0x21434E41, u32 node_count, then per node
 *   u32 id, i32 op, u8 ndim, u64 shape[4], u32 input_count, u32 input_ids[input_count],
 *   f64 attr_val, u32 meta[4] (kernel_h, kernel_w, stride, pad), u32 axes[4],
 *   u8 is_view [+ u64 strides[4], u32 view_source_id when set]      (absent in v9-era files)
 *   u8 has_weights [+ u8 dtype, f64 scale, data (int8 or f64) when set]
 * Nodes are rebuilt with the IR builders, so shapes come from shape inference as in
 * the reference loader (:132-176). The loader accepts both the current layout and the
 * older one without the is_view byte (stable/v9S files, e.g. pytorch_lenet.lancius),
 * which the reference's current loader rejects.
 */
#include "lancius/lancius_ir.h"
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define LANCIUS_MAGIC 0x21434E41u
#define MAX_NODES 1000000u
#define MAX_ELEMS 100000000u

typedef struct { const unsigned char* p; size_t n, at; int bad; } cursor;

static void rd(cursor* c, void* dst, size_t k) {
    if (c->bad || k > c->n - c->at) { c->bad = 1; memset(dst, 0, k); return; }
    memcpy(dst, c->p + c->at, k);
    c->at += k;
}

static void free_weights(lancius_graph* g) {
    for (uint32_t k = 0; k < g->node_count; k++) lancius_node_release_owned(g->nodes[k]);
}

/* one pass over the node records; with_view selects the record layout */
static lancius_graph* parse(const unsigned char* buf, size_t len, int with_view) {
    cursor c = { buf, len, 0, 0 };
    uint32_t magic = 0, count = 0;
    rd(&c, &magic, 4); rd(&c, &count, 4);
    if (c.bad || magic != LANCIUS_MAGIC || count > MAX_NODES) return NULL;
    lancius_graph* g = lancius_graph_create();
    if (!g) return NULL;
    uint32_t map_n = count + 1000;
    lancius_node** id_map = (lancius_node**)calloc(map_n, sizeof(lancius_node*));
    if (!id_map) { lancius_graph_destroy(g); return NULL; }
    for (uint32_t i = 0; i < count && !c.bad; i++) {
        uint32_t id = 0, nin = 0, ins[16] = { 0 }, meta[4], axes[4];
        int32_t op = 0;
        uint8_t ndim = 0, is_view = 0, has_w = 0;
        size_t shape[4];
        double attr = 0.0;
        rd(&c, &id, 4); rd(&c, &op, 4); rd(&c, &ndim, 1); rd(&c, shape, 32); rd(&c, &nin, 4);
        if (c.bad || id >= map_n || nin > 16 || ndim > 4) { c.bad = 1; break; }
        rd(&c, ins, 4 * (size_t)nin);
        for (uint32_t j = 0; j < nin; j++) if (ins[j] >= map_n || !id_map[ins[j]]) c.bad = 1;
        rd(&c, &attr, 8); rd(&c, meta, 16); rd(&c, axes, 16);
        size_t vstr[4] = { 0 };
        uint32_t vsrc = 0xFFFFFFFFu;
        if (with_view) {
            rd(&c, &is_view, 1);
            if (is_view) { rd(&c, vstr, 32); rd(&c, &vsrc, 4); }
        }
        rd(&c, &has_w, 1);
        if (c.bad) break;
        const lancius_node* a = nin > 0 ? id_map[ins[0]] : NULL;
        const lancius_node* b = nin > 1 ? id_map[ins[1]] : NULL;
        const lancius_node* d = nin > 2 ? id_map[ins[2]] : NULL;
        lancius_node* n = NULL;
        switch (op) {
            case LANCIUS_OP_INPUT:
                n = ndim == 4 ? lancius_input_4d(g, shape[0], shape[1], shape[2], shape[3]) : lancius_input(g, shape[0], shape[1]);
                break;
            case LANCIUS_OP_CONST: n = lancius_const(g, attr, shape[0], shape[1]); break;
            case LANCIUS_OP_ADD: n = lancius_add(g, a, b); break;
            case LANCIUS_OP_SUB: n = lancius_sub(g, a, b); break;
            case LANCIUS_OP_MUL: n = lancius_mul(g, a, b); break;
            case LANCIUS_OP_MATMUL: n = lancius_matmul(g, a, b); break;
            case LANCIUS_OP_RELU: n = lancius_relu(g, a); break;
            case LANCIUS_OP_SOFTMAX: n = lancius_softmax(g, a); break;
            case LANCIUS_OP_SUM: n = lancius_sum(g, a); break;
            case LANCIUS_OP_BROADCAST: n = a ? lancius_broadcast(g, a, shape[0], shape[1]) : NULL; break;
            case LANCIUS_OP_SUM_AXIS1: n = lancius_sum_axis1(g, a); break;
            case LANCIUS_OP_CONV2D: n = (a && b) ? lancius_conv2d(g, a, b, meta[2], meta[3]) : NULL; break;
            case LANCIUS_OP_CONV2D_RELU_FUSED:
                n = (a && b) ? lancius_conv2d(g, a, b, meta[2], meta[3]) : NULL;
                if (n) n->op = LANCIUS_OP_CONV2D_RELU_FUSED;
                break;
            case LANCIUS_OP_MAXPOOL2D: n = a ? lancius_maxpool2d(g, a, meta[0], meta[2]) : NULL; break;
            case LANCIUS_OP_FLATTEN: n = a ? lancius_flatten(g, a) : NULL; break;
            case LANCIUS_OP_RESHAPE: n = a ? lancius_reshape(g, a, ndim, shape[0], shape[1], shape[2], shape[3]) : NULL; break;
            case LANCIUS_OP_LAYERNORM: n = (a && b && d) ? lancius_layernorm(g, a, b, d) : NULL; break;
            case LANCIUS_OP_GELU: n = lancius_gelu(g, a); break;
            case LANCIUS_OP_TANH: n = lancius_tanh(g, a); break;
            case LANCIUS_OP_ATTENTION:
                n = (a && b && d) ? lancius_attention(g, a, b, d) : NULL;
                if (n) n->attr_val = attr;        /* keeps the unmasked flag across a save/load */
                break;
            case LANCIUS_OP_CROSS_ENTROPY: n = (a && b) ? lancius_cross_entropy(g, a, b) : NULL; break;
            default:
                fprintf(stderr, "[LANCIUS LOAD] op %d of node %u is not loadable, skipped\n", op, id);
                break;
        }
        if (!n) {
            if (op == LANCIUS_OP_INPUT || op == LANCIUS_OP_CONST || has_w) c.bad = 1;
            else continue;       /* like the reference: unknown ops are skipped */
            break;
        }
        n->kernel_h = meta[0]; n->kernel_w = meta[1]; n->stride = meta[2]; n->pad = meta[3];
        memcpy(n->axes, axes, sizeof(axes));
        if (is_view) {
            n->is_view = 1;
            memcpy(n->strides, vstr, sizeof(vstr));
            if (vsrc < map_n) n->view_source = id_map[vsrc];
        }
        id_map[id] = n;
        if (has_w) {
            size_t e = lancius_node_elements(n);
            uint8_t dt = 0;
            double scale = 1.0;
            rd(&c, &dt, 1); rd(&c, &scale, 8);
            if (c.bad || e > MAX_ELEMS || !lancius_dtype_is_valid(dt)) { c.bad = 1; break; }
            n->dtype = (lancius_dtype)dt;
            n->scale = scale;
            if (n->dtype == LANCIUS_DTYPE_INT8) {
                int8_t* w = (int8_t*)malloc(e ? e : 1);
                if (!w) { c.bad = 1; break; }
                rd(&c, w, e);
                lancius_node_bind_owned_heap_int8(n, w);
            } else {
                double* w = (double*)malloc((e ? e : 1) * sizeof(double));
                if (!w) { c.bad = 1; break; }
                rd(&c, w, e * sizeof(double));
                lancius_node_bind_owned_heap(n, w);
            }
        }
    }
    free(id_map);
    if (c.bad || c.at != c.n) {
        free_weights(g);
        lancius_graph_destroy(g);
        return NULL;
    }
    for (uint32_t i = 0; i < g->node_count; i++) lancius_runtime_sync_from_legacy(g->nodes[i]);
    return g;
}

lancius_graph* lancius_graph_load(const char* path) {
    FILE* f = path ? fopen(path, "rb") : NULL;
    if (!f) { lancius_set_error(LANCIUS_ERROR_IO); return NULL; }
    fseek(f, 0, SEEK_END);
    long len = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (len < 8) { fclose(f); lancius_set_error(LANCIUS_ERROR_INVALID_MODEL); return NULL; }
    unsigned char* buf = (unsigned char*)malloc((size_t)len);
    if (!buf) { fclose(f); lancius_set_error(LANCIUS_ERROR_OOM); return NULL; }
    size_t got = fread(buf, 1, (size_t)len, f);
    fclose(f);
    lancius_graph* g = got == (size_t)len ? parse(buf, got, 1) : NULL;
    if (!g && got == (size_t)len) g = parse(buf, got, 0);      /* record layout without is_view */
    free(buf);
    if (!g) lancius_set_error(LANCIUS_ERROR_INVALID_MODEL);
    return g;
}

void lancius_graph_save(lancius_graph* g, const char* path) {
    FILE* f = (g && path) ? fopen(path, "wb") : NULL;
    if (!f) { lancius_set_error(LANCIUS_ERROR_IO); return; }
    uint32_t magic = LANCIUS_MAGIC;
    fwrite(&magic, 4, 1, f);
    fwrite(&g->node_count, 4, 1, f);
    for (uint32_t i = 0; i < g->node_count; i++) {
        lancius_node* n = g->nodes[i];
        lancius_runtime_sync_from_legacy(n);
        int32_t op = (int32_t)n->op;
        fwrite(&n->id, 4, 1, f); fwrite(&op, 4, 1, f); fwrite(&n->ndim, 1, 1, f);
        fwrite(n->shape, 8, 4, f); fwrite(&n->input_count, 4, 1, f);
        for (uint32_t j = 0; j < n->input_count; j++) fwrite(&n->inputs[j]->id, 4, 1, f);
        fwrite(&n->attr_val, 8, 1, f);
        uint32_t meta[4] = { n->kernel_h, n->kernel_w, n->stride, n->pad };
        fwrite(meta, 4, 4, f); fwrite(n->axes, 4, 4, f);
        uint8_t v = n->is_view ? 1 : 0;
        fwrite(&v, 1, 1, f);
        if (v) {
            uint32_t src = n->view_source ? n->view_source->id : 0xFFFFFFFFu;
            fwrite(n->strides, 8, 4, f); fwrite(&src, 4, 1, f);
        }
        uint8_t hw = (n->op == LANCIUS_OP_INPUT && (n->runtime_data || n->runtime_data_int8)) ? 1 : 0;
        fwrite(&hw, 1, 1, f);
        if (hw) {
            size_t e = lancius_node_elements(n);
            uint8_t dt = lancius_dtype_is_valid((uint8_t)n->dtype) ? (uint8_t)n->dtype : 0;
            fwrite(&dt, 1, 1, f); fwrite(&n->scale, 8, 1, f);
            if (dt == LANCIUS_DTYPE_INT8) fwrite(n->runtime_data_int8, 1, e, f);
            else fwrite(n->runtime_data, 8, e, f);
        }
    }
    fclose(f);
}

/* A Lancius host program written against the reference's public headers only
 * (lancius_ir.h, lancius_scheduler.h, lancius_arena.h, lancius_threadpool.h,
 * lancius_stable_api.h, lancius_optimizer's fusion pass, lancius_graph_load) and
 * linked against liblancius_b200.so instead of the reference library: the same calls
 * now run on the GPU. Used by tests/test_gpu_dropin.py.
 *
 *   dropin_main stable <x> <w1> <w2> <h_out> <y_out>
 *       stable FFI: y = relu(x @ w1) @ w2 (x 64x784, w1 784x256, w2 256x10);
 *       lancius_compile_and_run twice, lancius_read_output of h and y
 *   dropin_main arena <x> <w1> <b1> <w2> <b2> <out>
 *       config-1 MLP through the IR builders; lancius_schedule_execute, then the same
 *       graph with a rebuilt schedule, then lancius_schedule_execute_parallel
 *       (all three outputs written one after another)
 *   dropin_main static <model.lancius> <image f32> <out>
 *       examples/run_edge.c's flow: load, fuse, schedule, lancius_schedule_execute_static
 *
 * Array files are raw little-endian doubles (the image: float32, as the reference ships it).
 */
#include "lancius/lancius_arena.h"
#include "lancius/lancius_error.h"
#include "lancius/lancius_ir.h"
#include "lancius/lancius_scheduler.h"
#include "lancius/lancius_stable_api.h"
#include "lancius/lancius_threadpool.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static double* read_f64(const char* path, size_t n) {
    double* p = (double*)malloc(n * sizeof(double));
    FILE* f = fopen(path, "rb");
    if (!p || !f || fread(p, sizeof(double), n, f) != n) { fprintf(stderr, "read %s failed\n", path); exit(2); }
    fclose(f);
    return p;
}

static void append_f64(const char* path, const double* p, size_t n, const char* mode) {
    FILE* f = fopen(path, mode);
    if (!f || fwrite(p, sizeof(double), n, f) != n) { fprintf(stderr, "write %s failed\n", path); exit(2); }
    fclose(f);
}

static int check(const char* what) {
    if (lancius_get_error() != LANCIUS_ERROR_OK) {
        fprintf(stderr, "%s: lancius error %d (%s)\n", what, lancius_get_error(), lancius_error_string(lancius_get_error()));
        exit(3);
    }
    return 0;
}

static int run_stable(char** a) {
    const size_t B = 64, IN = 784, H = 256, O = 10;
    double *x = read_f64(a[0], B * IN), *w1 = read_f64(a[1], IN * H), *w2 = read_f64(a[2], H * O);
    lancius_context ctx = lancius_create_context();
    lancius_graph_handle g = lancius_graph_create_stable(ctx);
    lancius_tensor_handle tx = lancius_add_input(g, B, IN), tw1 = lancius_add_input(g, IN, H),
                          tw2 = lancius_add_input(g, H, O);
    lancius_tensor_handle th = lancius_add_relu(g, lancius_add_matmul(g, tx, tw1));
    lancius_tensor_handle ty = lancius_add_matmul(g, th, tw2);
    if (!th || !ty) { fprintf(stderr, "build: %s\n", lancius_get_error_string(lancius_get_last_error())); return 3; }
    lancius_bind_data(tx, x);
    lancius_bind_data(tw1, w1);
    lancius_bind_data(tw2, w2);
    double* h = (double*)malloc(B * H * sizeof(double));
    double* y = (double*)malloc(B * O * sizeof(double));
    for (int run = 0; run < 2; run++) {
        lancius_status s = lancius_compile_and_run(g);
        if (s != LANCIUS_OK) { fprintf(stderr, "compile_and_run: %s\n", lancius_get_error_string(s)); return 3; }
        if (lancius_read_output(th, h, B * H * sizeof(double)) != LANCIUS_OK ||
            lancius_read_output(ty, y, B * O * sizeof(double)) != LANCIUS_OK) return 3;
    }
    append_f64(a[3], h, B * H, "wb");
    append_f64(a[4], y, B * O, "wb");
    if (lancius_tensor_get_dtype(ty) != LANCIUS_DTYPE_FP64) return 4;
    lancius_graph_destroy_stable(g);
    lancius_destroy_context(ctx);
    lancius_dropin_release();
    printf("stable ok\n");
    return 0;
}

static int run_arena(char** a) {
    const size_t B = 64, IN = 784, H = 256, O = 10;
    lancius_graph* g = lancius_graph_create();
    lancius_node *x = lancius_input(g, B, IN), *w1 = lancius_input(g, IN, H), *b1 = lancius_input(g, 1, H);
    lancius_node *w2 = lancius_input(g, H, O), *b2 = lancius_input(g, 1, O);
    lancius_node* h = lancius_relu(g, lancius_add(g, lancius_matmul(g, x, w1), lancius_broadcast(g, b1, B, H)));
    lancius_node* y = lancius_softmax(g, lancius_add(g, lancius_matmul(g, h, w2), lancius_broadcast(g, b2, B, O)));
    check("build");
    x->runtime_data = read_f64(a[0], B * IN);
    w1->runtime_data = read_f64(a[1], IN * H);
    b1->runtime_data = read_f64(a[2], H);
    w2->runtime_data = read_f64(a[3], H * O);
    b2->runtime_data = read_f64(a[4], O);
    lancius_arena* arena = lancius_arena_create(16u << 20);

    lancius_schedule* s = lancius_ir_schedule(g);
    lancius_schedule_execute(s, arena);
    check("lancius_schedule_execute");
    append_f64(a[5], y->runtime_data, B * O, "wb");

    /* a caller that rebuilds its schedule keeps its nodes' runtime_data: same buffers */
    lancius_schedule_destroy(s);
    memset(y->runtime_data, 0, B * O * sizeof(double));
    s = lancius_ir_schedule(g);
    lancius_schedule_execute(s, arena);
    check("lancius_schedule_execute (rebuilt schedule)");
    append_f64(a[5], y->runtime_data, B * O, "ab");

    lancius_pool* pool = lancius_pool_create(4);
    memset(y->runtime_data, 0, B * O * sizeof(double));
    lancius_schedule_execute_parallel(s, arena, pool);
    check("lancius_schedule_execute_parallel");
    append_f64(a[5], y->runtime_data, B * O, "ab");
    lancius_pool_destroy(pool);

    lancius_schedule_destroy(s);
    lancius_arena_destroy(arena);
    lancius_dropin_release();
    printf("arena ok\n");
    return 0;
}

static int run_static(char** a) {
    lancius_graph* g = lancius_graph_load(a[0]);
    if (!g) { fprintf(stderr, "load failed: %d\n", lancius_get_error()); return 3; }
    lancius_optimize_fusion(g);
    lancius_schedule* s = lancius_ir_schedule(g);
    lancius_node *in = NULL, *out = NULL;
    size_t total = 0;
    for (uint32_t i = 0; i < g->node_count; i++) {
        lancius_node* n = g->nodes[i];
        if (n->op == LANCIUS_OP_INPUT && n->ndim == 4 && n->shape[1] == 3 && !n->runtime_data) in = n;
        if (n->ndim == 2 && n->shape[1] == 10 && n->op != LANCIUS_OP_INPUT) out = n;
        total += lancius_node_bytes(n) + 32;
    }
    if (!in || !out) { fprintf(stderr, "input/output not found\n"); return 3; }
    size_t e = lancius_node_elements(in);
    float* img = (float*)malloc(e * sizeof(float));
    FILE* f = fopen(a[1], "rb");
    if (!f || fread(img, sizeof(float), e, f) != e) { fprintf(stderr, "read image failed\n"); return 2; }
    fclose(f);
    in->runtime_data = (double*)malloc(e * sizeof(double));
    for (size_t i = 0; i < e; i++) in->runtime_data[i] = img[i];
    void* flat = malloc(total);
    lancius_schedule_execute_static(s, flat);
    check("lancius_schedule_execute_static");
    if ((char*)out->runtime_data < (char*)flat || (char*)out->runtime_data >= (char*)flat + total) return 5;
    append_f64(a[2], out->runtime_data, lancius_node_elements(out), "wb");
    lancius_dropin_release();
    printf("static ok\n");
    return 0;
}

int main(int argc, char** argv) {
    if (argc >= 7 && !strcmp(argv[1], "stable")) return run_stable(argv + 2);
    if (argc >= 8 && !strcmp(argv[1], "arena")) return run_arena(argv + 2);
    if (argc >= 5 && !strcmp(argv[1], "static")) return run_static(argv + 2);
    fprintf(stderr, "usage: dropin_main stable|arena|static ...\n");
    return 1;
}

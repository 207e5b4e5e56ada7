/* The reference's stable FFI (bleeding/v11A1/src/core/lancius_stable_api.c:9-160):
 * opaque handles over the IR, a thread-local status, and compile_and_run = schedule +
 * lancius_schedule_execute -- which in this library runs the graph on the GPU and
 * copies the FP64 results back into the nodes' host buffers, so lancius_read_output
 * reads them as the reference does. Status codes and the messages' meaning are the
 * reference's. */
#include "lancius/lancius_stable_api.h"
#include "lancius/lancius_arena.h"
#include "lancius/lancius_error.h"
#include "lancius/lancius_ir.h"
#include "lancius/lancius_scheduler.h"

#include <stdlib.h>
#include <string.h>

static _Thread_local lancius_status tl_status = LANCIUS_OK;

/* dropin.cu: makes this thread's next executor runs copy every computed node back */
void lcu_dropin_force_all(int on);

static lancius_status status(lancius_status s) { tl_status = s; return s; }

LANCIUS_EXPORT lancius_status lancius_get_last_error(void) { return tl_status; }

LANCIUS_EXPORT const char* lancius_get_error_string(lancius_status err) {
    switch (err) {
        case LANCIUS_OK: return "Success";
        case LANCIUS_ERR_OOM: return "Out of Memory";
        case LANCIUS_ERR_SHAPE_MISMATCH: return "Shape Mismatch";
        case LANCIUS_ERR_NULL_PTR: return "Null Pointer";
        case LANCIUS_ERR_UNSUPPORTED_OP: return "Unsupported Operation";
    }
    return "Unknown Error";
}

typedef struct { lancius_arena* arena; } stable_ctx;
/* a graph handle carries what its runs need: the host arena the executor places
 * results in, and the schedule of the last run */
typedef struct { lancius_graph* g; lancius_arena* scratch; lancius_schedule* sched; } stable_graph;

LANCIUS_EXPORT lancius_context lancius_create_context(void) {
    stable_ctx* c = (stable_ctx*)calloc(1, sizeof(*c));
    if (!c || !(c->arena = lancius_arena_create(64u << 20))) { free(c); status(LANCIUS_ERR_OOM); return NULL; }
    status(LANCIUS_OK);
    return c;
}

LANCIUS_EXPORT void lancius_destroy_context(lancius_context ctx) {
    stable_ctx* c = (stable_ctx*)ctx;
    if (!c) return;
    lancius_arena_destroy(c->arena);
    free(c);
}

LANCIUS_EXPORT lancius_graph_handle lancius_graph_create_stable(lancius_context ctx) {
    if (!ctx) { status(LANCIUS_ERR_NULL_PTR); return NULL; }
    stable_graph* w = (stable_graph*)calloc(1, sizeof(*w));
    if (!w) { status(LANCIUS_ERR_OOM); return NULL; }
    w->g = lancius_graph_create();
    w->scratch = lancius_arena_create(16u << 20);
    if (!w->g || !w->scratch) {
        if (w->g) lancius_graph_destroy(w->g);
        if (w->scratch) lancius_arena_destroy(w->scratch);
        free(w);
        status(LANCIUS_ERR_OOM);
        return NULL;
    }
    status(LANCIUS_OK);
    return w;
}

LANCIUS_EXPORT void lancius_graph_destroy_stable(lancius_graph_handle h) {
    stable_graph* w = (stable_graph*)h;
    if (!w) return;
    if (w->sched) lancius_schedule_destroy(w->sched);
    lancius_arena_destroy(w->scratch);
    lancius_graph_destroy(w->g);
    free(w);
}

static lancius_tensor_handle made(lancius_node* n, lancius_status on_fail) {
    status(n ? LANCIUS_OK : on_fail);
    return n;
}

LANCIUS_EXPORT lancius_tensor_handle lancius_add_input(lancius_graph_handle h, size_t rows, size_t cols) {
    if (!h) { status(LANCIUS_ERR_NULL_PTR); return NULL; }
    return made(lancius_input(((stable_graph*)h)->g, rows, cols), LANCIUS_ERR_OOM);
}

LANCIUS_EXPORT lancius_tensor_handle lancius_add_matmul(lancius_graph_handle h, lancius_tensor_handle a,
                                                        lancius_tensor_handle b) {
    if (!h || !a || !b) { status(LANCIUS_ERR_NULL_PTR); return NULL; }
    return made(lancius_matmul(((stable_graph*)h)->g, (lancius_node*)a, (lancius_node*)b), LANCIUS_ERR_SHAPE_MISMATCH);
}

LANCIUS_EXPORT lancius_tensor_handle lancius_add_relu(lancius_graph_handle h, lancius_tensor_handle a) {
    if (!h || !a) { status(LANCIUS_ERR_NULL_PTR); return NULL; }
    return made(lancius_relu(((stable_graph*)h)->g, (lancius_node*)a), LANCIUS_ERR_OOM);
}

LANCIUS_EXPORT lancius_status lancius_bind_data(lancius_tensor_handle t, double* data) {
    if (!t || !data) return status(LANCIUS_ERR_NULL_PTR);
    lancius_node_bind_external((lancius_node*)t, data);   /* caller keeps ownership */
    return status(LANCIUS_OK);
}

LANCIUS_EXPORT lancius_status lancius_compile_and_run(lancius_graph_handle h) {
    stable_graph* w = (stable_graph*)h;
    if (!w) return status(LANCIUS_ERR_NULL_PTR);
    if (w->sched) lancius_schedule_destroy(w->sched);
    w->sched = lancius_ir_schedule(w->g);
    if (!w->sched) return status(LANCIUS_ERR_OOM);
    lancius_arena_reset(w->scratch);
    lancius_clear_error();
    /* any tensor may be read afterwards (lancius_read_output): copy every node back */
    lcu_dropin_force_all(1);
    lancius_schedule_execute(w->sched, w->scratch);
    lcu_dropin_force_all(0);
    /* the device path reports through the IR's thread-local error; fold it into the
     * stable status set (the reference's executor cannot fail past OOM) */
    switch (lancius_get_error()) {
        case LANCIUS_ERROR_OK: return status(LANCIUS_OK);
        case LANCIUS_ERROR_OOM: return status(LANCIUS_ERR_OOM);
        case LANCIUS_ERROR_SHAPE_MISMATCH: return status(LANCIUS_ERR_SHAPE_MISMATCH);
        case LANCIUS_ERROR_NULL_PTR: return status(LANCIUS_ERR_NULL_PTR);
        default: return status(LANCIUS_ERR_UNSUPPORTED_OP);
    }
}

LANCIUS_EXPORT lancius_status lancius_read_output(lancius_tensor_handle t, double* out, size_t bytes) {
    if (!t || !out) return status(LANCIUS_ERR_NULL_PTR);
    const lancius_node* n = (const lancius_node*)t;
    if (!n->runtime_data) return status(LANCIUS_ERR_NULL_PTR);
    if (bytes % sizeof(double)) return status(LANCIUS_ERR_SHAPE_MISMATCH);
    size_t e = lancius_node_elements(n), cap = bytes / sizeof(double);
    memcpy(out, n->runtime_data, (e < cap ? e : cap) * sizeof(double));
    return status(LANCIUS_OK);
}

LANCIUS_EXPORT int lancius_tensor_get_dtype(lancius_tensor_handle t) {
    if (!t) { status(LANCIUS_ERR_NULL_PTR); return -1; }
    status(LANCIUS_OK);
    return (int)((const lancius_node*)t)->dtype;
}

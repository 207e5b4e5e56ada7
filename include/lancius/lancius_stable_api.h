/*
 * lancius_stable_api.h -- the reference's FFI surface (opaque handles, thread-local
 * status), same names, codes and signatures as
 * bleeding/v11A1/include/lancius/lancius_stable_api.h:20-60. Here
 * lancius_compile_and_run executes the graph on the GPU (lancius_schedule_execute of
 * this library) and lancius_read_output returns the FP64 result copied back to the host.
 */
#ifndef LANCIUS_STABLE_API_H
#define LANCIUS_STABLE_API_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LANCIUS_EXPORT __attribute__((visibility("default")))

typedef void* lancius_context;
typedef void* lancius_graph_handle;
typedef void* lancius_tensor_handle;

typedef enum {
    LANCIUS_OK = 0,
    LANCIUS_ERR_OOM = -1,
    LANCIUS_ERR_SHAPE_MISMATCH = -2,
    LANCIUS_ERR_NULL_PTR = -3,
    LANCIUS_ERR_UNSUPPORTED_OP = -4
} lancius_status;

LANCIUS_EXPORT lancius_status lancius_get_last_error(void);
LANCIUS_EXPORT const char* lancius_get_error_string(lancius_status err);

LANCIUS_EXPORT lancius_context lancius_create_context(void);
LANCIUS_EXPORT void lancius_destroy_context(lancius_context ctx);

LANCIUS_EXPORT lancius_graph_handle lancius_graph_create_stable(lancius_context ctx);
LANCIUS_EXPORT void lancius_graph_destroy_stable(lancius_graph_handle g);

LANCIUS_EXPORT lancius_tensor_handle lancius_add_input(lancius_graph_handle g, size_t rows, size_t cols);
LANCIUS_EXPORT lancius_tensor_handle lancius_add_matmul(lancius_graph_handle g, lancius_tensor_handle a,
                                                        lancius_tensor_handle b);
LANCIUS_EXPORT lancius_tensor_handle lancius_add_relu(lancius_graph_handle g, lancius_tensor_handle a);

LANCIUS_EXPORT lancius_status lancius_bind_data(lancius_tensor_handle t, double* data_ptr);
LANCIUS_EXPORT lancius_status lancius_compile_and_run(lancius_graph_handle g);
LANCIUS_EXPORT lancius_status lancius_read_output(lancius_tensor_handle t, double* out_buffer, size_t buffer_size);

LANCIUS_EXPORT int lancius_tensor_get_dtype(lancius_tensor_handle t);

#ifdef __cplusplus
}
#endif
#endif

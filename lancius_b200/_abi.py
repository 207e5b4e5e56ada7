"""ctypes mirror of the Lancius C ABI (struct layouts and signatures).

The layouts follow include/lancius/lancius_ir.h, which is field-for-field the
reference's bleeding/v11A1/include/lancius/lancius_ir.h:31-62, so the same
bindings drive this package's library and any library built from the reference
sources.
"""
import ctypes as C

c_size = C.c_size_t
P = C.c_void_p


class LanciusNode(C.Structure):
    _fields_ = [
        ("id", C.c_uint32), ("op", C.c_int), ("shape", c_size * 4), ("ndim", C.c_uint8),
        ("kernel_h", C.c_uint32), ("kernel_w", C.c_uint32), ("stride", C.c_uint32), ("pad", C.c_uint32),
        ("axes", C.c_uint32 * 4), ("inputs", C.POINTER(C.c_void_p)), ("input_count", C.c_uint32),
        ("attr_val", C.c_double), ("runtime_data", C.POINTER(C.c_double)), ("dtype", C.c_int),
        ("scale", C.c_double), ("runtime_data_int8", C.POINTER(C.c_int8)), ("rt", P),
        ("is_view", C.c_uint8), ("strides", c_size * 4), ("view_source", P),
    ]


class LanciusGraph(C.Structure):
    _fields_ = [("arena", P), ("nodes", C.POINTER(C.POINTER(LanciusNode))), ("node_count", C.c_uint32),
                ("node_cap", C.c_uint32), ("next_id", C.c_uint32), ("rt_states", P), ("rt_cap", c_size)]


class LanciusWave(C.Structure):
    _fields_ = [("nodes", C.POINTER(C.POINTER(LanciusNode))), ("node_count", C.c_uint32)]


class LanciusSchedule(C.Structure):
    _fields_ = [("waves", C.POINTER(LanciusWave)), ("wave_count", C.c_uint32), ("plan", P), ("static_pool", P)]


class LanciusPlan(C.Structure):
    _fields_ = [("peak_memory", c_size), ("offsets", C.POINTER(c_size)), ("is_pooled", C.POINTER(C.c_uint8))]


NODE_P = C.POINTER(LanciusNode)
GRAPH_P = C.POINTER(LanciusGraph)
SCHED_P = C.POINTER(LanciusSchedule)
PLAN_P = C.POINTER(LanciusPlan)

# opcode numbering (lancius_ir.h)
OPS = ["NOP", "INPUT", "CONST", "ADD", "SUB", "MUL", "MATMUL", "RELU", "SOFTMAX", "SUM", "BROADCAST",
       "TRANSPOSE", "RELU_BWD", "SOFTMAX_BWD", "SUM_AXIS0", "SUM_AXIS1", "CONV2D", "MAXPOOL2D", "FLATTEN",
       "CONV2D_RELU_FUSED", "CROSS_ENTROPY", "CROSS_ENTROPY_BWD", "PERMUTE", "MATMUL_BATCHED", "CONV2D_BWD",
       "CONV2D_BWD_W", "MAXPOOL2D_BWD", "RESHAPE", "EMBEDDING", "LAYERNORM", "GELU", "ROPE", "ATTENTION",
       "KV_CACHE_READ", "KV_CACHE_WRITE", "RMSNORM", "SWIGLU", "GQA", "TANH"]
OP = {name: i for i, name in enumerate(OPS)}

DTYPE_FP64, DTYPE_INT8, DTYPE_FP32, DTYPE_INT32 = 0, 1, 2, 3

# builder signatures shared by every library exporting the Lancius IR API
IR_FUNCS = {
    "lancius_graph_create": (GRAPH_P, []),
    "lancius_graph_destroy": (None, [GRAPH_P]),
    "lancius_input": (NODE_P, [GRAPH_P, c_size, c_size]),
    "lancius_input_4d": (NODE_P, [GRAPH_P, c_size, c_size, c_size, c_size]),
    "lancius_const": (NODE_P, [GRAPH_P, C.c_double, c_size, c_size]),
    "lancius_add": (NODE_P, [GRAPH_P, NODE_P, NODE_P]),
    "lancius_sub": (NODE_P, [GRAPH_P, NODE_P, NODE_P]),
    "lancius_mul": (NODE_P, [GRAPH_P, NODE_P, NODE_P]),
    "lancius_matmul": (NODE_P, [GRAPH_P, NODE_P, NODE_P]),
    "lancius_relu": (NODE_P, [GRAPH_P, NODE_P]),
    "lancius_softmax": (NODE_P, [GRAPH_P, NODE_P]),
    "lancius_sum": (NODE_P, [GRAPH_P, NODE_P]),
    "lancius_broadcast": (NODE_P, [GRAPH_P, NODE_P, c_size, c_size]),
    "lancius_transpose": (NODE_P, [GRAPH_P, NODE_P]),
    "lancius_conv2d": (NODE_P, [GRAPH_P, NODE_P, NODE_P, C.c_uint32, C.c_uint32]),
    "lancius_maxpool2d": (NODE_P, [GRAPH_P, NODE_P, C.c_uint32, C.c_uint32]),
    "lancius_flatten": (NODE_P, [GRAPH_P, NODE_P]),
    "lancius_sum_axis0": (NODE_P, [GRAPH_P, NODE_P]),
    "lancius_sum_axis1": (NODE_P, [GRAPH_P, NODE_P]),
    "lancius_reshape": (NODE_P, [GRAPH_P, NODE_P, C.c_uint8, c_size, c_size, c_size, c_size]),
    "lancius_attention": (NODE_P, [GRAPH_P, NODE_P, NODE_P, NODE_P]),
    "lancius_layernorm": (NODE_P, [GRAPH_P, NODE_P, NODE_P, NODE_P]),
    "lancius_gelu": (NODE_P, [GRAPH_P, NODE_P]),
    "lancius_rmsnorm": (NODE_P, [GRAPH_P, NODE_P, NODE_P]),
    "lancius_swiglu": (NODE_P, [GRAPH_P, NODE_P, NODE_P]),
    "lancius_gqa": (NODE_P, [GRAPH_P, NODE_P, NODE_P, NODE_P, C.c_uint32, C.c_uint32]),
    "lancius_relu_bwd": (NODE_P, [GRAPH_P, NODE_P, NODE_P]),
    "lancius_softmax_bwd": (NODE_P, [GRAPH_P, NODE_P, NODE_P]),
    "lancius_cross_entropy": (NODE_P, [GRAPH_P, NODE_P, NODE_P]),
    "lancius_cross_entropy_bwd": (NODE_P, [GRAPH_P, NODE_P, NODE_P, NODE_P]),
    "lancius_conv2d_bwd": (NODE_P, [GRAPH_P, NODE_P, NODE_P, NODE_P, C.c_uint32, C.c_uint32]),
    "lancius_conv2d_bwd_w": (NODE_P, [GRAPH_P, NODE_P, NODE_P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]),
    "lancius_maxpool2d_bwd": (NODE_P, [GRAPH_P, NODE_P, NODE_P, C.c_uint32, C.c_uint32]),
    "lancius_node_bind_external_int8": (None, [NODE_P, P]),
    "lancius_optimize_fusion": (None, [GRAPH_P]),
    "lancius_graph_load": (GRAPH_P, [C.c_char_p]),
    "lancius_graph_save": (None, [GRAPH_P, C.c_char_p]),
    "lancius_node_bind_external": (None, [NODE_P, P]),
    "lancius_ir_schedule": (SCHED_P, [GRAPH_P]),
    "lancius_schedule_destroy": (None, [SCHED_P]),
    "lancius_build_memory_plan": (PLAN_P, [SCHED_P, GRAPH_P]),
    "lancius_memory_plan_destroy": (None, [PLAN_P]),
    "lancius_get_error": (C.c_int, []),
    "lancius_clear_error": (None, []),
}

# this package's additions
B200_FUNCS = {
    "lancius_attention_noncausal": (NODE_P, [GRAPH_P, NODE_P, NODE_P, NODE_P]),
    "lancius_tanh": (NODE_P, [GRAPH_P, NODE_P]),
    "lancius_build_memory_plan_ex": (PLAN_P, [SCHED_P, GRAPH_P, c_size, c_size, C.c_int]),
    "lancius_memory_plan_validate": (C.c_int, [PLAN_P, SCHED_P, GRAPH_P, c_size]),
    "lancius_schedule_peak_memory": (c_size, [SCHED_P]),
    "lcu_create": (P, [C.c_int]),
    "lcu_destroy": (None, [P]),
    "lcu_set_mode": (C.c_int, [P, C.c_int]),
    "lcu_stream": (P, [P]),
    "lcu_synchronize": (C.c_int, [P]),
    "lcu_check_stream": (C.c_int, [P]),
    "lcu_bind_plan": (C.c_int, [P, SCHED_P, GRAPH_P, PLAN_P]),
    "lcu_upload": (C.c_int, [P, NODE_P, P, C.c_int]),
    "lcu_download": (C.c_int, [P, NODE_P, P, C.c_int]),
    "lcu_download_async": (C.c_int, [P, NODE_P, C.c_void_p]),
    "lcu_watchdog_selftest": (C.c_int, [P]),
    "lcu_upload_bound_inputs": (C.c_int, [P]),
    "lcu_node_device_ptr": (P, [P, NODE_P]),
    "lcu_refresh_weights": (C.c_int, [P]),
    "lancius_schedule_execute_cuda": (None, [SCHED_P, P]),
    "lcu_last_launch_count": (C.c_int, [P]),
    "lcu_last_cuda_error": (C.c_char_p, []),
    "lcu_set_graph_replay": (C.c_int, [P, C.c_int]),
    "lcu_set_fusion": (C.c_int, [P, C.c_int]),
    "lcu_host_alloc": (P, [c_size]),
    "lcu_host_free": (None, [P]),
    "lcu_matmul": (C.c_int, [P, P, P, c_size, c_size, c_size, P, C.c_int, C.c_int, P]),
    "lcu_attention": (C.c_int, [P, P, P, P, c_size, c_size, c_size, c_size, C.c_int, C.c_int, P]),
    "lcu_conv2d": (C.c_int, [P, P, P, c_size, c_size, c_size, c_size, c_size, c_size, c_size, c_size, c_size,
                             C.c_int, C.c_int, P]),
    "lcu_layernorm": (C.c_int, [P, P, P, P, c_size, c_size, C.c_float, P]),
    "lcu_softmax": (C.c_int, [P, P, c_size, c_size, P]),
    "lcu_gelu": (C.c_int, [P, P, c_size, P]),
    "lcu_tanh": (C.c_int, [P, P, c_size, P]),
    "lcu_relu": (C.c_int, [P, P, c_size, P]),
    "lcu_add": (C.c_int, [P, P, P, c_size, P]),
    "lcu_sub": (C.c_int, [P, P, P, c_size, P]),
    "lcu_mul": (C.c_int, [P, P, P, c_size, P]),
    "lcu_broadcast": (C.c_int, [P, P, c_size, c_size, c_size, P]),
    "lcu_fill": (C.c_int, [P, C.c_float, c_size, P]),
    "lcu_sum_axis1": (C.c_int, [P, P, c_size, c_size, P]),
    "lcu_maxpool2d": (C.c_int, [P, P, c_size, c_size, c_size, c_size, c_size, c_size, P]),
    "lcu_build_info": (C.c_char_p, []),
    "lcu_sum": (C.c_int, [P, P, c_size, P]),
    "lcu_sum_axis0": (C.c_int, [P, P, c_size, c_size, P]),
    "lcu_transpose": (C.c_int, [P, P, c_size, c_size, P]),
    "lcu_relu_bwd": (C.c_int, [P, P, P, c_size, P]),
    "lcu_softmax_bwd": (C.c_int, [P, P, P, c_size, c_size, P]),
    "lcu_cross_entropy": (C.c_int, [P, P, P, c_size, c_size, P]),
    "lcu_cross_entropy_bwd": (C.c_int, [P, P, P, P, c_size, c_size, P]),
    "lcu_rmsnorm": (C.c_int, [P, P, P, c_size, c_size, C.c_float, P]),
    "lcu_swiglu": (C.c_int, [P, P, P, c_size, P]),
    "lcu_rope": (C.c_int, [P, P, c_size, c_size, c_size, c_size, C.c_int, P]),
    "lcu_gqa": (C.c_int, [P, P, P, P, c_size, c_size, c_size, c_size, P]),
    "lcu_attention_kv_cache": (C.c_int, [P, P, P, P, c_size, c_size, c_size, P]),
    "lcu_attention_kv_cache_batched": (C.c_int, [P, P, P, P, c_size, c_size, c_size, c_size, P]),
    "lcu_comm_unique_id": (C.c_int, [P, c_size]),
    "lcu_comm_create": (P, [C.c_int, C.c_int, P, C.c_int]),
    "lcu_comm_destroy": (None, [P]),
    "lcu_comm_abort": (None, [P]),
    "lcu_comm_size": (C.c_int, [P]),
    "lcu_gemm_colsplit": (C.c_int, [P, P, P, P, c_size, c_size, c_size, C.c_int, P]),
    "lcu_gemm_colsplit_fused": (C.c_int, [P, P, P, P, c_size, c_size, c_size, C.c_int, P]),
    "lcu_matmul_noalloc": (C.c_int, [P, P, P, c_size, c_size, c_size, P, C.c_int, C.c_int, P]),
    "lcu_noalloc_scratch_capacity": (c_size, []),
    "lcu_noalloc_prepare": (C.c_int, []),
}


def declare(lib, table):
    for name, (res, args) in table.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib

"""TEST INFRASTRUCTURE ONLY: the CPU parity checkers.

  Oracle()     -- liblcu_oracle.so, our FP64 restatement of the reference's kernels
                  and of its arena-mode executor (lcu_oracle.c cites the lines);
  reference()  -- _ref/liblancius_ref.so, the reference's own C sources compiled by
                  oracle/Makefile (present only where it was built).

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liblcu_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "liblancius_ref.so")
BASIS_REF_SO = os.path.join(HERE, "_ref", "libbasis_ref.so")

_D = C.POINTER(C.c_double)
_S = C.c_size_t


def _dp(a):
    return a.ctypes.data_as(_D)


class Oracle:
    def __init__(self):
        if not os.path.exists(ORACLE_SO):
            raise ImportError(f"{ORACLE_SO} not built: make -C {HERE}")
        lib = C.CDLL(ORACLE_SO, mode=os.RTLD_LOCAL)
        lib.orc_run_graph.restype = C.POINTER(_D)
        lib.orc_run_graph.argtypes = [C.c_void_p]
        lib.orc_free_results.argtypes = [C.c_void_p, C.POINTER(_D)]
        self.lib = lib

    # -- kernels ----------------------------------------------------------------
    def matmul(self, a, b):
        a = np.ascontiguousarray(a, np.float64); b = np.ascontiguousarray(b, np.float64)
        M, K = a.shape; N = b.shape[1]
        out = np.empty((M, N))
        self.lib.orc_matmul(_dp(out), _dp(a), _dp(b), _S(M), _S(K), _S(N))
        return out

    def attention(self, q, k, v, causal=True):
        q, k, v = (np.ascontiguousarray(x, np.float64) for x in (q, k, v))
        S, H, D = q.shape
        out = np.empty_like(q)
        self.lib.orc_attention(_dp(out), _dp(q), _dp(k), _dp(v), _S(S), _S(H), _S(D), C.c_int(1 if causal else 0))
        return out

    def naive_attention(self, q, k, v):
        q, k, v = (np.ascontiguousarray(x, np.float64) for x in (q, k, v))
        S, H, D = q.shape
        out = np.empty_like(q)
        self.lib.orc_naive_attention(_dp(out), _dp(q), _dp(k), _dp(v), _S(S), _S(H), _S(D))
        return out

    def conv2d(self, x, w, stride, pad, relu=False):
        x = np.ascontiguousarray(x, np.float64); w = np.ascontiguousarray(w, np.float64)
        N, Ci, H, W = x.shape; Co, _, Kh, Kw = w.shape
        Ho = (H + 2 * pad - Kh) // stride + 1; Wo = (W + 2 * pad - Kw) // stride + 1
        out = np.empty((N, Co, Ho, Wo))
        self.lib.orc_conv2d(_dp(out), _dp(x), _dp(w), _S(N), _S(Ci), _S(H), _S(W), _S(Co), _S(Kh), _S(Kw),
                            _S(stride), _S(pad), C.c_int(1 if relu else 0))
        return out

    def layernorm(self, x, gamma, beta, eps=1e-5):
        x = np.ascontiguousarray(x, np.float64)
        out = np.empty_like(x)
        self.lib.orc_layernorm(_dp(out), _dp(x), _dp(np.ascontiguousarray(gamma, np.float64)),
                               _dp(np.ascontiguousarray(beta, np.float64)), _S(x.shape[0]), _S(x.shape[1]),
                               C.c_double(eps))
        return out

    def gelu(self, x):
        x = np.ascontiguousarray(x, np.float64)
        out = np.empty_like(x)
        self.lib.orc_gelu(_dp(out), _dp(x), _S(x.size))
        return out

    def softmax(self, x):
        x = np.ascontiguousarray(x, np.float64)
        out = np.empty_like(x)
        self.lib.orc_softmax(_dp(out), _dp(x), _S(x.shape[0]), _S(x.shape[1]))
        return out

    def rmsnorm(self, x, gamma, eps=1e-5):
        x = np.ascontiguousarray(x, np.float64)
        out = np.empty_like(x)
        self.lib.orc_rmsnorm(_dp(out), _dp(x), _dp(np.ascontiguousarray(gamma, np.float64)), _S(x.shape[0]),
                             _S(x.shape[1]), C.c_double(eps))
        return out

    def maxpool2d(self, x, k, stride):
        x = np.ascontiguousarray(x, np.float64)
        N, Cc, H, W = x.shape
        out = np.empty((N, Cc, (H - k) // stride + 1, (W - k) // stride + 1))
        self.lib.orc_maxpool2d(_dp(out), _dp(x), _S(N), _S(Cc), _S(H), _S(W), _S(k), _S(stride))
        return out

    # -- graphs -----------------------------------------------------------------
    def run_graph(self, graph, nodes=None):
        """Arena-mode CPU execution of a graph whose INPUTs are bound (Graph.bind).
        Returns {node_id: ndarray} for `nodes` (default: every node)."""
        res = self.lib.orc_run_graph(C.cast(graph.ptr, C.c_void_p))
        out = {}
        try:
            for n in (nodes if nodes is not None else graph.nodes()):
                p = res[n.id]
                if p:
                    out[n.id] = np.ctypeslib.as_array(p, shape=(n.size,)).copy().reshape(n.shape)
        finally:
            self.lib.orc_free_results(C.cast(graph.ptr, C.c_void_p), res)
        return out


def reference_available():
    return os.path.exists(REF_SO)


def reference():
    """The reference's own library (compiled from its sources), with the IR bindings."""
    import lancius_b200._abi as abi
    if not reference_available():
        raise ImportError(f"{REF_SO} not built: make -C {HERE} ref")
    lib = C.CDLL(REF_SO, mode=os.RTLD_LOCAL)
    table = {k: v for k, v in abi.IR_FUNCS.items()}
    abi.declare(lib, table)
    lib.lancius_arena_create.restype = C.c_void_p
    lib.lancius_arena_create.argtypes = [_S]
    lib.lancius_arena_destroy.argtypes = [C.c_void_p]
    lib.lancius_schedule_execute.argtypes = [abi.SCHED_P, C.c_void_p]
    lib.lancius_schedule_execute.restype = None
    lib.lancius_schedule_attach_pool.argtypes = [abi.SCHED_P, C.c_void_p, abi.PLAN_P]
    for name in ("kernel_attention",):
        getattr(lib, name).restype = None
    return lib


def run_reference_graph(lib, graph, nodes, arena_bytes=64 << 20):
    """Executes `graph` (built with the reference library) in arena mode with the
    reference's own lancius_schedule_execute; returns {node_id: ndarray}."""
    sched = lib.lancius_ir_schedule(graph.ptr)
    arena = lib.lancius_arena_create(arena_bytes)
    try:
        lib.lancius_schedule_execute(sched, arena)
        out = {}
        for n in nodes:
            p = n.c.runtime_data
            out[n.id] = np.ctypeslib.as_array(p, shape=(n.size,)).copy().reshape(n.shape)
        return out
    finally:
        lib.lancius_arena_destroy(arena)
        lib.lancius_schedule_destroy(sched)


def basis_reference():
    """The reference's BASIS graph builder (src/basis/stage6_ir/graph.c, compiled here), or
    None when it was not built."""
    if not os.path.exists(BASIS_REF_SO):
        return None
    return C.CDLL(BASIS_REF_SO, mode=os.RTLD_LOCAL)

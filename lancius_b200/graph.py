"""Python front end for the Lancius graph API (same builder names as the C API).

`Graph(lib)` drives any library exporting the Lancius IR symbols: this package's
liblancius_b200.so by default. Nodes are `Node` handles; host FP64 data bound to
INPUT nodes is kept alive by the Graph.
"""
import ctypes as C

import numpy as np

from . import _abi
from ._lib import load


class LanciusError(RuntimeError):
    def __init__(self, code, what=""):
        detail = ""
        try:
            msg = load().lcu_last_cuda_error()
            if msg and msg != b"no error":
                detail = f" (CUDA: {msg.decode()})"
        except Exception:
            pass
        super().__init__(f"{what}: lancius error {code}{detail}")
        self.code = code


class Node:
    __slots__ = ("ptr", "graph")

    def __init__(self, ptr, graph):
        self.ptr = ptr
        self.graph = graph

    @property
    def c(self):
        return self.ptr.contents

    @property
    def id(self):
        return self.c.id

    @property
    def op(self):
        return _abi.OPS[self.c.op]

    @property
    def shape(self):
        c = self.c
        return tuple(c.shape[i] for i in range(c.ndim))

    @property
    def size(self):
        n = 1
        for s in self.shape:
            n *= s
        return n

    def inputs(self):
        c = self.c
        return [c.inputs[i] for i in range(c.input_count)]

    def __repr__(self):
        return f"Node({self.id}, {self.op}, {self.shape})"


class Schedule:
    def __init__(self, graph):
        self.graph = graph
        self.lib = graph.lib
        self.ptr = self.lib.lancius_ir_schedule(graph.ptr)
        if not self.ptr:
            raise LanciusError(self.lib.lancius_get_error(), "lancius_ir_schedule")

    def waves(self):
        s = self.ptr.contents
        out = []
        for w in range(s.wave_count):
            wave = s.waves[w]
            out.append([wave.nodes[i].contents.id for i in range(wave.node_count)])
        return out

    def close(self):
        if self.ptr:
            self.lib.lancius_schedule_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Graph:
    @classmethod
    def load(cls, path, lib=None):
        """lancius_graph_load: weights stay in the loaded INPUT nodes (owned heap FP64)."""
        g = cls.__new__(cls)
        g.lib = lib if lib is not None else load()
        g.ptr = g.lib.lancius_graph_load(path.encode())
        if not g.ptr:
            raise LanciusError(g.lib.lancius_get_error(), f"lancius_graph_load({path})")
        g._keep = {}
        return g

    def save(self, path):
        self.lib.lancius_graph_save(self.ptr, path.encode())

    def __init__(self, lib=None):
        self.lib = lib if lib is not None else load()
        self.ptr = self.lib.lancius_graph_create()
        if not self.ptr:
            raise LanciusError(self.lib.lancius_get_error(), "lancius_graph_create")
        self._keep = {}

    # -- builders (names of the C API without the lancius_ prefix) -------------
    def _mk(self, fname, *args):
        conv = [a.ptr if isinstance(a, Node) else a for a in args]
        p = getattr(self.lib, fname)(self.ptr, *conv)
        if not p:
            raise LanciusError(self.lib.lancius_get_error(), fname)
        return Node(p, self)

    def input(self, r, c): return self._mk("lancius_input", r, c)
    def input_4d(self, n, c, h, w): return self._mk("lancius_input_4d", n, c, h, w)
    def const(self, val, r, c): return self._mk("lancius_const", float(val), r, c)
    def add(self, a, b): return self._mk("lancius_add", a, b)
    def sub(self, a, b): return self._mk("lancius_sub", a, b)
    def mul(self, a, b): return self._mk("lancius_mul", a, b)
    def matmul(self, a, b): return self._mk("lancius_matmul", a, b)
    def relu(self, a): return self._mk("lancius_relu", a)
    def softmax(self, a): return self._mk("lancius_softmax", a)
    def sum(self, a): return self._mk("lancius_sum", a)
    def broadcast(self, a, r, c): return self._mk("lancius_broadcast", a, r, c)
    def transpose(self, a): return self._mk("lancius_transpose", a)
    def conv2d(self, x, w, stride, pad): return self._mk("lancius_conv2d", x, w, stride, pad)
    def maxpool2d(self, x, k, stride): return self._mk("lancius_maxpool2d", x, k, stride)
    def flatten(self, x): return self._mk("lancius_flatten", x)
    def sum_axis0(self, a): return self._mk("lancius_sum_axis0", a)
    def sum_axis1(self, a): return self._mk("lancius_sum_axis1", a)
    def layernorm(self, x, g, b): return self._mk("lancius_layernorm", x, g, b)
    def gelu(self, a): return self._mk("lancius_gelu", a)
    def rmsnorm(self, x, g): return self._mk("lancius_rmsnorm", x, g)
    def attention(self, q, k, v): return self._mk("lancius_attention", q, k, v)
    def swiglu(self, gate, up): return self._mk("lancius_swiglu", gate, up)
    def gqa(self, q, k, v, hq, hkv): return self._mk("lancius_gqa", q, k, v, hq, hkv)
    def relu_bwd(self, grad, fwd): return self._mk("lancius_relu_bwd", grad, fwd)
    def softmax_bwd(self, grad, y): return self._mk("lancius_softmax_bwd", grad, y)
    def cross_entropy(self, logits, targets): return self._mk("lancius_cross_entropy", logits, targets)
    def cross_entropy_bwd(self, logits, targets, g): return self._mk("lancius_cross_entropy_bwd", logits, targets, g)
    def conv2d_bwd(self, grad, x, w, stride, pad): return self._mk("lancius_conv2d_bwd", grad, x, w, stride, pad)
    def conv2d_bwd_w(self, grad, x, kh, kw, stride, pad): return self._mk("lancius_conv2d_bwd_w", grad, x, kh, kw, stride, pad)
    def maxpool2d_bwd(self, grad, x, k, stride): return self._mk("lancius_maxpool2d_bwd", grad, x, k, stride)
    def attention_noncausal(self, q, k, v): return self._mk("lancius_attention_noncausal", q, k, v)
    def tanh(self, a): return self._mk("lancius_tanh", a)

    def reshape(self, x, *shape):
        s = list(shape) + [0] * (4 - len(shape))
        return self._mk("lancius_reshape", x, len(shape), *s)

    def optimize_fusion(self):
        self.lib.lancius_optimize_fusion(self.ptr)

    # -- data ------------------------------------------------------------------
    def bind(self, node, array):
        a = np.ascontiguousarray(array, dtype=np.float64)
        if a.size != node.size:
            raise ValueError(f"bind {node}: {a.size} values for {node.size} elements")
        self._keep[node.id] = a
        self.lib.lancius_node_bind_external(node.ptr, a.ctypes.data_as(C.c_void_p))
        return a

    def bind_int8(self, node, array, scale):
        """INT8 weights as the reference's quantizer leaves them (lancius_quantize.c:19-28):
        dtype INT8, per-tensor scale, data in runtime_data_int8."""
        a = np.ascontiguousarray(array, dtype=np.int8)
        self._keep[(node.id, "i8")] = a
        node.c.dtype = _abi.DTYPE_INT8
        node.c.scale = float(scale)
        self.lib.lancius_node_bind_external_int8(node.ptr, a.ctypes.data_as(C.c_void_p))
        return a

    def nodes(self):
        g = self.ptr.contents
        return [Node(g.nodes[i], self) for i in range(g.node_count)]

    def schedule(self):
        return Schedule(self)

    def close(self):
        if self.ptr:
            self.lib.lancius_graph_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

"""ctypes binding of the BASIS stage-6 graph API (include/basis/stage6_ir/graph.h, the
reference's legacy 2-D graph builder) and of basis_graph_lower(), which turns a BASIS
graph into a Lancius graph for the B200 executor."""
import ctypes as C

from . import _abi
from ._lib import load
from .graph import Graph, LanciusError, Node

OPS = ["INPUT", "MATMUL", "ADD", "RELU", "TANH", "BROADCAST_ADD"]


class BasisNode(C.Structure):
    _fields_ = [("id", C.c_int), ("op", C.c_int), ("input_ids", C.c_int * 2), ("rows", C.c_size_t),
                ("cols", C.c_size_t), ("name", C.c_char_p)]


class BasisGraphC(C.Structure):
    _fields_ = [("nodes", C.POINTER(BasisNode)), ("node_count", C.c_size_t), ("node_cap", C.c_size_t)]


BG_P = C.POINTER(BasisGraphC)
BN_P = C.POINTER(BasisNode)

FUNCS = {
    "basis_graph_new": (BG_P, []),
    "basis_graph_input": (BN_P, [BG_P, C.c_char_p, C.c_size_t, C.c_size_t]),
    "basis_graph_matmul": (BN_P, [BG_P, BN_P, BN_P]),
    "basis_graph_add": (BN_P, [BG_P, BN_P, BN_P]),
    "basis_graph_broadcast_add": (BN_P, [BG_P, BN_P, BN_P]),
    "basis_graph_relu": (BN_P, [BG_P, BN_P]),
    "basis_graph_tanh": (BN_P, [BG_P, BN_P]),
    "basis_graph_print": (None, [BG_P]),
    "basis_graph_free": (None, [BG_P]),
}


def declare(lib):
    _abi.declare(lib, FUNCS)
    if hasattr(lib, "basis_graph_lower"):     # this library only
        lib.basis_graph_lower.restype = C.c_int
        lib.basis_graph_lower.argtypes = [BG_P, _abi.GRAPH_P, C.POINTER(_abi.NODE_P)]
    return lib


class BasisGraph:
    """A BASIS graph built through `lib` (this library by default, or the reference's
    own libbasis for parity checks). Nodes are referred to by id: the C array moves as
    it grows, so node pointers are re-fetched for every call."""

    def __init__(self, lib=None):
        self.lib = declare(lib) if lib is not None else declare(load())
        self.ptr = self.lib.basis_graph_new()

    def _node(self, i):
        return C.pointer(self.ptr.contents.nodes[i]) if i is not None else None

    def _mk(self, fname, *args):
        p = getattr(self.lib, fname)(self.ptr, *args)
        return p.contents.id if p else None

    def input(self, name, r, c): return self._mk("basis_graph_input", name.encode(), r, c)
    def matmul(self, a, b): return self._mk("basis_graph_matmul", self._node(a), self._node(b))
    def add(self, a, b): return self._mk("basis_graph_add", self._node(a), self._node(b))
    def broadcast_add(self, a, bias): return self._mk("basis_graph_broadcast_add", self._node(a), self._node(bias))
    def relu(self, a): return self._mk("basis_graph_relu", self._node(a))
    def tanh(self, a): return self._mk("basis_graph_tanh", self._node(a))

    def nodes(self):
        g = self.ptr.contents
        out = []
        for i in range(g.node_count):
            n = g.nodes[i]
            out.append((n.id, OPS[n.op], tuple(n.input_ids), n.rows, n.cols,
                        n.name.decode() if n.name else None))
        return out

    def lower(self, graph=None):
        """Lancius graph (this library) computing the BASIS graph; returns (graph, {id: Node})."""
        graph = graph or Graph()
        n = self.ptr.contents.node_count
        arr = (_abi.NODE_P * max(n, 1))()
        if self.lib.basis_graph_lower(self.ptr, graph.ptr, arr) != 0:
            raise LanciusError(-4, "basis_graph_lower")
        return graph, {i: Node(arr[i], graph) for i in range(n)}

    def close(self):
        if self.ptr:
            self.lib.basis_graph_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

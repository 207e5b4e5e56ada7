"""Parity at the benchmark configurations' full sizes (FP32-exact mode), with both parts
of the bar against the FP64 oracle: normwise max|d|/max|ref| <= 1e-4 and elementwise
|d| <= 1e-4*|ref| + a*max|ref|, a = conftest.exact_elem_abs(K) for the longest reduction
K feeding the output (1e-6 up to K = 128, 8e-9*K beyond: the tensor cores' truncating
FP32 accumulation).

The GPU always runs the full-size problem. Where the FP64 oracle would take minutes on
the host, it checks a subset whose values depend on nothing else: whole images of the
conv stack, whole sequences of the encoder (each batch element is its own subgraph),
whole rows of a square product (a row of C depends only on that row of A).
Conv stack: reference lancius_vision_ops.c:60-81; encoder: lancius_scheduler.c:109-120
(LayerNorm, GELU), lancius_kernels.c:278-332 (attention); GEMM: lancius_scheduler.c:190-235.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_close
import lancius_b200 as L
from lancius_b200 import MODE_FP32_EXACT, EPI_NONE, configs

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

NORM = 1e-4


@pytest.fixture(scope="module")
def device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    d = L.Device(0)
    yield d
    d.close()


def run_graph(device, built):
    sched = built.graph.schedule()
    device.set_graph_replay(False)
    device.bind(sched)
    for node, arr in built.inputs:
        device.upload(node, arr)
    device.execute(sched)
    device.synchronize()
    return [device.download(o) for o in built.outputs]


def oracle_of(orc, built):
    built.bind_host()
    r = orc.run_graph(built.graph, built.outputs)
    return [r[o.id] for o in built.outputs]


def test_conv_stack_b32_224(device, orc):
    """Config 3 at batch 32 x 224^2; images 0, 17 and 31 checked (each through its own
    batch-1 oracle graph with the same weights)."""
    (y,) = run_graph(device, configs.conv_stack(L.Graph(), batch=32, hw=224))
    assert y.shape == (32, 1000)
    for i in (0, 17, 31):
        (ref,) = oracle_of(orc, configs.conv_stack(L.Graph(), batch=32, hw=224, rows=(i, i + 1)))
        assert_close(y[i:i + 1], ref, NORM, k=128 * 9)


def test_encoder_b16_s512_12_layers(device, orc):
    """Config 4 (BERT-base shape, 12 layers, S512, batch 16) on the GPU; sequences 0 and 15
    checked against the oracle's run of a batch-1 graph drawing the same sequence."""
    ys = run_graph(device, configs.encoder(L.Graph(), batch=16, seq=512, layers=12))
    for e in (0, 15):
        (ref,) = oracle_of(orc, configs.encoder(L.Graph(), batch=1, seq=512, layers=12, first=e))
        assert_close(ys[e], ref, NORM, k=3072)


def test_gemm_4096_full(device, orc):
    """Config 5, N = 4096, through the graph API; every element checked."""
    b = configs.gemm(L.Graph(), 4096)
    (y,) = run_graph(device, b)
    (ref,) = oracle_of(orc, b)
    assert_close(y, ref, NORM, k=4096)


ROWS = np.array([0, 1, 777, 2048, 4095, 5000, 8191, 9999, 12345, 16383])


@pytest.mark.parametrize("n", [8192, 16384])
def test_gemm_square_sampled_rows(device, orc, n):
    """Config 5 at N = 8192 and 16384 (K > 8192: split-K) through lcu_matmul and, for
    16384, the fused column-split GEMM on a one-rank communicator; 64 rows of C checked."""
    lib = L.load()
    b = configs.gemm(L.Graph(), n)
    (_, a), (_, w) = b.inputs
    rows = np.unique(np.concatenate([ROWS[ROWS < n], np.linspace(0, n - 1, 64 - len(ROWS[ROWS < n])).astype(int)]))
    ref = orc.matmul(np.ascontiguousarray(a[rows]), w)
    da = torch.tensor(a.astype(np.float32), device="cuda")
    dw = torch.tensor(w.astype(np.float32), device="cuda")
    del a
    c = torch.full((n, n), float("nan"), device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr())
    assert lib.lcu_matmul(P(c), P(da), P(dw), n, n, n, None, EPI_NONE, MODE_FP32_EXACT, None) == 0
    torch.cuda.synchronize()
    assert_close(c[torch.from_numpy(rows).cuda()].double().cpu().numpy(), ref, NORM, k=8192)
    if n == 16384:
        uid = C.create_string_buffer(128)
        assert lib.lcu_comm_unique_id(uid, 128) == 0
        comm = lib.lcu_comm_create(1, 0, C.c_char_p(uid.raw), 0)
        assert comm
        try:
            c.fill_(float("nan"))
            torch.cuda.synchronize()
            assert lib.lcu_gemm_colsplit_fused(comm, P(c), P(da), P(dw), n, n, n, MODE_FP32_EXACT, None) == 0
            torch.cuda.synchronize()
            assert_close(c[torch.from_numpy(rows).cuda()].double().cpu().numpy(), ref, NORM, k=8192)
        finally:
            lib.lcu_comm_destroy(comm)

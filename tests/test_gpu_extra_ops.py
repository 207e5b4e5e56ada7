"""GPU parity of the training, LLM and INT8 operators (executor path) against the
FP64 oracle; the oracle itself is pinned to the reference executor on these graphs
(test_oracle_extra_ops.py). FP32 storage: normwise 1e-4."""
import numpy as np
import pytest

from conftest import assert_close
import lancius_b200 as L
import opgraphs

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    d = L.Device(0)
    yield d
    d.close()


@pytest.mark.parametrize("build", [opgraphs.training_ops, opgraphs.llm_ops, opgraphs.int8_matmul,
                                   opgraphs.int8_conv, opgraphs.int8_matmul_large, opgraphs.int8_conv_large,
                                   opgraphs.int8_conv_large_k144])
def test_extra_ops_on_gpu(device, orc, build):
    g = L.Graph()
    r = build(g)
    inputs, outputs = r[0], r[-1]
    for n, arr in inputs.items():
        g.bind(n, np.asarray(arr, np.float32).astype(np.float64))   # FP32-exact inputs: same quantisation
    if len(r) == 3:
        for n, (q, scale) in r[1].items():
            g.bind_int8(n, q, scale)
    s = g.schedule()
    device.set_graph_replay(False)
    device.bind(s)
    device.upload_bound_inputs()
    device.execute(s)
    if "large" in build.__name__:   # absmax + quantise (+ transpose / re-pitch) + tcgen05 kind::i8 GEMM
        assert device.last_launch_count >= 3
    want = orc.run_graph(g, outputs)
    for o in outputs:
        got = device.download(o)
        assert_close(got, want[o.id], 1e-4)
        if build.__name__.startswith("int8"):
            # integer accumulation is exact: the FP32 result is the reference's value rounded once
            assert np.array_equal(np.asarray(got, np.float32), np.asarray(want[o.id], np.float32))


def test_rope_and_gqa_per_op(orc):
    import ctypes as C
    from lancius_b200 import data, load
    lib = load()
    B, S, H, D = 1, 40, 4, 64
    q = data.normal(1, (B, S, H, D)); k = data.normal(2, (B, S, H, D))
    qd = torch.tensor(q.astype(np.float32), device="cuda"); kd = torch.tensor(k.astype(np.float32), device="cuda")
    assert lib.lcu_rope(C.c_void_p(qd.data_ptr()), C.c_void_p(kd.data_ptr()), B, S, H, D, 3, None) == 0
    torch.cuda.synchronize()
    qr, kr = q.copy(), k.copy()
    dp = lambda a: a.ctypes.data_as(C.POINTER(C.c_double))
    orc.lib.orc_rope(dp(qr), dp(kr), C.c_size_t(B), C.c_size_t(S), C.c_size_t(H), C.c_size_t(D), C.c_int(3))
    assert_close(qd.cpu().numpy(), qr, 1e-5)
    assert_close(kd.cpu().numpy(), kr, 1e-5)


@pytest.mark.parametrize("B,S,H,D", [(1, 1, 2, 64), (1, 37, 4, 64), (1, 5000, 8, 64), (3, 777, 2, 80),
                                     (2, 1500, 4, 128), (1, 300, 2, 256), (1, 65, 3, 20), (2, 3001, 3, 32)])
def test_kv_cache_attention(orc, B, S, H, D):
    """lcu_attention_kv_cache(_batched) against the oracle's restatement of
    kernel_attention_kv_cache: single split (short caches) and split-KV merges."""
    import ctypes as C
    from lancius_b200 import data, load
    lib = load()
    q = data.normal(21, (B, H * D)); kc = data.normal(22, (B, S, H, D)); vc = data.normal(23, (B, S, H, D))
    q, kc, vc = (a.astype(np.float32).astype(np.float64) for a in (q, kc, vc))
    dev = [torch.tensor(a.astype(np.float32), device="cuda") for a in (q, kc, vc)]
    out = torch.empty((B, H * D), device="cuda")
    ptr = lambda t: C.c_void_p(t.data_ptr())
    if B == 1:
        assert lib.lcu_attention_kv_cache(ptr(out), ptr(dev[0]), ptr(dev[1]), ptr(dev[2]), S, H, D, None) == 0
    else:
        assert lib.lcu_attention_kv_cache_batched(ptr(out), ptr(dev[0]), ptr(dev[1]), ptr(dev[2]), B, S, H, D,
                                                  None) == 0
    torch.cuda.synchronize()
    dp = lambda a: a.ctypes.data_as(C.POINTER(C.c_double))
    want = np.empty((B, H * D))
    for b in range(B):
        row = np.empty(H * D)
        qb, kb, vb = (np.ascontiguousarray(a[b]) for a in (q, kc, vc))
        orc.lib.orc_attention_kv_cache(dp(row), dp(qb), dp(kb), dp(vb), C.c_size_t(S), C.c_size_t(H), C.c_size_t(D))
        want[b] = row
    assert_close(out.cpu().numpy(), want, 1e-4)


def test_kv_cache_attention_rejects_large_head_dim():
    import ctypes as C
    from lancius_b200 import load
    t = torch.zeros(4, device="cuda")
    p = C.c_void_p(t.data_ptr())
    assert load().lcu_attention_kv_cache(p, p, p, p, 1, 1, 512, None) != 0


def test_int8_weights_repacked_on_upload(device, orc):
    """The tensor-core INT8 MATMUL reads a K-major copy of the weights made at upload
    time: uploading new weights must change the next result."""
    from lancius_b200 import data
    g = L.Graph()
    inputs, int8s, outputs = opgraphs.int8_matmul_large(g)
    for n, arr in inputs.items():
        g.bind(n, np.asarray(arr, np.float32).astype(np.float64))
    (wnode, (wq, scale)), = int8s.items()
    g.bind_int8(wnode, wq, scale)
    s = g.schedule()
    device.set_graph_replay(True)
    device.bind(s)
    device.upload_bound_inputs()
    device.execute(s)
    first = device.download(outputs[0])
    wq2 = np.round(data.uniform(99, wq.shape, -127, 127)).astype(np.int8)
    g.bind_int8(wnode, wq2, scale)
    device.upload_bound_inputs()
    device.execute(s)                      # replays the captured graph
    second = device.download(outputs[0])
    want = orc.run_graph(g, outputs)[outputs[0].id]
    assert not np.array_equal(first, second)
    assert np.array_equal(np.asarray(second, np.float32), np.asarray(want, np.float32))

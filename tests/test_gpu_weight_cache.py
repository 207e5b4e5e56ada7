"""TF32 hi/lo operand handling of the tensor-core MATMUL. MATMULs whose weights are INPUT
nodes read hi/lo copies made at upload time. Checks that a re-upload and lcu_refresh_weights remake them,
that grouped waves (distinct and shared weights) index them correctly, and that the cached
path gives the same bytes as splitting per run (LCU_NO_WEIGHT_CACHE=1). Activations (A) are
split inside the GEMM (raw-A mode); it must match the separate split pass (LCU_NO_RAW_A=1)
bit for bit, and shapes it cannot take (K % 4 != 0) fall back to the pass."""
import os

import numpy as np
import pytest

from conftest import assert_close
import lancius_b200 as L

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

M, K, N = 256, 512, 384          # 50M multiply-adds: tensor-core path


@pytest.fixture(scope="module")
def device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    d = L.Device(0)
    yield d
    d.close()


def rnd(seed, *shape):
    return np.random.default_rng(seed).standard_normal(shape)


def test_reupload_and_refresh(device):
    g = L.Graph()
    x, w = g.input(M, K), g.input(K, N)
    y = g.matmul(x, w)
    s = g.schedule()
    device.bind(s)
    xa, w1, w2 = rnd(1, M, K), rnd(2, K, N), rnd(3, K, N)
    device.upload(x, xa)
    device.upload(w, w1)
    device.execute(s)
    assert_close(device.download(y), xa @ w1, 1e-4, k=K)
    device.upload(w, w2)                      # a new upload re-splits the weight
    device.execute(s)
    assert_close(device.download(y), xa @ w2, 1e-4, k=K)
    # a write through the device pointer needs an explicit refresh
    assert device.lib.lcu_fill(device.device_ptr(w), 0.5, K * N, device.stream) == 0
    device.refresh_weights()
    device.execute(s)
    assert_close(device.download(y), xa @ np.full((K, N), 0.5), 1e-4, k=K)


def test_grouped_distinct_and_shared_weights(device):
    g = L.Graph()
    x1, x2 = g.input(M, K), g.input(M, K)
    wq, wk, wv = g.input(K, N), g.input(K, N), g.input(K, N)
    outs = [g.matmul(x1, wq), g.matmul(x1, wk), g.matmul(x1, wv), g.matmul(x2, wq)]
    s = g.schedule()
    device.bind(s)
    arrs = {n: rnd(10 + i, *n.shape) for i, n in enumerate([x1, x2, wq, wk, wv])}
    for n, a in arrs.items():
        device.upload(n, a)
    device.execute(s)
    refs = [arrs[x1] @ arrs[wq], arrs[x1] @ arrs[wk], arrs[x1] @ arrs[wv], arrs[x2] @ arrs[wq]]
    for o, r in zip(outs, refs):
        assert_close(device.download(o), r, 1e-4, k=K)


def test_cached_equals_per_run_split(device):
    g = L.Graph()
    x, w, bias = g.input(M, K), g.input(K, N), g.input(1, N)
    y = g.relu(g.add(g.matmul(x, w), g.broadcast(bias, M, N)))
    s = g.schedule()
    xa, wa, ba = rnd(21, M, K), rnd(22, K, N), rnd(23, 1, N)

    def run():
        device.bind(s)
        for n, a in ((x, xa), (w, wa), (bias, ba)):
            device.upload(n, a)
        device.execute(s)
        return device.download(y, np.float32)

    cached = run()
    os.environ["LCU_NO_WEIGHT_CACHE"] = "1"
    try:
        per_run = run()
    finally:
        del os.environ["LCU_NO_WEIGHT_CACHE"]
    os.environ["LCU_NO_RAW_A"] = "1"      # A split by a separate pass instead of inside the GEMM
    try:
        a_split = run()
    finally:
        del os.environ["LCU_NO_RAW_A"]
    assert np.array_equal(cached, per_run)
    assert np.array_equal(cached, a_split)
    assert_close(cached, np.maximum(xa @ wa + ba, 0), 1e-4, k=K)


@pytest.mark.parametrize("k", [510, 513, 1000])
def test_raw_a_shapes(device, k):
    g = L.Graph()
    x, w = g.input(300, k), g.input(k, 200)
    y = g.matmul(x, w)
    s = g.schedule()
    device.bind(s)
    xa, wa = rnd(31, 300, k), rnd(32, k, 200)
    device.upload(x, xa)
    device.upload(w, wa)
    device.execute(s)
    assert_close(device.download(y), xa @ wa, 1e-4, k=min(k, 8192))


# grouped waves, ragged edges (M, N not multiples of the 256x256 tile, odd chunk counts per
# epilogue warp) and the fused bias/ReLU/residual epilogue, against FP64
EPI_SHAPES = [(256, 8192, 256, 1), (1000, 4096, 1000, 1), (512, 768, 768, 16), (300, 1000, 200, 3), (8192, 3072, 768, 1),
              (130, 64, 40, 2)]


@pytest.mark.parametrize("m,k,n,groups", EPI_SHAPES)
def test_gemm_epilogue_shapes(device, m, k, n, groups):
    g = L.Graph()
    w, bias = g.input(k, n), g.input(1, n)
    xs = [g.input(m, k) for _ in range(groups)]
    rs = [g.input(m, n) for _ in range(groups)]
    ys = [g.add(g.relu(g.add(g.matmul(x, w), g.broadcast(bias, m, n))), r) for x, r in zip(xs, rs)]
    s = g.schedule()
    wa, ba = rnd(41, k, n), rnd(42, 1, n)
    xa = [rnd(50 + i, m, k) for i in range(groups)]
    ra = [rnd(70 + i, m, n) for i in range(groups)]
    device.bind(s)
    device.upload(w, wa)
    device.upload(bias, ba)
    for node, a in zip(xs + rs, xa + ra):
        device.upload(node, a)
    device.execute(s)
    out = [device.download(y) for y in ys]
    for i in range(groups):
        assert_close(out[i], np.maximum(xa[i] @ wa + ba, 0) + ra[i], 1e-4, k=min(k, 8192))
    device.execute(s)                         # a rerun gives the same bytes
    assert all(np.array_equal(device.download(y), a) for y, a in zip(ys, out))


def conv_ref(x, w, stride, pad):
    t = torch.nn.functional.conv2d(torch.from_numpy(x), torch.from_numpy(w), stride=stride, padding=pad)
    return t.numpy()


def test_conv_weights_reupload_refresh_and_per_run(device):
    """The tensor-core conv reads [Co][Kh][Kw][Ci] hi/lo weight copies made at upload time:
    a re-upload and lcu_refresh_weights remake them, and the bytes equal splitting per run."""
    n, ci, hw, co = 2, 32, 32, 64           # 64 x 2048 x 288 multiply-adds per image: tensor cores
    g = L.Graph()
    x, w = g.input_4d(n, ci, hw, hw), g.input_4d(co, ci, 3, 3)
    y = g.relu(g.conv2d(x, w, 1, 1))
    s = g.schedule()
    xa, w1, w2 = rnd(81, n, ci, hw, hw), rnd(82, co, ci, 3, 3), rnd(83, co, ci, 3, 3)
    kk = ci * 9

    def run(wa):
        device.bind(s)
        device.upload(x, xa)
        device.upload(w, wa)
        device.execute(s)
        return device.download(y, np.float32)

    cached = run(w1)
    assert_close(cached, np.maximum(conv_ref(xa, w1, 1, 1), 0), 1e-4, k=kk)
    device.upload(w, w2)                      # a new upload re-splits the weight
    device.execute(s)
    assert_close(device.download(y), np.maximum(conv_ref(xa, w2, 1, 1), 0), 1e-4, k=kk)
    assert device.lib.lcu_fill(device.device_ptr(w), 0.25, co * kk, device.stream) == 0
    device.refresh_weights()
    device.execute(s)
    assert_close(device.download(y), np.maximum(conv_ref(xa, np.full(w1.shape, 0.25), 1, 1), 0), 1e-4, k=kk)
    os.environ["LCU_NO_WEIGHT_CACHE"] = "1"
    try:
        per_run = run(w1)
    finally:
        del os.environ["LCU_NO_WEIGHT_CACHE"]
    assert np.array_equal(cached, per_run)

"""GPU parity of the per-op C ABI (lcu_*) against the FP64 oracle.

Tolerances: FP32-exact mode normwise rel <= 1e-4; TF32
fast mode <= 2e-2. Inputs are FP64 from the seeded generators, rounded to FP32
for the device; the oracle sees the FP64 values.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_close, rel_err
from lancius_b200 import EPI_GELU, EPI_NONE, EPI_RELU, MODE_FP32_EXACT, MODE_TF32, data, load

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return load()


_live = []


def dev(a):
    """device copy of `a`; kept alive for the module so a raw pointer taken from it
    stays valid (a temporary would go back to torch's caching allocator)."""
    t = torch.tensor(np.asarray(a, np.float32), device="cuda")
    _live.append(t)
    if len(_live) > 64:
        del _live[:32]
    return t


def P(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def run(rc):
    assert rc == 0, f"lancius error {rc}"
    torch.cuda.synchronize()


@pytest.mark.parametrize("M,K,N", [(64, 784, 256), (64, 256, 10), (1, 1, 1), (7, 13, 5), (130, 257, 129),
                                   (512, 768, 768), (256, 3072, 768), (1024, 1024, 1024), (33, 0, 17)])
@pytest.mark.parametrize("epi", [EPI_NONE, EPI_RELU, EPI_GELU])
def test_matmul(lib, orc, M, K, N, epi):
    a = data.uniform(1, (M, K), -1, 1)
    b = data.uniform(2, (K, N), -1, 1)
    bias = data.normal(3, (N,))
    ref = (orc.matmul(a, b) if K else np.zeros((M, N))) + bias
    if epi == EPI_RELU:
        ref = np.maximum(ref, 0)
    elif epi == EPI_GELU:
        ref = orc.gelu(ref)
    da, db, dbias = dev(a), dev(b), dev(bias)
    out = torch.empty((M, N), device="cuda")
    run(lib.lcu_matmul(P(out), P(da), P(db), M, K, N, P(dbias), epi, MODE_FP32_EXACT, None))
    assert_close(out.cpu().numpy(), ref, 1e-4, k=K)


@pytest.mark.parametrize("M,K,N", [(256, 16384, 256), (300, 4099, 130), (128, 64, 256), (1000, 2000, 3000)])
def test_matmul_tensor_core_exact(lib, orc, M, K, N):
    """3xTF32 path (these shapes are above the tensor-core threshold) stays within 1e-4
    even at K = 16384, the largest reduction of the GEMM sweep."""
    a = data.uniform(6, (M, K), -1, 1)
    b = data.uniform(7, (K, N), -1, 1)
    ref = orc.matmul(a, b)
    out = torch.empty((M, N), device="cuda")
    run(lib.lcu_matmul(P(out), P(dev(a)), P(dev(b)), M, K, N, None, EPI_NONE, MODE_FP32_EXACT, None))
    assert_close(out.cpu().numpy(), ref, 1e-4, k=min(K, 8192))   # K > 8192 is split, partials summed


@pytest.mark.parametrize("M,K,N", [(512, 768, 3072), (2048, 2048, 2048)])
def test_matmul_tf32_mode(lib, orc, M, K, N):
    a = data.uniform(4, (M, K), -1, 1)
    b = data.uniform(5, (K, N), -1, 1)
    ref = orc.matmul(a, b)
    out = torch.empty((M, N), device="cuda")
    run(lib.lcu_matmul(P(out), P(dev(a)), P(dev(b)), M, K, N, None, EPI_NONE, MODE_TF32, None))
    assert_close(out.cpu().numpy(), ref, 2e-2)


@pytest.mark.parametrize("B,S,H,D,causal", [(1, 64, 1, 64, 1), (2, 100, 3, 64, 1), (8, 512, 8, 64, 1),
                                            (2, 512, 12, 64, 0), (1, 200, 2, 128, 0), (1, 1, 1, 64, 1),
                                            # tcgen05 path: odd tile count (unpaired middle tile), a
                                            # ragged last tile, and more tile pairs than SMs (several
                                            # items per persistent CTA), causal and not
                                            (1, 300, 3, 64, 1), (2, 129, 2, 64, 1), (10, 256, 20, 64, 1),
                                            (10, 256, 20, 64, 0), (1, 1000, 2, 64, 1)])
def test_attention(lib, orc, B, S, H, D, causal):
    q = data.normal(11, (B, S, H, D))
    k = data.normal(12, (B, S, H, D))
    v = data.normal(13, (B, S, H, D))
    ref = np.stack([orc.attention(q[i], k[i], v[i], bool(causal)) for i in range(B)])
    out = torch.empty((B, S, H, D), device="cuda")
    run(lib.lcu_attention(P(out), P(dev(q)), P(dev(k)), P(dev(v)), B, S, H, D, causal, MODE_FP32_EXACT, None))
    y = out.cpu().numpy()
    assert_close(y, ref, 1e-4)


@pytest.mark.parametrize("growth,causal", [(0.02, 1), (0.02, 0)])
def test_attention_running_max_raised(lib, orc, growth, causal):
    """Scores that grow along the keys raise a row's running max after its first key tile, so
    O is rescaled in TMEM mid-item. The scores reach ~40 (natural units), so their FP32
    rounding alone (~|s| * 2^-23 per term) moves outputs by a few 1e-6 of max|ref|: the
    elementwise abs term is 1e-5 here, the normwise bound stays 1e-4."""
    B, S, H, D = 2, 512, 4, 64
    q = data.normal(17, (B, S, H, D))
    k = data.normal(18, (B, S, H, D)) * (1.0 + growth * np.arange(S))[None, :, None, None]
    v = data.normal(19, (B, S, H, D))
    ref = np.stack([orc.attention(q[i], k[i], v[i], bool(causal)) for i in range(B)])
    out = torch.empty((B, S, H, D), device="cuda")
    run(lib.lcu_attention(P(out), P(dev(q)), P(dev(k)), P(dev(v)), B, S, H, D, causal, MODE_FP32_EXACT, None))
    assert_close(out.cpu().numpy(), ref, 1e-4, elem_abs=1e-5)


@pytest.mark.parametrize("M,K,N", [(1024, 3072, 768), (520, 768, 1000)])
def test_matmul_tile_widths(lib, orc, M, K, N):
    """The tensor-core GEMM's 256 x 192 tiles (chosen when they take fewer rounds of the SMs,
    as for the encoder's FFN2 / O-projection shapes) and its 256 x 256 tiles, forced by
    LCU_GEMM_BN: both match the FP64 reference, ragged N included."""
    import os
    a = data.uniform(31, (M, K), -1, 1)
    b = data.uniform(32, (K, N), -1, 1)
    bias = data.normal(33, (N,))
    ref = np.maximum(orc.matmul(a, b) + bias, 0)
    outs = []
    for bn in ("192", "256"):
        os.environ["LCU_GEMM_BN"] = bn
        try:
            out = torch.empty((M, N), device="cuda")
            run(lib.lcu_matmul(P(out), P(dev(a)), P(dev(b)), M, K, N, P(dev(bias)), EPI_RELU, MODE_FP32_EXACT, None))
            outs.append(out.cpu().numpy())
        finally:
            del os.environ["LCU_GEMM_BN"]
        assert_close(outs[-1], ref, 1e-4, k=K)


@pytest.mark.parametrize("M,K,N", [(512, 768, 3072), (2048, 2048, 2048), (300, 1000, 260), (4096, 16384, 256)])
def test_matmul_bf16_mode(lib, orc, M, K, N):
    """BF16 fast mode: both operands rounded to BF16, tcgen05 kind::f16, FP32 accumulate
    (normwise 2e-2); odd K and N exercise the zero padding of the K-major BF16 copies,
    K = 16384 the split-K reduction."""
    from lancius_b200 import MODE_BF16
    a = data.uniform(8, (M, K), -1, 1)
    b = data.uniform(9, (K, N), -1, 1)
    bias = data.normal(10, (N,))
    ref = np.maximum(orc.matmul(a, b) + bias, 0)
    out = torch.empty((M, N), device="cuda")
    run(lib.lcu_matmul(P(out), P(dev(a)), P(dev(b)), M, K, N, P(dev(bias)), EPI_RELU, MODE_BF16, None))
    err = assert_close(out.cpu().numpy(), ref, 2e-2)
    assert err > 1e-5          # BF16 operands really were used


@pytest.mark.parametrize("B,S,H,causal", [(8, 512, 8, 1), (2, 512, 12, 0), (1, 300, 3, 1)])
def test_attention_tf32_mode(lib, orc, B, S, H, causal):
    """The one-pass TF32 fast mode of the tensor-core attention (normwise 2e-2)."""
    D = 64
    q, k, v = (data.normal(s, (B, S, H, D)) for s in (14, 15, 16))
    ref = np.stack([orc.attention(q[i], k[i], v[i], bool(causal)) for i in range(B)])
    out = torch.empty((B, S, H, D), device="cuda")
    run(lib.lcu_attention(P(out), P(dev(q)), P(dev(k)), P(dev(v)), B, S, H, D, causal, MODE_TF32, None))
    err = assert_close(out.cpu().numpy(), ref, 2e-2)
    assert err > 1e-6          # the single pass really ran (FP32-exact stays near 1e-7)


@pytest.mark.parametrize("shape", [(2, 3, 17, 19, 8, 3, 3, 1, 1), (2, 64, 28, 28, 128, 3, 3, 2, 1),
                                   (4, 3, 64, 64, 64, 3, 3, 1, 1), (2, 128, 30, 30, 256, 3, 3, 2, 1),
                                   (3, 64, 25, 25, 128, 3, 3, 1, 1),
                                   (1, 3, 32, 32, 6, 5, 5, 1, 2), (4, 5, 9, 9, 7, 1, 1, 1, 0),
                                   # direct NHWC implicit-GEMM path (Ci % 16 == 0, Wo % 8 == 0)
                                   (2, 64, 32, 32, 128, 3, 3, 1, 1), (4, 32, 64, 64, 64, 3, 3, 2, 1),
                                   (3, 16, 24, 24, 200, 3, 3, 1, 1), (2, 64, 48, 48, 96, 1, 1, 1, 0),
                                   (2, 16, 64, 64, 48, 5, 5, 2, 2),
                                   # register-blocked short-reduction stems (4 pixels x 16 channels a thread)
                                   (2, 3, 30, 32, 32, 3, 3, 2, 1), (1, 1, 16, 16, 16, 3, 3, 1, 1), (2, 3, 20, 24, 48, 1, 1, 1, 0)])
@pytest.mark.parametrize("relu", [0, 1])
def test_conv2d(lib, orc, shape, relu):
    N, Ci, H, W, Co, Kh, Kw, s, p = shape
    x = data.normal(21, (N, Ci, H, W))
    w = data.normal(22, (Co, Ci, Kh, Kw), 0, np.sqrt(2.0 / (Ci * Kh * Kw)))
    ref = orc.conv2d(x, w, s, p, bool(relu))
    out = torch.empty(ref.shape, device="cuda")
    run(lib.lcu_conv2d(P(out), P(dev(x)), P(dev(w)), N, Ci, H, W, Co, Kh, Kw, s, p, relu, MODE_FP32_EXACT, None))
    assert_close(out.cpu().numpy(), ref, 1e-4, k=Ci * Kh * Kw)


@pytest.mark.parametrize("shape", [(2, 3, 40, 44, 64, 3, 3, 1, 1), (3, 3, 37, 29, 32, 3, 3, 2, 1),
                                   (2, 1, 33, 35, 128, 3, 3, 1, 0), (2, 3, 21, 23, 96, 1, 1, 1, 0)])
@pytest.mark.parametrize("relu", [0, 1])
def test_conv_small_tc_nhwc(lib, orc, shape, relu):
    """The tensor-core stem conv (K = Ci*Kh*Kw <= 32, 3xTF32) that feeds an NHWC conv:
    ragged pixel counts (P % 128 != 0), stride 2, no padding, Co = 32..128. Its NHWC output
    matches the FP64 reference, and its lo copy is exactly tf32_lo of every output."""
    N, Ci, H, W, Co, Kh, Kw, s, p = shape
    f = lib.lcu_conv2d_small_tc_nhwc
    f.restype = C.c_int
    f.argtypes = [C.c_void_p] * 4 + [C.c_size_t] * 9 + [C.c_int, C.c_int, C.c_void_p]
    x = data.normal(23, (N, Ci, H, W))
    w = data.normal(24, (Co, Ci, Kh, Kw), 0, np.sqrt(2.0 / (Ci * Kh * Kw)))
    ref = orc.conv2d(x, w, s, p, bool(relu))
    Ho, Wo = ref.shape[2], ref.shape[3]
    out = torch.empty((N, Ho, Wo, Co), device="cuda")
    lo = torch.empty((N, Ho, Wo, Co), device="cuda")
    run(f(P(out), P(lo), P(dev(x)), P(dev(w)), N, Ci, H, W, Co, Kh, Kw, s, p, relu, MODE_FP32_EXACT, None))
    y = np.ascontiguousarray(out.cpu().numpy().transpose(0, 3, 1, 2))
    assert_close(y, ref, 1e-4, k=Ci * Kh * Kw)
    hi = (y.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
    d = (y - hi).view(np.uint32)
    want = ((d + np.uint32(0x1000)) & np.uint32(0xFFFFE000)).view(np.float32)   # round to nearest TF32
    assert np.array_equal(np.ascontiguousarray(lo.cpu().numpy().transpose(0, 3, 1, 2)), want)


@pytest.mark.parametrize("shape", [(2, 64, 32, 32, 128, 3, 3, 1, 1), (2, 16, 64, 64, 48, 5, 5, 2, 2)])
def test_conv2d_split_on_chip_matches_split_pass(lib, shape):
    """The direct conv splits its NHWC input tiles into TF32 hi/lo on chip; the result is
    bit-identical to splitting the whole input first (LCU_NO_RAW_A=1)."""
    import os
    N, Ci, H, W, Co, Kh, Kw, s, p = shape
    x, w = dev(data.normal(23, (N, Ci, H, W))), dev(data.normal(24, (Co, Ci, Kh, Kw)))
    Ho, Wo = (H + 2 * p - Kh) // s + 1, (W + 2 * p - Kw) // s + 1
    outs = []
    for flag in ("0", "1"):
        os.environ["LCU_NO_RAW_A"] = flag
        try:
            out = torch.empty((N, Co, Ho, Wo), device="cuda")
            run(lib.lcu_conv2d(P(out), P(x), P(w), N, Ci, H, W, Co, Kh, Kw, s, p, 1, MODE_FP32_EXACT, None))
            outs.append(out.cpu().numpy())
        finally:
            del os.environ["LCU_NO_RAW_A"]
    assert np.array_equal(outs[0], outs[1])


@pytest.mark.parametrize("rows,hidden", [(8192, 768), (3, 10), (17, 2048), (5, 3000)])
def test_layernorm(lib, orc, rows, hidden):
    x = data.normal(31, (rows, hidden), 0.5, 2.0)
    gma = data.normal(32, (hidden,), 1.0, 0.1)
    bta = data.normal(33, (hidden,))
    ref = orc.layernorm(x, gma, bta)
    out = torch.empty((rows, hidden), device="cuda")
    run(lib.lcu_layernorm(P(out), P(dev(x)), P(dev(gma)), P(dev(bta)), rows, hidden, C.c_float(1e-5), None))
    assert_close(out.cpu().numpy(), ref, 1e-4)


def test_softmax_gelu_tanh_relu(lib, orc):
    x = data.normal(41, (64, 10), 0, 3)
    o = torch.empty((64, 10), device="cuda")
    run(lib.lcu_softmax(P(o), P(dev(x)), 64, 10, None))
    assert_close(o.cpu().numpy(), orc.softmax(x), 1e-5)
    y = data.normal(42, (1000003,), 0, 4)
    y[:4] = [150.0, -150.0, 0.0, 1e-3]
    dy = dev(y)
    o = torch.empty(y.shape, device="cuda")
    run(lib.lcu_gelu(P(o), P(dy), y.size, None))
    assert_close(o.cpu().numpy(), orc.gelu(y), 1e-5)
    run(lib.lcu_tanh(P(o), P(dy), y.size, None))
    assert_close(o.cpu().numpy(), np.tanh(y), 1e-5)
    run(lib.lcu_relu(P(o), P(dy), y.size, None))
    assert np.array_equal(o.cpu().numpy(), np.maximum(y.astype(np.float32), 0))


def test_elementwise_exact(lib):
    for n in (1, 3, 4, 1023, 1 << 20):
        a = data.normal(51, (n,)).astype(np.float32)
        b = data.normal(52, (n,)).astype(np.float32)
        da, db = dev(a), dev(b)
        o = torch.empty(n, device="cuda")
        for fn, ref in ((lib.lcu_add, a + b), (lib.lcu_sub, a - b), (lib.lcu_mul, a * b)):
            run(fn(P(o), P(da), P(db), n, None))
            assert np.array_equal(o.cpu().numpy(), ref)
    # misaligned views take the scalar path
    a = data.normal(53, (1001,)).astype(np.float32)
    da = dev(a)
    o = torch.empty(1001, device="cuda")
    run(lib.lcu_add(C.c_void_p(o.data_ptr() + 4), C.c_void_p(da.data_ptr() + 4), C.c_void_p(da.data_ptr() + 4), 1000, None))
    assert np.array_equal(o.cpu().numpy()[1:], a[1:] * 2)


def test_broadcast_fill_sum_maxpool(lib, orc):
    v = data.normal(61, (7,)).astype(np.float32)
    o = torch.empty((5, 7), device="cuda")
    run(lib.lcu_broadcast(P(o), P(dev(v)), 7, 5, 7, None))
    assert np.array_equal(o.cpu().numpy(), np.tile(v, (5, 1)))
    run(lib.lcu_broadcast(P(o), P(dev(v[:1])), 1, 35, 1, None))
    assert np.all(o.cpu().numpy() == v[0])
    run(lib.lcu_fill(P(o), C.c_float(2.5), 35, None))
    assert np.all(o.cpu().numpy() == 2.5)
    x = data.normal(62, (8192, 3136))
    s = torch.empty(8192, device="cuda")
    run(lib.lcu_sum_axis1(P(s), P(dev(x)), 8192, 3136, None))
    assert_close(s.cpu().numpy(), x.sum(1), 1e-5)
    x = data.normal(63, (2, 3, 9, 8))
    ref = orc.maxpool2d(x, 2, 2)
    o = torch.empty(ref.shape, device="cuda")
    run(lib.lcu_maxpool2d(P(o), P(dev(x)), 2, 3, 9, 8, 2, 2, None))
    assert np.array_equal(o.cpu().numpy(), ref.astype(np.float32))


def test_bad_arguments(lib):
    x = torch.zeros(16, device="cuda")
    assert lib.lcu_matmul(None, P(x), P(x), 4, 4, 4, None, 0, 0, None) == -2
    assert lib.lcu_matmul(P(x), P(x), P(x), 4, 1, 4, None, 7, 0, None) == -4
    assert lib.lcu_attention(P(x), P(x), P(x), P(x), 1, 1, 1, 48, 1, 0, None) == -4
    assert lib.lcu_conv2d(P(x), P(x), P(x), 1, 1, 1, 1, 1, 3, 3, 1, 0, 0, 0, None) == -3

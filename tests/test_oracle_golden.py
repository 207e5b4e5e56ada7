"""The FP64 oracle pinned against the reference's own known answers and against
the reference library itself (compiled from its sources by oracle/Makefile)."""
import ctypes as C
import ctypes.util

import numpy as np
import pytest

import lancius_b200 as L
from lancius_b200 import configs, data
import oracle


def glibc_rand_inputs(n, seed=42):
    """q, k, v exactly as stable/v9S/examples/audit_flash_attention.c:72-77 draws them
    (srand(42); per element q, k, v from rand()/RAND_MAX*2-1)."""
    libc = C.CDLL(ctypes.util.find_library("c"))
    libc.srand(seed)
    r = np.array([libc.rand() for _ in range(3 * n)], dtype=np.float64) / 2147483647.0 * 2.0 - 1.0
    return r[0::3].copy(), r[1::3].copy(), r[2::3].copy()


def test_flash_attention_known_answer(orc):
    """audit_flash_attention.c:56-95: flash == naive causal attention, max |d| < 1e-5, S512 H8 D64."""
    S, H, D = 512, 8, 64
    q, k, v = (x.reshape(S, H, D) for x in glibc_rand_inputs(S * H * D))
    flash = orc.attention(q, k, v, causal=True)
    naive = orc.naive_attention(q, k, v)
    assert np.max(np.abs(flash - naive)) < 1e-5


def test_flash_attention_matches_reference_kernel(orc, ref):
    S, H, D = 128, 4, 64
    q, k, v = (data.normal(s, (S, H, D)) for s in (1, 2, 3))
    out = np.empty((S, H, D))
    dp = lambda a: a.ctypes.data_as(C.POINTER(C.c_double))
    ref.kernel_attention(dp(out), dp(np.ascontiguousarray(q)), dp(np.ascontiguousarray(k)),
                         dp(np.ascontiguousarray(v)), C.c_size_t(S), C.c_size_t(H), C.c_size_t(D))
    assert np.max(np.abs(orc.attention(q, k, v) - out)) < 1e-12


def test_ffi_known_answer(orc):
    """stable/v9S/examples/audit_ffi.c:35-61: MatMul(2x3, ones 3x4) -> ReLU == [4,4,4,4,5,5,5,5]."""
    g = L.Graph()
    a, b = g.input(2, 3), g.input(3, 4)
    d = g.relu(g.matmul(a, b))
    g.bind(a, np.array([-1.0, 2, 3, 4, -5, 6]))
    g.bind(b, np.ones(12))
    assert orc.run_graph(g, [d])[d.id].ravel().tolist() == [4.0] * 4 + [5.0] * 4


def test_rmsnorm_known_answer(orc):
    """stable/v9S/examples/audit_modern_llm.c:29-35: RMSNorm(ones, gamma=2) == 2."""
    y = orc.rmsnorm(np.ones((4, 16)), np.full(16, 2.0))
    assert np.allclose(y, 2.0, atol=1e-6)


@pytest.mark.parametrize("build", [
    lambda g: configs.mlp(g),
    lambda g: configs.attention(g, batch=2, seq=96, heads=2),
    lambda g: configs.conv_stack(g, batch=1, hw=20),
    # encoder-shaped: LAYERNORM, GELU, residual ADD, causal ATTENTION (the only kind the
    # reference has); pins the oracle's layernorm (lancius_kernels.c:217-236) and GELU (:238-246)
    lambda g: configs.encoder(g, batch=2, seq=24, layers=2, d_model=64, heads=4, ffn=128, causal=True),
])
def test_oracle_graph_equals_reference_executor(orc, ref, build):
    """Same graph built with this library and with the reference library; the oracle's
    arena-mode run must equal the reference's own lancius_schedule_execute."""
    g1 = L.Graph()
    b1 = build(g1)
    b1.bind_host()
    mine = orc.run_graph(g1, b1.outputs)
    g2 = L.Graph(ref)
    b2 = build(g2)
    b2.bind_host()
    theirs = oracle.run_reference_graph(ref, g2, b2.outputs)
    for o1, o2 in zip(b1.outputs, b2.outputs):
        r = theirs[o2.id]
        assert np.max(np.abs(mine[o1.id] - r)) <= 1e-12 * max(1.0, np.max(np.abs(r)))


ENCODER_GOLDEN = lambda g: configs.encoder(g, batch=2, seq=24, layers=2, d_model=64, heads=4,
                                            ffn=128, causal=True)


def test_committed_golden_fixtures(orc):
    """tests/golden/*.npz were produced by the reference library (make_golden.py)."""
    import os
    here = os.path.join(os.path.dirname(__file__), "golden")
    for name, build in (("mlp", lambda g: configs.mlp(g)),
                        ("attention_b2_s96_h2", lambda g: configs.attention(g, batch=2, seq=96, heads=2)),
                        ("conv_b1_hw20", lambda g: configs.conv_stack(g, batch=1, hw=20)),
                        ("encoder_causal_b2_s24_l2", ENCODER_GOLDEN)):
        fx = np.load(os.path.join(here, f"{name}.npz"))
        g = L.Graph()
        b = build(g)
        b.bind_host()
        got = orc.run_graph(g, b.outputs)
        for i, o in enumerate(b.outputs):
            want = fx[f"out{i}"]
            assert np.max(np.abs(got[o.id] - want)) <= 1e-12 * max(1.0, np.max(np.abs(want)))


def test_layernorm_gelu_oracle_equals_reference_kernels(orc, ref):
    """orc.layernorm / orc.gelu against the reference's kernel_layernorm and kernel_gelu
    (lancius_kernels.c:217-246) called directly, including GELU's +-100 clamp and a
    constant row (zero variance)."""
    dp = lambda a: a.ctypes.data_as(C.POINTER(C.c_double))
    rows, hid = 37, 768
    x = data.normal(11, (rows, hid), 0.0, 3.0)
    x[5, :] = 2.5
    gamma, beta = data.normal(12, (hid,)), data.normal(13, (hid,))
    out = np.empty_like(x)
    ref.kernel_layernorm(dp(out), dp(x), dp(gamma), dp(beta), C.c_size_t(rows), C.c_size_t(hid), C.c_double(1e-5))
    assert np.max(np.abs(orc.layernorm(x, gamma, beta) - out)) <= 1e-12 * np.max(np.abs(out))
    xg = np.concatenate([data.normal(14, (4096,), 0.0, 4.0), [-150.0, -100.0, -99.9, 0.0, 99.9, 100.0, 150.0]])
    outg = np.empty_like(xg)
    ref.kernel_gelu(dp(outg), dp(xg), C.c_size_t(xg.size))
    assert np.max(np.abs(orc.gelu(xg) - outg)) <= 1e-12 * np.max(np.abs(outg))

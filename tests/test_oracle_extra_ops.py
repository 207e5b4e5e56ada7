"""Oracle restatements of the training, LLM and INT8 operators against the reference's
own executor (same graph built with both libraries)."""
import numpy as np
import pytest

import lancius_b200 as L
import opgraphs
import oracle


def run_both(orc, ref, build):
    outs = []
    for lib in (None, ref):
        g = L.Graph(lib)
        r = build(g)
        inputs, outputs = r[0], r[-1]
        for n, arr in inputs.items():
            g.bind(n, arr)
        if len(r) == 3:
            for n, (q, scale) in r[1].items():
                g.bind_int8(n, q, scale)
        if lib is None:
            res = orc.run_graph(g, outputs)
        else:
            res = oracle.run_reference_graph(ref, g, outputs)
        outs.append([res[o.id] for o in outputs])
        outs[-1].append(g)
    return outs


@pytest.mark.parametrize("build", [opgraphs.training_ops, opgraphs.llm_ops, opgraphs.int8_matmul,
                                   opgraphs.int8_conv])
def test_extra_ops_match_reference(orc, ref, build):
    mine, theirs = run_both(orc, ref, build)
    for a, b in zip(mine[:-1], theirs[:-1]):
        assert a.shape == b.shape
        assert np.max(np.abs(a - b)) <= 1e-11 * max(1.0, np.max(np.abs(b)))


def test_rope_known_values(orc):
    q = np.zeros((1, 3, 1, 4)); k = np.zeros((1, 3, 1, 4))
    q[..., 0] = 1.0; k[..., 1] = 1.0
    import ctypes as C
    dp = lambda a: a.ctypes.data_as(C.POINTER(C.c_double))
    orc.lib.orc_rope(dp(q), dp(k), C.c_size_t(1), C.c_size_t(3), C.c_size_t(1), C.c_size_t(4), C.c_int(0))
    # position s rotates pair (0,1) by angle s (frequency 1)
    assert np.allclose(q[0, :, 0, 0], np.cos([0, 1, 2])) and np.allclose(q[0, :, 0, 1], np.sin([0, 1, 2]))
    assert np.allclose(k[0, :, 0, 0], -np.sin([0, 1, 2]))


@pytest.mark.parametrize("S,H,D", [(1, 2, 16), (37, 4, 64), (300, 3, 80)])
def test_kv_cache_attention_matches_reference(orc, ref, S, H, D):
    """orc_attention_kv_cache against the reference's kernel_attention_kv_cache
    (lancius_kernels.c:338-379) on the same FP64 inputs."""
    import ctypes as C
    from lancius_b200 import data
    q = data.normal(11, (H * D,)); kc = data.normal(12, (S, H, D)); vc = data.normal(13, (S, H, D))
    dp = lambda a: a.ctypes.data_as(C.POINTER(C.c_double))
    mine = np.empty(H * D); theirs = np.empty(H * D)
    orc.lib.orc_attention_kv_cache(dp(mine), dp(q), dp(kc), dp(vc), C.c_size_t(S), C.c_size_t(H), C.c_size_t(D))
    ref.kernel_attention_kv_cache(dp(theirs), dp(q), dp(kc), dp(vc), C.c_size_t(S), C.c_size_t(H), C.c_size_t(D))
    assert np.max(np.abs(mine - theirs)) <= 1e-12 * max(1.0, np.max(np.abs(theirs)))

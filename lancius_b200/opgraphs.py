"""Small graphs exercising the executor opcodes outside the five benchmark configs
(training and LLM operators, INT8 weights); shared by the parity tests."""
import numpy as np

from . import data


def training_ops(g, seed=5):
    """conv -> relu -> maxpool -> flatten -> matmul -> softmax cross entropy, and the
    backward nodes the reference autodiff emits (lancius_autodiff.c:44-207)."""
    x = g.input_4d(2, 3, 8, 8)
    w = g.input_4d(4, 3, 3, 3)
    conv = g.conv2d(x, w, 1, 1)
    act = g.relu(conv)
    pool = g.maxpool2d(act, 2, 2)
    flat = g.flatten(pool)                            # [2, 64]
    wf = g.input(64, 5)
    logits = g.matmul(flat, wf)                       # [2, 5]
    tgt = g.input(2, 5)
    loss = g.cross_entropy(logits, tgt)
    one = g.const(1.0, 1, 1)
    dlog = g.cross_entropy_bwd(logits, tgt, one)
    sm = g.softmax(logits)
    dsm = g.softmax_bwd(dlog, sm)
    dflat = g.matmul(dlog, g.transpose(wf))           # [2, 64]
    dpool = g.reshape(dflat, 2, 4, 4, 4)
    dact = g.maxpool2d_bwd(dpool, act, 2, 2)
    dconv = g.relu_bwd(dact, conv)
    dx = g.conv2d_bwd(dconv, x, w, 1, 1)
    dw = g.conv2d_bwd_w(dconv, x, 3, 3, 1, 1)
    colsum = g.sum_axis0(dlog)
    total = g.sum(dflat)
    inputs = {x: data.normal(seed, (2, 3, 8, 8)), w: data.normal(seed + 1, (4, 3, 3, 3), 0, 0.3),
              wf: data.normal(seed + 2, (64, 5), 0, 0.2), tgt: np.eye(5)[[1, 3]]}
    return inputs, [loss, dlog, dsm, dx, dw, colsum, total, dflat]


def llm_ops(g, seed=6, S=48, Hq=8, Hkv=2, D=64):
    q = g.reshape(g.input(S, Hq * D), S, Hq, D)
    k = g.reshape(g.input(S, Hkv * D), S, Hkv, D)
    v = g.reshape(g.input(S, Hkv * D), S, Hkv, D)
    att = g.gqa(q, k, v, Hq, Hkv)
    x = g.input(S, 96)
    gamma = g.input(1, 96)
    rms = g.rmsnorm(x, gamma)
    up = g.input(S, 96)
    sw = g.swiglu(rms, up)
    ins = [n for n in g.nodes() if n.op == "INPUT"]
    shapes = [n.shape for n in ins]
    inputs = {n: data.normal(seed + i, s) for i, (n, s) in enumerate(zip(ins, shapes))}
    return inputs, [att, rms, sw]


def int8_matmul(g, seed=7, M=33, K=70, N=20):
    """MATMUL whose B is INT8 with a per-tensor scale: the reference quantizes A on the
    fly (lancius_scheduler.c:195-220)."""
    a = g.input(M, K)
    b = g.input(K, N)
    out = g.matmul(a, b)
    wq = np.round(data.uniform(seed + 1, (K, N), -127, 127)).astype(np.int8)
    return {a: data.normal(seed, (M, K))}, {b: (wq, 0.01)}, [out]

"""Small graphs exercising the executor opcodes outside the five benchmark configs
(training and LLM operators, INT8 weights); shared by the parity tests."""
import numpy as np

from lancius_b200 import data


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


def int8_conv(g, seed=9, N=2, Ci=3, HW=20, Co=8, k=3, stride=1, pad=1, relu=True):
    """CONV2D (optionally ReLU-fused) with INT8 OIHW weights and a per-tensor scale:
    the reference quantizes the FP activation on the fly (lancius_vision_ops.c:16-57)."""
    x = g.input_4d(N, Ci, HW, HW)
    w = g.input_4d(Co, Ci, k, k)
    out = g.conv2d(x, w, stride, pad)
    if relu:
        out = g.relu(out)
        g.optimize_fusion()            # CONV2D_RELU_FUSED, as the reference's optimizer emits it
    wq = np.round(data.uniform(seed + 1, (Co, Ci, k, k), -127, 127)).astype(np.int8)
    return {x: data.normal(seed, (N, Ci, HW, HW))}, {w: (wq, 0.02)}, [out]


def int8_matmul_large(g):
    """INT8 MATMUL big enough for the tensor-core path (2^24+ multiply-adds)."""
    return int8_matmul(g, seed=17, M=300, K=520, N=390)


def int8_conv_large(g):
    """INT8 conv through the tensor-core implicit GEMM: K = 27 (re-pitched weights)."""
    return int8_conv(g, seed=19, N=4, Ci=3, HW=64, Co=64, k=3, stride=1, pad=1, relu=False)


def int8_conv_large_k144(g):
    """INT8 conv, K = 144 (16-byte rows as they are), stride 2, ReLU."""
    return int8_conv(g, seed=23, N=4, Ci=16, HW=64, Co=96, k=3, stride=2, pad=1, relu=True)

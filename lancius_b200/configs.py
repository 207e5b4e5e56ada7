"""The five benchmark configurations, built only through the Lancius graph API.

Each builder takes a Graph (this package's library or any library exporting the
Lancius IR) and returns a Built record: the graph, the INPUT nodes with their
seeded FP64 data, the output node(s) and the algorithmic work per graph. The
formulations (bias as ADD(BROADCAST), GAP as RESHAPE->SUM_AXIS1->MUL(CONST)->RESHAPE,
one subgraph per batch element for attention) are the ones the reference IR can
express unchanged.
"""
from dataclasses import dataclass, field

import numpy as np

from . import data


@dataclass
class Built:
    name: str
    graph: object
    inputs: list = field(default_factory=list)      # [(Node, ndarray float64)]
    outputs: list = field(default_factory=list)     # [Node]
    flops: float = 0.0                              # algorithmic FLOPs per graph execution
    bytes: float = 0.0                              # algorithmic HBM bytes (FP32) per execution
    meta: dict = field(default_factory=dict)

    def bind_host(self):
        for node, arr in self.inputs:
            self.graph.bind(node, arr)


def _inp(b, node, arr):
    b.inputs.append((node, np.ascontiguousarray(arr, dtype=np.float64)))
    return node


def _linear(g, b, x, w_arr, bias_arr, rows):
    """x[rows, K] @ W[K, N] + bias, bias added through BROADCAST + ADD."""
    K, N = w_arr.shape
    w = _inp(b, g.input(K, N), w_arr)
    bias = _inp(b, g.input(1, N), bias_arr.reshape(1, N))
    return g.add(g.matmul(x, w), g.broadcast(bias, rows, N))


def mlp(g, batch=64, seed=0, rows=None):
    """Config 1: 784 -> 256 (+bias, ReLU) -> 10 (+bias) -> softmax.
    rows=(start, stop) builds the graph for that block of the seeded batch (sharding)."""
    b = Built("mlp", g)
    xfull = data.uniform(seed, (batch, 784), 0.0, 1.0)
    if rows is not None:
        xfull = xfull[rows[0]:rows[1]]
        batch = xfull.shape[0]
    x = _inp(b, g.input(batch, 784), xfull)
    w1 = data.normal(data.sub_seed(seed, 1), (784, 256), 0.0, 1.0 / np.sqrt(784))
    w2 = data.normal(data.sub_seed(seed, 2), (256, 10), 0.0, 1.0 / np.sqrt(256))
    h = g.relu(_linear(g, b, x, w1, np.zeros(256), batch))
    out = g.softmax(_linear(g, b, h, w2, np.zeros(10), batch))
    b.outputs = [out]
    b.flops = 2.0 * batch * (784 * 256 + 256 * 10)
    b.bytes = 4.0 * (batch * 784 + 784 * 256 + 256 + 256 * 10 + 10 + batch * 10)
    return b


def attention(g, batch=8, seq=512, heads=8, head_dim=64, seed=1, causal=True):
    """Config 2: per batch element Q,K,V [S, H*D] -> [S,H,D] views -> ATTENTION -> [S, H*D]."""
    b = Built("attention", g)
    hd = heads * head_dim
    for e in range(batch):
        qkv = []
        for t in range(3):
            arr = data.normal(data.sub_seed(seed, 3 * e + t), (seq, hd))
            qkv.append(g.reshape(_inp(b, g.input(seq, hd), arr), seq, heads, head_dim))
        a = g.attention(*qkv) if causal else g.attention_noncausal(*qkv)
        b.outputs.append(g.reshape(a, seq, hd))
    pairs = seq * (seq + 1) / 2 if causal else seq * seq
    b.flops = 2.0 * 2.0 * batch * heads * head_dim * pairs
    b.bytes = 16.0 * batch * seq * hd
    b.meta = dict(batch=batch, seq=seq, heads=heads, head_dim=head_dim, causal=causal)
    return b


def conv_stack(g, batch=32, hw=224, seed=2, fuse=True, rows=None):
    """Config 3: three 3x3 conv+ReLU (3->64 s1, 64->128 s2, 128->256 s2), GAP, Linear 256->1000.
    rows=(start, stop) builds the graph for that block of the seeded batch's images."""
    b = Built("conv_stack", g)
    xfull = data.normal(seed, (batch, 3, hw, hw))
    if rows is not None:
        xfull = xfull[rows[0]:rows[1]]
        batch = xfull.shape[0]
    x = _inp(b, g.input_4d(batch, 3, hw, hw), xfull)
    layers = [(3, 64, 1), (64, 128, 2), (128, 256, 2)]
    flops = 0.0
    h, cur = x, hw
    for i, (ci, co, s) in enumerate(layers):
        fan = ci * 9
        w = _inp(b, g.input_4d(co, ci, 3, 3), data.normal(data.sub_seed(seed, i + 1), (co, ci, 3, 3), 0.0, np.sqrt(2.0 / fan)))
        h = g.relu(g.conv2d(h, w, s, 1))
        cur = (cur + 2 - 3) // s + 1
        flops += 2.0 * batch * co * cur * cur * ci * 9
    C = layers[-1][1]
    flat = g.reshape(h, batch * C, cur * cur)
    mean = g.mul(g.sum_axis1(flat), g.const(1.0 / (cur * cur), batch * C, 1))
    pooled = g.reshape(mean, batch, C)
    wfc = data.normal(data.sub_seed(seed, 9), (C, 1000), 0.0, np.sqrt(2.0 / C))
    b.outputs = [_linear(g, b, pooled, wfc, np.zeros(1000), batch)]
    if fuse:
        g.optimize_fusion()
    b.flops = flops + 2.0 * batch * C * 1000
    b.meta = dict(batch=batch, hw=hw)
    return b


def encoder(g, batch=16, seq=512, layers=12, d_model=768, heads=12, ffn=3072, seed=3, first=0, causal=False):
    """Config 4: pre-LN BERT-shape encoder, GELU FFN, unmasked attention, eps 1e-5.

    One subgraph per batch element (the IR has no slice op); weight INPUT nodes are
    shared by all batch elements. `first` numbers the batch elements from there (a
    rank's shard of a larger batch draws the same sequences as the full batch)."""
    b = Built("encoder", g)
    hd = d_model // heads
    xs = [_inp(b, g.input(seq, d_model), data.normal(data.sub_seed(seed, 100000 + first + e), (seq, d_model)))
          for e in range(batch)]
    k = 0

    def wt(shape, std=0.02):
        nonlocal k
        k += 1
        return data.normal(data.sub_seed(seed, k), shape, 0.0, std)

    def vec(arr_or_n, fill=0.0):
        n = arr_or_n
        return _inp(b, g.input(1, n), np.full((1, n), fill))

    for _ in range(layers):
        g1, be1, g2, be2 = vec(d_model, 1.0), vec(d_model), vec(d_model, 1.0), vec(d_model)
        W = {nm: _inp(b, g.input(*shp), wt(shp)) for nm, shp in
             [("q", (d_model, d_model)), ("k", (d_model, d_model)), ("v", (d_model, d_model)),
              ("o", (d_model, d_model)), ("f1", (d_model, ffn)), ("f2", (ffn, d_model))]}
        B = {nm: vec(n) for nm, n in [("q", d_model), ("k", d_model), ("v", d_model), ("o", d_model),
                                      ("f1", ffn), ("f2", d_model)]}

        def lin(x, nm, n):
            return g.add(g.matmul(x, W[nm]), g.broadcast(B[nm], seq, n))

        for e in range(batch):
            x = xs[e]
            h = g.layernorm(x, g1, be1)
            q, kk, v = (g.reshape(lin(h, nm, d_model), seq, heads, hd) for nm in ("q", "k", "v"))
            att = g.attention(q, kk, v) if causal else g.attention_noncausal(q, kk, v)
            a = g.reshape(att, seq, d_model)
            o = g.add(lin(a, "o", d_model), x)
            h2 = g.layernorm(o, g2, be2)
            f = g.gelu(lin(h2, "f1", ffn))
            xs[e] = g.add(lin(f, "f2", d_model), o)
    b.outputs = xs
    M = batch * seq
    b.flops = layers * (2.0 * M * d_model * (4 * d_model + 2 * ffn) + 4.0 * batch * heads * seq * seq * hd)
    b.meta = dict(batch=batch, seq=seq, layers=layers, d_model=d_model, heads=heads, ffn=ffn)
    return b


def gemm(g, n, seed=4):
    """Config 5: square C = A * B with A, B ~ U[-1, 1)."""
    b = Built(f"gemm{n}", g)
    a = _inp(b, g.input(n, n), data.uniform(data.sub_seed(seed, 1), (n, n), -1.0, 1.0))
    w = _inp(b, g.input(n, n), data.uniform(data.sub_seed(seed, 2), (n, n), -1.0, 1.0))
    b.outputs = [g.matmul(a, w)]
    b.flops = 2.0 * n ** 3
    b.bytes = 12.0 * n * n
    return b

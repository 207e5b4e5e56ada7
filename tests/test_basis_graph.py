"""BASIS stage-6 graph API: node tables identical to the reference's own builder
(src/basis/stage6_ir/graph.c), and its lowering onto the Lancius IR computes the BASIS
semantics (checked on the oracle here, on the GPU in test_gpu_graph.py)."""
import numpy as np
import pytest

import oracle
from lancius_b200 import data
from lancius_b200.basis import BasisGraph


def build_mlp(g, depth=6):
    """An MLP-shaped BASIS graph: matmul + broadcast bias, relu / tanh, a residual add,
    plus rejected shapes; more than 16 nodes so the node array grows."""
    x = g.input("x", 5, 8)
    h = x
    ids = {"x": x, "w": [], "b": []}
    for i in range(depth):
        w = g.input(f"w{i}", 8, 8)
        b = g.input(f"b{i}", 1, 8)
        ids["w"].append(w); ids["b"].append(b)
        z = g.broadcast_add(g.matmul(h, w), b)
        h = g.add(g.tanh(z) if i % 2 else g.relu(z), h)
    bad = [g.matmul(x, ids["b"][0]), g.add(x, ids["w"][0]), g.broadcast_add(x, ids["w"][0])]
    return h, ids, bad


def test_node_table_matches_reference():
    ref = oracle.basis_reference()
    if ref is None:
        pytest.skip("reference BASIS library (oracle/_ref) not built here")
    mine, theirs = BasisGraph(), BasisGraph(ref)
    m = build_mlp(mine)
    t = build_mlp(theirs)
    assert m[2] == t[2] == [None, None, None]
    assert mine.nodes() == theirs.nodes()
    assert len(mine.nodes()) > 16


def test_lowering_computes_basis_semantics(orc):
    g = BasisGraph()
    out, ids, _ = build_mlp(g)
    lg, m = g.lower()
    rng_inputs = {}
    x = data.normal(41, (5, 8)); rng_inputs[ids["x"]] = x
    for i, (w, b) in enumerate(zip(ids["w"], ids["b"])):
        rng_inputs[w] = data.normal(42 + i, (8, 8), 0, 0.5)
        rng_inputs[b] = data.normal(60 + i, (1, 8))
    for bid, arr in rng_inputs.items():
        lg.bind(m[bid], arr)
    got = orc.run_graph(lg, [m[out]])[m[out].id]
    h = x
    for i in range(len(ids["w"])):
        z = h @ rng_inputs[ids["w"][i]] + rng_inputs[ids["b"][i]]
        h = (np.tanh(z) if i % 2 else np.maximum(z, 0.0)) + h
    assert np.max(np.abs(got - h)) <= 1e-12 * max(1.0, np.max(np.abs(h)))

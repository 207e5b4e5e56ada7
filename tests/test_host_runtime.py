"""Host runtime (C11): IR builders, wave scheduler and memory planner against the
reference library, plus the planner's non-overlap guarantee. CPU only."""
import ctypes as C

import numpy as np
import pytest

import lancius_b200 as L
from lancius_b200 import _abi, configs, data
import oracle

BUILDS = {
    "mlp": lambda g: configs.mlp(g),
    "attention": lambda g: configs.attention(g, batch=3, seq=64, heads=2),
    "conv": lambda g: configs.conv_stack(g, batch=2, hw=16),
    "encoder": lambda g: configs.encoder(g, batch=2, seq=16, layers=2, d_model=32, heads=2, ffn=64),
}


def structure(g):
    out = []
    for n in g.nodes():
        c = n.c
        ins = [c.inputs[i].contents.id if False else C.cast(c.inputs[i], _abi.NODE_P).contents.id
               for i in range(c.input_count)]
        out.append((n.id, c.op, n.shape, (c.kernel_h, c.kernel_w, c.stride, c.pad), c.attr_val, tuple(ins)))
    return out


@pytest.mark.parametrize("name", ["mlp", "attention", "conv"])
def test_ir_and_waves_match_reference(ref, name):
    ours, theirs = L.Graph(), L.Graph(ref)
    BUILDS[name](ours)
    BUILDS[name](theirs)
    assert structure(ours) == structure(theirs)
    assert ours.schedule().waves() == theirs.schedule().waves()


def test_builder_error_paths(ref):
    for lib in (None, ref):
        g = L.Graph(lib)
        a, b = g.input(2, 3), g.input(4, 5)
        with pytest.raises(L.LanciusError):
            g.matmul(a, b)                       # inner dims differ -> NULL
        x = g.input_4d(1, 3, 8, 8)
        w = g.input_4d(4, 2, 3, 3)
        with pytest.raises(L.LanciusError):
            g.conv2d(x, w, 1, 1)                 # channel mismatch -> NULL
        with pytest.raises(L.LanciusError):
            g.softmax(x)                         # softmax needs rank 2


def _plan(g, sched, fn="lancius_build_memory_plan"):
    return getattr(g.lib, fn)(sched.ptr, g.ptr)


@pytest.mark.parametrize("name", list(BUILDS))
def test_planner_no_overlap(name):
    g = L.Graph()
    BUILDS[name](g)
    s = g.schedule()
    for elem, views in ((0, 0), (4, 0), (4, 1)):
        p = g.lib.lancius_build_memory_plan_ex(s.ptr, g.ptr, elem, 256, views)
        assert p
        assert g.lib.lancius_memory_plan_validate(p, s.ptr, g.ptr, elem) == 0
        assert p.contents.peak_memory > 0
        g.lib.lancius_memory_plan_destroy(p)


def test_reference_planner_aliases_live_tensors(ref):
    """The reference planner (lancius_memory_planner.c:122-127,140,162) hands live bytes
    to new tensors; the validator catches it on the MLP graph, ours does not."""
    gr = L.Graph(ref)
    configs.mlp(gr)
    sr = gr.schedule()
    bad = ref.lancius_build_memory_plan(sr.ptr, gr.ptr)
    # validate the reference's plan with our validator (same struct layout, same graph layout)
    lib = L.load()
    assert lib.lancius_memory_plan_validate(C.cast(bad, _abi.PLAN_P), C.cast(sr.ptr, _abi.SCHED_P),
                                            C.cast(gr.ptr, _abi.GRAPH_P), 0) != 0
    ref.lancius_memory_plan_destroy(bad)
    g = L.Graph()
    configs.mlp(g)
    s = g.schedule()
    good = g.lib.lancius_build_memory_plan(s.ptr, g.ptr)
    assert g.lib.lancius_memory_plan_validate(good, s.ptr, g.ptr, 0) == 0
    g.lib.lancius_memory_plan_destroy(good)


def test_planned_pool_gives_reference_results(ref):
    """Our plan drives the REFERENCE CPU executor through its own attach_pool path and
    reproduces the arena-mode answer exactly. The reference's own plan does not: it lets
    tensors that are alive together share pool bytes, and the output differs by more than 1e-3."""
    lib = L.load()
    for planner in ("ours", "reference"):
        g = L.Graph(ref)
        b = configs.mlp(g)
        b.bind_host()
        s = g.schedule()
        if planner == "ours":
            plan = lib.lancius_build_memory_plan(C.cast(s.ptr, _abi.SCHED_P), C.cast(g.ptr, _abi.GRAPH_P))
        else:
            plan = ref.lancius_build_memory_plan(s.ptr, g.ptr)
        pool = np.zeros(plan.contents.peak_memory // 8 + 64)
        ref.lancius_schedule_attach_pool(s.ptr, pool.ctypes.data_as(C.c_void_p), C.cast(plan, _abi.PLAN_P))
        arena = ref.lancius_arena_create(16 << 20)
        ref.lancius_schedule_execute(s.ptr, arena)
        o = b.outputs[0]
        got = np.ctypeslib.as_array(o.c.runtime_data, shape=(o.size,)).reshape(o.shape).copy()
        ref.lancius_arena_destroy(arena)
        g2 = L.Graph(ref)
        b2 = configs.mlp(g2)
        b2.bind_host()
        want = oracle.run_reference_graph(ref, g2, b2.outputs)[b2.outputs[0].id]
        if planner == "ours":
            assert np.max(np.abs(got - want)) == 0.0
        else:
            assert np.max(np.abs(got - want)) > 1e-3


def test_random_dag_plans_valid():
    rng = np.random.default_rng(0)
    for trial in range(30):
        g = L.Graph()
        pool = [g.input(8, 8) for _ in range(3)]
        for _ in range(rng.integers(5, 40)):
            a, b = pool[rng.integers(len(pool))], pool[rng.integers(len(pool))]
            op = rng.integers(5)
            n = [lambda: g.add(a, b), lambda: g.mul(a, b), lambda: g.matmul(a, b), lambda: g.relu(a),
                 lambda: g.reshape(a, 4, 16)][op]()
            if n.shape == (8, 8):
                pool.append(n)
        s = g.schedule()
        for views in (0, 1):
            p = g.lib.lancius_build_memory_plan_ex(s.ptr, g.ptr, 4, 256, views)
            assert g.lib.lancius_memory_plan_validate(p, s.ptr, g.ptr, 4) == 0
            g.lib.lancius_memory_plan_destroy(p)


def test_fusion_pass_matches_reference(ref):
    ours, theirs = L.Graph(), L.Graph(ref)
    configs.conv_stack(ours, batch=1, hw=16, fuse=True)
    configs.conv_stack(theirs, batch=1, hw=16, fuse=True)
    assert structure(ours) == structure(theirs)
    ops = [n.op for n in ours.nodes()]
    assert ops.count("CONV2D_RELU_FUSED") == 3 and ops.count("NOP") == 3

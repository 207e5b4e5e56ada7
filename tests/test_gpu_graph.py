"""End-to-end parity: configs built through the Lancius graph API, executed by
lancius_schedule_execute_cuda, compared with the FP64 oracle's arena-mode run of
the same graph object (normwise rel <= 1e-4, FP32-exact mode)."""
import numpy as np
import pytest

from conftest import assert_close
import lancius_b200 as L
from lancius_b200 import configs

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    d = L.Device(0)
    yield d
    d.close()


def run_gpu(device, built, replay=False, plan=None):
    sched = built.graph.schedule()
    device.set_graph_replay(replay)
    device.bind(sched, plan)
    for node, arr in built.inputs:
        device.upload(node, arr)
    device.execute(sched)
    device.synchronize()
    return [device.download(o) for o in built.outputs], sched


def oracle_outputs(orc, built):
    built.bind_host()
    r = orc.run_graph(built.graph, built.outputs)
    return [r[o.id] for o in built.outputs]


def test_ffi_known_answer(device):
    """stable/v9S/examples/audit_ffi.c:35-61: MatMul(2x3 . ones 3x4) -> ReLU == [4]*4 + [5]*4 exactly."""
    g = L.Graph()
    a, b = g.input(2, 3), g.input(3, 4)
    d = g.relu(g.matmul(a, b))
    s = g.schedule()
    device.bind(s)
    device.upload(a, np.array([-1.0, 2, 3, 4, -5, 6]))
    device.upload(b, np.ones(12))
    device.execute(s)
    out = device.download(d)
    assert out.ravel().tolist() == [4.0] * 4 + [5.0] * 4


@pytest.mark.parametrize("replay", [False, True])
def test_mlp_config(device, orc, replay):
    b = configs.mlp(L.Graph())
    (y,), _ = run_gpu(device, b, replay=replay)
    (ref,) = oracle_outputs(orc, b)
    assert_close(y, ref, 1e-4)
    assert np.allclose(y.sum(1), 1.0, atol=1e-5)
    if replay:  # a second replay gives the same bytes
        device.execute()
        assert np.array_equal(device.download(b.outputs[0]), y)


def test_attention_config(device, orc):
    b = configs.attention(L.Graph())      # batch 8, seq 512, 8 heads, head_dim 64, causal
    ys, _ = run_gpu(device, b)
    refs = oracle_outputs(orc, b)
    for y, r in zip(ys, refs):
        assert_close(y, r, 1e-4)


def test_conv_stack_reduced(device, orc):
    b = configs.conv_stack(L.Graph(), batch=2, hw=64)
    (y,), _ = run_gpu(device, b)
    (ref,) = oracle_outputs(orc, b)
    assert_close(y, ref, 1e-4, k=128 * 9)


@pytest.mark.parametrize("replay", [False, True])
def test_conv_global_pool_from_tile_sums(device, replay):
    """A global average pool over a tensor-core conv's NCHW output adds up per-tile channel
    sums stored by the conv's epilogue. Ragged on both axes: Co = 96 fills part of a
    128-channel tile, and Ho = 24 is 10 + 10 + 4 output rows. Checked against FP64 and
    against reading the conv output (LCU_NO_GAP_FUSE=1); the conv output itself is still
    stored and downloadable."""
    import os
    from lancius_b200 import data
    n, ci, hw, co = 4, 64, 24, 96
    xa = data.normal(71, (n, ci, hw, hw))
    wa = data.normal(72, (co, ci, 3, 3), 0.0, 0.06)

    def run():
        g = L.Graph()
        x, w = g.input_4d(n, ci, hw, hw), g.input_4d(co, ci, 3, 3)
        h = g.relu(g.conv2d(x, w, 1, 1))
        pooled = g.sum_axis1(g.reshape(h, n * co, hw * hw))
        g.optimize_fusion()
        s = g.schedule()
        device.set_graph_replay(replay)
        device.bind(s)
        device.upload(x, xa)
        device.upload(w, wa)
        device.execute(s)
        conv = [m for m in g.nodes() if m.op in ("CONV2D", "CONV2D_RELU_FUSED")][0]
        return device.download(pooled), device.download(conv)

    y, conv_out = run()
    os.environ["LCU_NO_GAP_FUSE"] = "1"
    try:
        y_ref_path, _ = run()
    finally:
        del os.environ["LCU_NO_GAP_FUSE"]
    t = torch.nn.functional.conv2d(torch.from_numpy(xa), torch.from_numpy(wa), padding=1).clamp_min(0).numpy()
    assert_close(conv_out, t, 1e-4, k=ci * 9)
    ref = t.reshape(n * co, hw * hw).sum(axis=1)
    assert_close(y.reshape(-1), ref, 1e-4, k=ci * 9 * hw * hw)
    assert_close(y, y_ref_path, 1e-5, elem_rel=1e-5, elem_abs=1e-6)


def test_encoder_reduced(device, orc):
    b = configs.encoder(L.Graph(), batch=2, seq=128, layers=2)
    ys, _ = run_gpu(device, b)
    refs = oracle_outputs(orc, b)
    for y, r in zip(ys, refs):
        assert_close(y, r, 1e-4, k=3072)


@pytest.mark.parametrize("mode", ["tf32", "bf16"])
def test_encoder_fast_modes(orc, mode):
    """The encoder graph in the fast modes (normwise 2e-2): BF16 GEMMs with TF32 attention,
    or everything in one TF32 pass."""
    d = L.Device(0, L.MODE_TF32 if mode == "tf32" else L.MODE_BF16)
    try:
        b = configs.encoder(L.Graph(), batch=2, seq=128, layers=2)
        ys, _ = run_gpu(d, b)
        for y, r in zip(ys, oracle_outputs(orc, b)):
            assert_close(y, r, 2e-2)
    finally:
        d.close()


def test_caller_plan_path(device, orc):
    """A caller-supplied lancius_memory_plan (the reference contract) is validated and used
    as-is: no fusion, every node in its planned slot."""
    g = L.Graph()
    b = configs.mlp(g)
    sched = g.schedule()
    plan = g.lib.lancius_build_memory_plan(sched.ptr, g.ptr)
    try:
        device.set_graph_replay(False)
        device.bind(sched, plan)
        for node, arr in b.inputs:
            device.upload(node, arr)
        device.execute(sched)
        y = device.download(b.outputs[0])
    finally:
        g.lib.lancius_memory_plan_destroy(plan)
    (ref,) = oracle_outputs(orc, b)
    assert_close(y, ref, 1e-4)


def test_fused_launch_count(device):
    """MLP: one launch per graph. Layer 1 (bias + ReLU in the epilogue) and layer 2 (bias +
    row softmax) run in one kernel: the last CTA of each 16-row block computes that block's
    layer 2 from the finished hidden rows. The two-launch form gives
    the same bits. The one-launch form is opt-in (LCU_MLP_FUSE=1); the default is two."""
    import os
    os.environ["LCU_MLP_FUSE"] = "1"
    try:
        b = configs.mlp(L.Graph())
        (y,), _ = run_gpu(device, b)
        assert device.last_launch_count == 1
        device.execute()                       # the tickets were reset: a second run is identical
        assert np.array_equal(device.download(b.outputs[0]), y)
    finally:
        del os.environ["LCU_MLP_FUSE"]
    b2 = configs.mlp(L.Graph())
    (y2,), _ = run_gpu(device, b2)
    assert device.last_launch_count == 2
    assert np.array_equal(y, y2)


def test_mlp_fused_other_shapes(device, orc):
    """The one-launch two-layer form on ragged shapes: rows not a multiple of 16, hidden
    width not a multiple of 32, GELU between the layers, 32 output columns."""
    import os
    from lancius_b200 import data
    os.environ["LCU_MLP_FUSE"] = "1"
    try:
        _mlp_fused_shapes(device, orc, data)
    finally:
        del os.environ["LCU_MLP_FUSE"]


def _mlp_fused_shapes(device, orc, data):
    for M, K, N1, N2, act in ((37, 100, 70, 7, "relu"), (130, 64, 96, 32, "gelu"), (5, 33, 40, 3, "relu")):
        g = L.Graph()
        bb = configs.Built("mlp_shape", g)
        x = configs._inp(bb, g.input(M, K), data.uniform(81, (M, K), -1, 1))
        h = configs._linear(g, bb, x, data.normal(82, (K, N1), 0, 0.2), data.normal(83, (N1,)), M)
        h = g.relu(h) if act == "relu" else g.gelu(h)
        y = g.softmax(configs._linear(g, bb, h, data.normal(84, (N1, N2), 0, 0.2), data.normal(85, (N2,)), M))
        bb.outputs = [y]
        (got,), _ = run_gpu(device, bb)
        assert device.last_launch_count == 1, (M, K, N1, N2)
        (ref,) = oracle_outputs(orc, bb)
        assert_close(got, ref, 1e-4)


def test_lenet_model_file_on_gpu(device, orc):
    """stable/v9S/pytorch_lenet.lancius loaded by lancius_graph_load and run on the GPU:
    conv5x5(pad 2)+ReLU+maxpool x2, flatten, matmul+add+ReLU, matmul+add; vs ONNX Runtime's
    golden output (normwise 1e-4, FP32-exact) and vs the FP64 oracle."""
    import os
    gold = os.path.join(os.path.dirname(__file__), "golden")
    g = L.Graph.load(os.path.join(gold, "pytorch_lenet.lancius"))
    nodes = g.nodes()
    x = next(n for n in nodes if n.op == "INPUT" and len(n.shape) == 4 and n.shape[1] == 3 and not n.c.runtime_data)
    out = [n for n in nodes if len(n.shape) == 2 and n.shape[1] == 10 and n.op != "INPUT"][-1]
    inp = np.fromfile(os.path.join(gold, "parity_input.bin"), dtype=np.float32).astype(np.float64)
    g.bind(x, inp)
    s = g.schedule()
    device.set_graph_replay(False)
    device.bind(s)
    device.upload_bound_inputs()           # weights came with the file; the image was bound above
    device.execute(s)
    y = device.download(out).ravel()
    ort = np.fromfile(os.path.join(gold, "baseline_out.bin"), dtype=np.float32)
    assert_close(y, ort, 1e-4, elem_rel=False)
    assert_close(y, orc.run_graph(g, [out])[out.id].ravel(), 1e-4)


def test_basis_graph_lowered_on_gpu(device, orc):
    """A BASIS stage-6 graph (the reference's legacy builder API), lowered onto the Lancius
    IR and run by the B200 executor, against the oracle on the same lowered graph."""
    from lancius_b200 import data
    from lancius_b200.basis import BasisGraph
    g = BasisGraph()
    x = g.input("x", 64, 784)
    w1, b1 = g.input("w1", 784, 256), g.input("b1", 1, 256)
    w2, b2 = g.input("w2", 256, 10), g.input("b2", 1, 10)
    h = g.relu(g.broadcast_add(g.matmul(x, w1), b1))
    y = g.tanh(g.broadcast_add(g.matmul(h, w2), b2))
    lg, m = g.lower()
    arrays = {x: data.normal(1, (64, 784)), w1: data.normal(2, (784, 256), 0, 0.05), b1: data.normal(3, (1, 256)),
              w2: data.normal(4, (256, 10), 0, 0.1), b2: data.normal(5, (1, 10))}
    for bid, arr in arrays.items():
        lg.bind(m[bid], np.asarray(arr, np.float32).astype(np.float64))
    s = lg.schedule()
    device.set_graph_replay(False)
    device.bind(s)
    device.upload_bound_inputs()
    device.execute(s)
    want = orc.run_graph(lg, [m[y]])[m[y].id]
    assert_close(device.download(m[y]), want, 1e-4)


def test_watchdog_reported_by_synchronize(device):
    """A kernel whose bounded mbarrier wait gives up (nothing ever arrives) records it in the
    watchdog word; lcu_synchronize reports LANCIUS_ERROR_INTERNAL once and clears it. The
    GPU stays usable: the next execution runs normally."""
    lib = device.lib
    assert lib.lcu_synchronize(device.ptr) == 0
    assert lib.lcu_watchdog_selftest(lib.lcu_stream(device.ptr)) == 0
    assert lib.lcu_synchronize(device.ptr) == -10
    assert lib.lcu_synchronize(device.ptr) == 0
    b = configs.mlp(L.Graph(), batch=8, seed=5)
    run_gpu(device, b)


def test_watchdog_reported_by_blocking_per_op_calls(device):
    """The blocking per-op launchers (tensor-core lcu_matmul, lcu_matmul_noalloc, lcu_conv2d)
    read the watchdog words before they return: a trip left by the self-test kernel turns the
    next call's result into LANCIUS_ERROR_INTERNAL, once; lcu_check_stream does the same for
    the asynchronous launchers."""
    import ctypes as C
    lib = device.lib
    p = lambda t: C.c_void_p(t.data_ptr())
    M = K = N = 512
    a = torch.randn(M, K, device="cuda")
    b = torch.randn(K, N, device="cuda")
    c = torch.empty(M, N, device="cuda")
    x = torch.randn(2, 32, 32, 32, device="cuda")
    w = torch.randn(64, 32, 3, 3, device="cuda")   # 64 x 2048 x 288: the tensor-core conv
    y = torch.empty(2, 64, 32, 32, device="cuda")
    torch.cuda.synchronize()
    calls = [
        lambda: lib.lcu_matmul(p(c), p(a), p(b), M, K, N, None, L.EPI_NONE, L.MODE_FP32_EXACT, None),
        lambda: lib.lcu_matmul_noalloc(p(c), p(a), p(b), M, K, N, None, L.EPI_NONE, L.MODE_FP32_EXACT, None),
        lambda: lib.lcu_conv2d(p(y), p(x), p(w), 2, 32, 32, 32, 64, 3, 3, 1, 1, 1, L.MODE_FP32_EXACT, None),
        lambda: lib.lcu_check_stream(None),
    ]
    for call in calls:
        assert lib.lcu_check_stream(None) == 0
        assert lib.lcu_watchdog_selftest(None) == 0
        assert call() == -10
        assert call() == 0
    ref = (a.double() @ b.double()).float()
    assert torch.allclose(c, ref, rtol=1e-3, atol=1e-3)


def test_conv_chain_nhwc_handoff(device, orc):
    """A conv output read only by the next conv stays NHWC between them (producer stores
    NHWC and its tf32_lo, consumer reads both in place). Same bytes as with the hand-off off
    and as with the consumer splitting on chip, and downloads of
    an NHWC-kept output (FP64 and FP32) come back NCHW. The first conv's output is dead
    after the second conv and its slot is reused by the third, so only the last two conv
    outputs are compared (the second is kept NHWC and read in the last wave)."""
    import os
    from lancius_b200 import data

    def build():
        g = L.Graph()
        x = g.input_4d(2, 3, 64, 64)
        w1, w2, w3 = g.input_4d(32, 3, 3, 3), g.input_4d(64, 32, 3, 3), g.input_4d(64, 64, 3, 3)
        h1 = g.relu(g.conv2d(x, w1, 1, 1))
        h2 = g.relu(g.conv2d(h1, w2, 2, 1))
        y = g.conv2d(h2, w3, 1, 1)
        g.optimize_fusion()
        arrs = [(x, data.normal(61, (2, 3, 64, 64))), (w1, data.normal(62, (32, 3, 3, 3), 0, 0.3)),
                (w2, data.normal(63, (64, 32, 3, 3), 0, 0.06)), (w3, data.normal(64, (64, 64, 3, 3), 0, 0.04))]
        return g, arrs, [y]

    def run():
        g, arrs, outs = build()
        s = g.schedule()
        device.bind(s)
        for n, a in arrs:
            device.upload(n, a)
        device.execute(s)
        # every conv node's output, intermediate ones included, through both download paths
        convs = [n for n in g.nodes() if n.op in ("CONV2D", "CONV2D_RELU_FUSED")][1:]
        return [device.download(n) for n in convs], [device.download(n, np.float32) for n in convs], (g, arrs, convs)

    y64, y32, (g, arrs, convs) = run()
    variants = []
    # NHWC split on chip (same kernels otherwise: same bytes); NCHW throughout (the stem
    # runs on CUDA cores in exact FP32 order instead of the tensor-core stem: within the
    # conv bound)
    # NHWC stores from the threads instead of TMA blocks (same bytes)
    exact = ("LCU_NO_NHWC_LO", "LCU_CONV_NO_TMA_OUT")
    for var in exact + ("LCU_NO_NHWC_HANDOFF",):
        os.environ[var] = "1"
        try:
            variants.append((var, run()[:2]))
        finally:
            del os.environ[var]
    assert len(convs) == 2
    for var, (r64, r32) in variants:
        for a, b in list(zip(y64, r64)) + list(zip(y32, r32)):
            if var in exact:
                assert np.array_equal(a, b), var
            else:
                assert_close(a, b, 1e-4, k=64 * 9)
    for n, a in arrs:
        g.bind(n, a)
    ref = orc.run_graph(g, convs)
    for n, y in zip(convs, y64):
        assert_close(y, ref[n.id], 1e-4, k=64 * 9)


def test_mlp_softmax_head_folded(device, orc):
    """MATMUL -> ADD(bias) -> SOFTMAX over 10 columns runs as one small-product GEMM whose
    epilogue does the row softmax; the bytes equal the unfused graph's (GEMM, ADD, SOFTMAX
    launched separately) and match the FP64 reference."""
    outs = []
    for fuse in (True, False):
        device.set_fusion(fuse)
        try:
            b = configs.mlp(L.Graph())
            (y,), _ = run_gpu(device, b)
            outs.append((y, b))
        finally:
            device.set_fusion(True)
    assert np.array_equal(outs[0][0], outs[1][0])
    (ref,) = oracle_outputs(orc, outs[0][1])
    assert_close(outs[0][0], ref, 1e-4)

"""The reference's own entry points, linked from a C program against liblancius_b200.so
(tests/dropin/dropin_main.c, built by tests/dropin/Makefile): the stable FFI
(lancius_compile_and_run / lancius_read_output, reference lancius_stable_api.c:119-150),
lancius_schedule_execute and _parallel (lancius_scheduler.c:311-413) and
lancius_schedule_execute_static as examples/run_edge.c calls it (:475-520). Each runs on
the GPU and is compared with the FP64 oracle (normwise <= 1e-4 plus the elementwise
bound |d| <= 1e-4*|ref| + 1e-6*max|ref|, FP32-exact) and, for LeNet, with ONNX Runtime's
golden output."""
import os
import subprocess

import numpy as np
import pytest

from conftest import assert_close
import lancius_b200 as L
from lancius_b200 import configs, data

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")
EXE = os.path.join(HERE, "dropin", "dropin_main")


@pytest.fixture(scope="module")
def exe():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    L.load()
    subprocess.run(["make", "-C", os.path.join(HERE, "dropin")], check=True, capture_output=True)
    return EXE


def run(exe, *args):
    r = subprocess.run([exe, *map(str, args)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, f"rc {r.returncode}\n{r.stdout}\n{r.stderr}"
    return r


def test_stable_ffi_on_gpu(exe, orc, tmp_path):
    x = data.uniform(0, (64, 784), 0.0, 1.0)
    w1 = data.normal(21, (784, 256), 0.0, 1 / 28)
    w2 = data.normal(22, (256, 10), 0.0, 1 / 16)
    for name, arr in (("x", x), ("w1", w1), ("w2", w2)):
        arr.astype(np.float64).tofile(tmp_path / name)
    run(exe, "stable", tmp_path / "x", tmp_path / "w1", tmp_path / "w2", tmp_path / "h", tmp_path / "y")
    h_ref = np.maximum(orc.matmul(x, w1), 0.0)
    y_ref = orc.matmul(h_ref, w2)
    # the intermediate h is readable too, as after the reference's run
    assert_close(np.fromfile(tmp_path / "h").reshape(64, 256), h_ref, 1e-4)
    assert_close(np.fromfile(tmp_path / "y").reshape(64, 10), y_ref, 1e-4)


def test_schedule_execute_arena_and_parallel_on_gpu(exe, orc, tmp_path):
    b = configs.mlp(L.Graph())
    files = []
    for i, (_, arr) in enumerate(b.inputs):      # x, w1, b1, w2, b2
        p = tmp_path / f"in{i}"
        arr.tofile(p)
        files.append(p)
    run(exe, "arena", *files, tmp_path / "out")
    got = np.fromfile(tmp_path / "out").reshape(3, 64, 10)
    b.bind_host()
    want = orc.run_graph(b.graph, b.outputs)[b.outputs[0].id]
    for k in range(3):   # execute, execute with a rebuilt schedule, execute_parallel
        assert_close(got[k], want, 1e-4)
        assert np.allclose(got[k].sum(axis=1), 1.0, atol=1e-5)


def test_schedule_execute_static_lenet_on_gpu(exe, orc, tmp_path):
    run(exe, "static", os.path.join(GOLD, "pytorch_lenet.lancius"), os.path.join(GOLD, "parity_input.bin"),
        tmp_path / "out")
    y = np.fromfile(tmp_path / "out")
    ort = np.fromfile(os.path.join(GOLD, "baseline_out.bin"), dtype=np.float32)
    assert_close(y, ort, 1e-4, elem_rel=False)
    g = L.Graph.load(os.path.join(GOLD, "pytorch_lenet.lancius"))
    nodes = g.nodes()
    x = next(n for n in nodes if n.op == "INPUT" and len(n.shape) == 4 and n.shape[1] == 3 and not n.c.runtime_data)
    out = [n for n in nodes if len(n.shape) == 2 and n.shape[1] == 10 and n.op != "INPUT"][-1]
    g.bind(x, np.fromfile(os.path.join(GOLD, "parity_input.bin"), dtype=np.float32).astype(np.float64))
    assert_close(y, orc.run_graph(g, [out])[out.id].ravel(), 1e-4)

"""The .lancius load path (reference lancius_serialize.c) and the LeNet golden vectors
the reference ships: stable/v9S/pytorch_lenet.lancius (v9 record layout), its
parity_input.bin, ONNX Runtime's baseline_out.bin and the reference's own
lancius_out.bin. Parity bar from stable/v9S/audit_pytorch_parity.py:62-72:
normwise max|d|/max|ref| < 1e-5."""
import os

import numpy as np

import lancius_b200 as L
from conftest import rel_err

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def lenet():
    g = L.Graph.load(os.path.join(GOLD, "pytorch_lenet.lancius"))
    nodes = g.nodes()
    x = next(n for n in nodes if n.op == "INPUT" and len(n.shape) == 4 and n.shape[1] == 3 and not n.c.runtime_data)
    out = [n for n in nodes if len(n.shape) == 2 and n.shape[1] == 10 and n.op != "INPUT"][-1]
    inp = np.fromfile(os.path.join(GOLD, "parity_input.bin"), dtype=np.float32).astype(np.float64)
    return g, x, out, inp


def test_lenet_oracle_matches_onnxruntime_and_reference(orc):
    g, x, out, inp = lenet()
    assert [n.op for n in g.nodes()].count("CONV2D") == 2
    g.bind(x, inp)
    y = orc.run_graph(g, [out])[out.id].ravel()
    ort = np.fromfile(os.path.join(GOLD, "baseline_out.bin"), dtype=np.float32)
    ref = np.fromfile(os.path.join(GOLD, "lancius_out.bin"), dtype=np.float32)
    assert rel_err(y, ort) < 1e-5
    assert np.array_equal(y.astype(np.float32), ref)          # the reference's own output, bit for bit


def test_save_load_round_trip(tmp_path):
    g, x, out, inp = lenet()
    p = str(tmp_path / "lenet_v1.lancius")
    g.save(p)
    h = L.Graph.load(p)
    a = [(n.op, n.shape, n.c.kernel_h, n.c.stride, n.c.pad) for n in g.nodes()]
    b = [(n.op, n.shape, n.c.kernel_h, n.c.stride, n.c.pad) for n in h.nodes()]
    assert a == b
    for n1, n2 in zip(g.nodes(), h.nodes()):
        if n1.c.runtime_data:
            assert np.array_equal(np.ctypeslib.as_array(n1.c.runtime_data, shape=(n1.size,)),
                                  np.ctypeslib.as_array(n2.c.runtime_data, shape=(n2.size,)))


def test_malformed_files_rejected(tmp_path):
    src = open(os.path.join(GOLD, "pytorch_lenet.lancius"), "rb").read()
    for i, blob in enumerate([b"", src[:100], src[:-1], b"XXXX" + src[4:], src + b"\0"]):
        p = tmp_path / f"bad{i}.lancius"
        p.write_bytes(blob)
        try:
            L.Graph.load(str(p))
            assert False, f"case {i} loaded"
        except L.LanciusError as e:
            assert e.code in (-6, -8)

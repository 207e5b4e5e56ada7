"""Regenerates the golden fixtures in this folder from the REFERENCE library
(oracle/_ref/liblancius_ref.so, compiled from the reference's own C sources by
`make -C oracle ref`): seeded config inputs -> reference lancius_schedule_execute
(arena mode) -> outputs saved as .npz. Run from the repository root:
    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import lancius_b200 as L  # noqa: E402
from lancius_b200 import configs  # noqa: E402
import oracle  # noqa: E402

CASES = {
    "mlp": lambda g: configs.mlp(g),
    "attention_b2_s96_h2": lambda g: configs.attention(g, batch=2, seq=96, heads=2),
    "conv_b1_hw20": lambda g: configs.conv_stack(g, batch=1, hw=20),
    # LAYERNORM + GELU + residual + causal ATTENTION through the reference executor
    "encoder_causal_b2_s24_l2": lambda g: configs.encoder(g, batch=2, seq=24, layers=2, d_model=64,
                                                          heads=4, ffn=128, causal=True),
}

if __name__ == "__main__":
    ref = oracle.reference()
    for name, build in CASES.items():
        g = L.Graph(ref)
        b = build(g)
        b.bind_host()
        res = oracle.run_reference_graph(ref, g, b.outputs)
        np.savez_compressed(os.path.join(os.path.dirname(__file__), f"{name}.npz"),
                            **{f"out{i}": res[o.id] for i, o in enumerate(b.outputs)})
        print(name, [res[o.id].shape for o in b.outputs])

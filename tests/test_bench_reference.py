"""The bench's reference arm and cpu_baseline run the reference's own executor on bounded
samples of each workload (CPU only; needs oracle/_ref built from the reference sources)."""
import json
import subprocess
import sys
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_cpu_baseline_samples(ref):
    sys.path.insert(0, ROOT)
    import bench
    for cfg in ("mlp", "gemm4096"):
        val, info = bench.cpu_baseline(cfg, steps=1)
        assert val > 0 and info["kind"] == "reference" and info["cores"] >= 1


def test_reference_arm_line(ref):
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", "mlp",
                          "--steps", "1", "--warmup", "1"], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["metric"] == "graph inferences/sec" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "reference"

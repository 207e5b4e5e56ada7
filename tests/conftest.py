import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle.Oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle
    if not oracle.reference_available():
        pytest.skip("reference library (oracle/_ref) not built here")
    return oracle.reference()


def rel_err(y, ref_y):
    """normwise relative error max|y - ref| / max|ref| (the reference's own parity
    metric, stable/v9S/audit_pytorch_parity.py:62-64)"""
    y = np.asarray(y, np.float64)
    ref_y = np.asarray(ref_y, np.float64)
    return float(np.max(np.abs(y - ref_y)) / max(np.max(np.abs(ref_y)), 1e-300))


def assert_close(y, ref_y, norm_tol, elem_rel=None, elem_abs=None):
    """normwise bound, plus (optionally) |y-ref| <= elem_rel*|ref| + elem_abs*max|ref|"""
    assert np.all(np.isfinite(y)), "non-finite output"
    e = rel_err(y, ref_y)
    assert e <= norm_tol, f"normwise rel err {e:.3e} > {norm_tol:.1e}"
    if elem_rel is not None:
        y = np.asarray(y, np.float64)
        ref_y = np.asarray(ref_y, np.float64)
        bound = elem_rel * np.abs(ref_y) + elem_abs * np.max(np.abs(ref_y))
        bad = np.abs(y - ref_y) > bound
        assert not bad.any(), f"{bad.sum()} elements outside elementwise bound (worst {np.max(np.abs(y-ref_y)-bound):.3e})"
    return e

"""GPU test of lcu_matmul_noalloc, the GEMM entry point that never allocates.

It exists for callers that may not call cudaMalloc while running (device memory
owned by another allocator, or a fixed memory budget); its scratch is a fixed
array inside the library. Its output must match lcu_matmul's on the same inputs,
within the FP32-exact bar of the other GEMM tests (normwise rel <= 1e-4, both
also checked against the FP64 oracle), on two calls in a row -- the second call
reuses the array the first one left behind. This file is collected last.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_close, rel_err
from lancius_b200 import EPI_GELU, EPI_NONE, EPI_RELU, MODE_FP32_EXACT, MODE_TF32, data, load

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return load()


def _p(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


CASES = [(512, 768, 768, EPI_NONE, MODE_FP32_EXACT), (300, 1000, 130, EPI_RELU, MODE_FP32_EXACT),
         (256, 2048, 512, EPI_GELU, MODE_TF32),
         # K > 8192: split-K, partial sums in the fixed array and the reduce kernel
         (64, 16384, 96, EPI_RELU, MODE_FP32_EXACT)]


def test_noalloc_matches_matmul_twice(lib, orc):
    assert lib.lcu_noalloc_prepare() == 0
    keep = []
    for M, K, N, epi, mode in CASES:
        a = data.uniform(71, (M, K), -1, 1)
        b = data.uniform(72, (K, N), -1, 1)
        bias = data.normal(73, (N,))
        da, db, dbias = (torch.tensor(x.astype(np.float32), device="cuda") for x in (a, b, bias))
        keep += [da, db, dbias]
        ref_out = torch.empty((M, N), device="cuda")
        assert lib.lcu_matmul(_p(ref_out), _p(da), _p(db), M, K, N, _p(dbias), epi, mode, None) == 0
        torch.cuda.synchronize()
        want = ref_out.cpu().numpy()
        tol = 1e-4 if mode == MODE_FP32_EXACT else 2e-2
        oracle = orc.matmul(a, b) + bias
        if epi == EPI_RELU:
            oracle = np.maximum(oracle, 0)
        elif epi == EPI_GELU:
            oracle = orc.gelu(oracle)
        for call in range(2):
            out = torch.full((M, N), float("nan"), device="cuda")
            rc = lib.lcu_matmul_noalloc(_p(out), _p(da), _p(db), M, K, N, _p(dbias), epi, mode, None)
            assert rc == 0, f"call {call}: lancius error {rc}"
            got = out.cpu().numpy()
            assert_close(got, want, tol, k=min(K, 8192))
            assert_close(got, oracle, tol, k=min(K, 8192))


def test_noalloc_rejects_oversize(lib):
    x = torch.zeros(16, device="cuda")
    cap = lib.lcu_noalloc_scratch_capacity()
    assert cap == 64 << 20
    n = 4096   # 3xTF32 needs ~16 * (n*n + n*n) bytes = 512 MiB > capacity
    rc = lib.lcu_matmul_noalloc(_p(x), _p(x), _p(x), n, n, n, None, EPI_NONE, MODE_FP32_EXACT, None)
    assert rc == -9   # LANCIUS_ERROR_OVERFLOW, nothing launched
    assert lib.lcu_matmul_noalloc(_p(x), _p(x), _p(x), 4, 0, 4, None, EPI_NONE, MODE_FP32_EXACT, None) == -3
    # sizes whose byte counts would wrap size_t are rejected before any arithmetic on them
    big = 1 << 40
    assert lib.lcu_matmul_noalloc(_p(x), _p(x), _p(x), big, big, big, None, EPI_NONE, MODE_FP32_EXACT, None) == -9

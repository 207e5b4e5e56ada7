"""Column-split GEMM (lcu_gemm_colsplit, NCCL all-gather; lcu_gemm_colsplit_fused, epilogue
stores into every rank's C over NVLink) against the FP64 oracle: one rank on one GPU here,
and 2 ranks (one process per GPU) when 2 GPUs are visible."""
import ctypes as C
import multiprocessing as mproc

import numpy as np
import pytest

from conftest import assert_close
from lancius_b200 import MODE_FP32_EXACT, data, load

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

SHAPES = {"plain": (384, 1536, 1024), "splitk": (128, 9000, 256)}   # K > 8192: split-K reduce stores


def operands(M, K, N):
    return data.uniform(81, (M, K), -1, 1), data.uniform(82, (K, N), -1, 1)


def _rank(rank, world, uid, q, fused=False, shape="plain", swap_c=False):
    M, K, N = SHAPES[shape]
    import torch
    from lancius_b200 import load as _load
    lib = _load()
    torch.cuda.set_device(rank)
    comm = lib.lcu_comm_create(world, rank, C.c_char_p(uid), rank)
    if not comm:
        q.put((rank, None, lib.lancius_get_error()))
        return
    a, b = operands(M, K, N)
    ns = N // world
    da = torch.tensor(a.astype(np.float32), device="cuda")
    db = torch.tensor(np.ascontiguousarray(b[:, rank * ns:(rank + 1) * ns]).astype(np.float32), device="cuda")
    c = torch.empty((M, N), device="cuda")
    fn = lib.lcu_gemm_colsplit_fused if fused else lib.lcu_gemm_colsplit
    rc = 0
    for call in range(2 if fused else 1):   # the fused path's second call reuses the opened peer C
        if swap_c and call == 1 and rank == world - 1:
            # only the last rank brings a new C: every rank must reopen its mappings
            c = torch.empty((M, N), device="cuda")
        c.fill_(float("nan"))
        torch.cuda.synchronize()
        rc = rc or fn(comm, C.c_void_p(c.data_ptr()), C.c_void_p(da.data_ptr()), C.c_void_p(db.data_ptr()),
                      M, K, N, MODE_FP32_EXACT, None)
        torch.cuda.synchronize()
    q.put((rank, c.cpu().numpy() if rc == 0 else None, rc))
    lib.lcu_comm_destroy(comm)


def run_ranks(world, fused=False, shape="plain", swap_c=False):
    lib = load()
    uid = C.create_string_buffer(128)
    assert lib.lcu_comm_unique_id(uid, 128) == 0
    ctx = mproc.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, uid.raw, q, fused, shape, swap_c)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return out


@pytest.mark.parametrize("world", [1, 2])
@pytest.mark.parametrize("fused,shape", [(False, "plain"), (True, "plain"), (True, "splitk")])
def test_colsplit_matches_oracle(orc, world, fused, shape):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    a, b = operands(*SHAPES[shape])
    ref = orc.matmul(a, b)
    for rank, c, rc in run_ranks(world, fused, shape):
        assert rc == 0, f"rank {rank}: error {rc}"
        assert_close(c, ref, 1e-4, k=min(SHAPES[shape][1], 8192))


def test_colsplit_fused_new_c_on_one_rank(orc):
    """The second fused call passes a new C on one rank only; the C records are exchanged
    collectively on every call, so all ranks reopen together and both results are right."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    a, b = operands(*SHAPES["plain"])
    ref = orc.matmul(a, b)
    for rank, c, rc in run_ranks(2, True, "plain", swap_c=True):
        assert rc == 0, f"rank {rank}: error {rc}"
        assert_close(c, ref, 1e-4, k=SHAPES["plain"][1])

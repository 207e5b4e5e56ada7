"""Multi-rank host logic on CPU (gloo, world size 2): batch sharding reproduces the
single-process result, and a rank that fails is seen by the other as an error
within a short process-group timeout (no hang)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import lancius_b200 as L
from lancius_b200 import configs
from lancius_b200.shard import shard_range


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import oracle
    import torch
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=6))
    try:
        rows = shard_range(128, rank, world)
        g = L.Graph()
        b = configs.mlp(g, batch=128, rows=rows)
        b.bind_host()
        y = oracle.Oracle().run_graph(g, b.outputs)[b.outputs[0].id]
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure on rank 1 before the gather")
        parts = [torch.zeros(shard_range(128, r, world)[1] - shard_range(128, r, world)[0], 10, dtype=torch.float64)
                 for r in range(world)]
        dist.all_gather(parts, torch.from_numpy(y))
        q.put((rank, "ok", torch.cat(parts).numpy()))
    except Exception as ex:  # reported to the parent; the process exits normally
        q.put((rank, "error", str(ex)[:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, status, payload = q.get(timeout=120)
        res[r] = (status, payload)
    for p in procs:
        p.join(timeout=60)
    return res


def test_shard_range():
    assert [shard_range(10, r, 3) for r in range(3)] == [(0, 4), (4, 7), (7, 10)]
    assert shard_range(256, 7, 8) == (224, 256)
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_sharded_batch_equals_full_batch(orc):
    res = _run("ok")
    g = L.Graph()
    b = configs.mlp(g, batch=128)
    b.bind_host()
    full = orc.run_graph(g, b.outputs)[b.outputs[0].id]
    for r in range(2):
        status, y = res[r]
        assert status == "ok"
        assert np.array_equal(y, full)


def test_failed_rank_is_detected():
    res = _run("fail")
    assert res[1][0] == "error" and "injected" in res[1][1]
    assert res[0][0] == "error"      # the surviving rank's collective errors out instead of hanging

"""The multi-rank host logic of bench.py on CPU ranks (gloo, world size 2).

With --gpus N every rank times its own shard of the work (its own C2 head group, its own
decode batch: weak scaling, no data-path collective); the reported time is the max over the
ranks and the throughput is the whole job's.  These tests run that reduction and the env
parsing on two spawned CPU processes, the way torchrun would start them.
"""

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from datetime import timedelta
    import bench
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        w, r, local = bench.dist_setup(world)
        timings = [1.0 + rank, 10.0 - rank, 0.5 * (rank + 1)]  # this rank's phase times (ms)
        out = bench.max_over_ranks(timings, w, torch.device("cpu"))
        q.put((r, local, out))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_two_cpu_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = sorted(q.get(timeout=120) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert [r for r, _, _ in res] == [0, 1]
    for _, _, out in res:
        assert out == [2.0, 10.0, 1.0]  # every rank sees the slowest rank's time per entry
    assert all(p.exitcode == 0 for p in procs)


def test_single_rank_is_identity():
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.max_over_ranks([3, 4.5], 1, torch.device("cpu")) == [3.0, 4.5]


def test_dist_setup_rejects_mismatched_world(monkeypatch):
    sys.path.insert(0, str(ROOT))
    import bench
    monkeypatch.setenv("WORLD_SIZE", "4")
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("LOCAL_RANK", "1")
    with pytest.raises(SystemExit):
        bench.dist_setup(2)
    assert bench.dist_setup(4) == (4, 1, 1)

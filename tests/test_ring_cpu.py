"""The sequence-sharded ring (``ultrametric.ring``) on gloo CPU ranks: the rotation schedule,
the per-chunk list splitting, causal hop skipping and the log-sum-exp merge, with the CPU
oracle standing in for the two device operations (``oracle/ring_oracle.py``); checked
against masked dense attention of the whole sequence.  Plus a rank that fails before the
first exchange: its peer's wait ends with an error after the short process-group timeout
instead of hanging.
"""

import os
import socket
import sys
import time
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(N, RB, H=2, Hkv=1, D=16, causal=True, seed=0):
    sys.path.insert(0, str(ROOT))
    from oracle import block_list_oracle as blo
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(1, H, N, D, generator=gen, dtype=torch.float64)
    k = torch.randn(1, Hkv, N, D, generator=gen, dtype=torch.float64)
    v = torch.randn(1, Hkv, N, D, generator=gen, dtype=torch.float64)
    NB = N // RB
    router = blo.tree_router(1, H, NB, 4)
    lists, counts, mc = blo.build_block_lists(router, [2] * H, is_causal=causal, sink_block=True,
                                              local_blocks=0, arity=2)
    return q, k, v, torch.from_numpy(lists).to(torch.int32), torch.from_numpy(counts).to(torch.int32)


def _local_rows(rank, world, N, layout):
    """This rank's rows of the global sequence, in its local order."""
    if layout == "zigzag":
        c = N // (2 * world)
        return torch.cat([torch.arange(rank * c, (rank + 1) * c),
                          torch.arange((2 * world - 1 - rank) * c, (2 * world - rank) * c)])
    Nl = N // world
    return torch.arange(rank * Nl, (rank + 1) * Nl)


def _ring_worker(rank, world, port, q_out, N, RB, causal, fail_rank, layout="contiguous"):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "sparse-ai_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from datetime import timedelta
    from oracle import ring_oracle
    from ultrametric.block_list import BlockLists
    from ultrametric.ring import ring_block_list_attention
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure before the first exchange")
        q, k, v, lists, counts = _problem(N, RB, causal=causal)
        rows = _local_rows(rank, world, N, layout)
        bl = BlockLists(lists, counts, lists.shape[-1])
        t0 = time.time()
        out, lse = ring_block_list_attention(
            q[:, :, rows].contiguous(), k[:, :, rows].contiguous(), v[:, :, rows].contiguous(), bl,
            route_block=RB, is_causal=causal, attn=ring_oracle.chunk_attention,
            merge_factory=ring_oracle.LseMergeCPU, layout=layout)
        # numpy: pickled by value (a torch tensor would travel as a file descriptor, which
        # the receiver cannot open once this process has exited)
        q_out.put((rank, "ok", out.numpy(), lse.numpy(), time.time() - t0))
    except Exception as e:  # report to the test instead of hanging
        q_out.put((rank, "error", repr(e), None, 0.0))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, N, RB, causal, fail_rank=-1, layout="contiguous"):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ring_worker, args=(r, world, port, q, N, RB, causal, fail_rank, layout))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = {}
        for _ in procs:
            r, status, a, b, dt = q.get(timeout=180)
            res[r] = (status, a, b, dt)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return res


@pytest.mark.parametrize("world,causal,layout", [(2, True, "contiguous"), (3, True, "contiguous"),
                                                 (3, False, "contiguous"), (2, True, "zigzag"),
                                                 (3, True, "zigzag"), (2, False, "zigzag")])
def test_ring_matches_whole_sequence_attention(world, causal, layout):
    N, RB = 192 * world * (2 if layout == "zigzag" else 1), 64
    res = _run(world, N, RB, causal, layout=layout)
    sys.path.insert(0, str(ROOT))
    from oracle import ring_oracle
    q, k, v, lists, counts = _problem(N, RB, causal=causal)
    ref_out, ref_lse = ring_oracle.chunk_attention(q, k, v, lists, counts, RB, causal, q.shape[-1] ** -0.5)
    for r in range(world):
        status, out, lse, _ = res[r]
        assert status == "ok", out
        out, lse = torch.from_numpy(out), torch.from_numpy(lse)
        rows = _local_rows(r, world, N, layout)
        # partial LSEs travel as fp32 (like the kernel's): ~1e-7 on the merge weights
        torch.testing.assert_close(out, ref_out[:, :, rows], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(lse.to(torch.float32), ref_lse[:, :, rows], rtol=1e-6, atol=1e-6)


def test_ring_peer_failure_ends_with_an_error():
    t0 = time.time()
    res = _run(2, 256, 64, True, fail_rank=1)
    assert res[1][0] == "error" and "injected" in res[1][1]
    assert res[0][0] == "error"  # the surviving rank's exchange failed instead of hanging
    assert time.time() - t0 < 150


def test_chunk_lists_split_and_rebase():
    sys.path.insert(0, str(ROOT / "sparse-ai_b200"))
    from ultrametric.ring import chunk_lists, ring_hops
    lists = torch.tensor([[[[0, 2, 5, 7], [1, 4, 0, 0]]]], dtype=torch.int32)
    counts = torch.tensor([[[4, 2]]], dtype=torch.int32)
    sub, n = chunk_lists(lists, counts, 0, 2, 4, 8)
    assert n.tolist() == [[[2, 1]]]
    assert sub[0, 0, 0, :2].tolist() == [1, 3] and sub[0, 0, 1, :1].tolist() == [0]
    assert int(sub[0, 0, 0, 2:].abs().sum()) == 0
    assert ring_hops(1, 3, True) == [(0, 1, True), (1, 0, False)]
    assert [c for _, c, _ in ring_hops(0, 3, False)] == [0, 2, 1]


def test_chunk_lists_multi_rebases_two_ranges():
    sys.path.insert(0, str(ROOT / "sparse-ai_b200"))
    from ultrametric.ring import RingPlan, chunk_lists_multi
    from ultrametric.block_list import BlockLists
    # 8 key blocks; local query blocks = global blocks 1 and 6; local keys = chunks [0,2) and [6,8)
    lists = torch.zeros(1, 1, 8, 8, dtype=torch.int32)
    counts = torch.zeros(1, 1, 8, dtype=torch.int32)
    lists[0, 0, 1, :2] = torch.tensor([0, 1])
    counts[0, 0, 1] = 2
    lists[0, 0, 6, :4] = torch.tensor([0, 3, 6, 7])
    counts[0, 0, 6] = 4
    sub, n = chunk_lists_multi(lists, counts, [(1, 2), (6, 7)], [(0, 2), (6, 8)])
    assert n.tolist() == [[[2, 3]]]
    assert sub[0, 0, 0, :2].tolist() == [0, 1]
    assert sub[0, 0, 1, :3].tolist() == [0, 2, 3]   # 3 (not held) dropped, 6 -> 2, 7 -> 3
    assert int(sub[0, 0, 1, 3:].abs().sum()) == 0
    # zigzag plans balance causal work: every rank computes the same number of hops
    NB, world = 8, 2
    full = torch.arange(NB, dtype=torch.int32).view(1, 1, 1, NB).expand(1, 1, NB, NB).contiguous()
    cnt = (torch.arange(NB, dtype=torch.int32) + 1).view(1, 1, NB)
    bl = BlockLists(full, cnt, NB)
    hops = [len(RingPlan(bl, world, r, NB // world * 16, 16, True, layout="zigzag").hops)
            for r in range(world)]
    assert hops == [2, 2]
    work = [int(sum(c.sum() for _, _, _, c in RingPlan(bl, world, r, NB // world * 16, 16, True,
                                                    layout="zigzag").hops)) for r in range(world)]
    assert work[0] == work[1]

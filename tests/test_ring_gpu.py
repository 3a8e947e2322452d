"""The sequence-sharded ring's device side: the log-sum-exp merge kernel, and the ring's
per-rank hops (chunk lists, causal diagonal, hop skipping, merges) run one rank after
another on one GPU, against the whole-sequence forward and the oracle.  With two or more
GPUs, the ring itself over NCCL between two processes."""

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

from helpers import assert_half_close, tree_router
from oracle import attention_oracle as ao
from oracle import block_list_oracle as blo
from oracle import ring_oracle
from ultrametric import block_list_attention, build_block_lists
from ultrametric.block_list import BlockLists
from ultrametric.ring import _CudaMerge, ring_emulate

pytestmark = pytest.mark.gpu
DEV = "cuda"
ROOT = Path(__file__).resolve().parent.parent


def test_lse_merge_kernel_matches_cpu_merge():
    gen = torch.Generator().manual_seed(3)
    Z, H, N, D = 1, 3, 200, 128
    parts = []
    for i in range(3):
        o = torch.randn(Z, H, N, D, generator=gen).bfloat16()
        lse = torch.randn(Z, H, N, generator=gen) * 3
        lse[0, 0, i * 10:(i + 1) * 10] = float("-inf")  # rows without keys in this part
        parts.append((o, lse))
    parts[0][1][0, 1, 50:60] = float("-inf")
    parts[1][1][0, 1, 50:60] = float("-inf")
    parts[2][1][0, 1, 50:60] = float("-inf")  # rows with no key at all
    q_like = parts[0][0]
    gm, cm = _CudaMerge(q_like.to(DEV)), ring_oracle.LseMergeCPU(q_like)
    out_g = torch.empty(Z, H, N, D, dtype=torch.bfloat16, device=DEV)
    out_c = torch.empty(Z, H, N, D, dtype=torch.bfloat16)
    for i, (o, lse) in enumerate(parts):
        last = i == len(parts) - 1
        gm(o.to(DEV), lse.to(DEV), i == 0, out_g if last else None)
        cm(o, lse, i == 0, out_c if last else None)
    torch.testing.assert_close(gm.acc.cpu(), cm.acc.float(), rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(gm.lse.cpu(), cm.lse.float(), rtol=1e-6, atol=1e-5)
    assert torch.equal(gm.lse.cpu()[0, 1, 50:60], torch.full((10,), float("-inf")))
    assert int(out_g.cpu()[0, 1, 50:60].float().abs().sum()) == 0
    assert_half_close(out_g.cpu(), out_c.float(), "merge out")


@pytest.mark.parametrize("world,causal,layout", [(4, True, "contiguous"), (2, False, "contiguous"),
                                                 (4, True, "zigzag"), (2, True, "zigzag")])
def test_ring_emulation_matches_whole_forward(world, causal, layout):
    """C5-shaped (H=16/8 heads of 128, causal + sink, tree routes) at N=4096; both ring
    layouts (contiguous chunks, and the balanced zigzag pair of chunks per rank)."""
    Z, H, Hkv, N, D, RB, TD = 1, 16, 8, 4096, 128, 128, 6
    gen = torch.Generator().manual_seed(5)
    q = torch.randn(Z, H, N, D, generator=gen).bfloat16().to(DEV)
    k = torch.randn(Z, Hkv, N, D, generator=gen).bfloat16().to(DEV)
    v = torch.randn(Z, Hkv, N, D, generator=gen).bfloat16().to(DEV)
    router = tree_router(Z, H, N // RB, TD).to(DEV)
    bl = build_block_lists(router, 3, is_causal=causal, sink_block=True, arity=2)
    out_r, lse_r = ring_emulate(q, k, v, bl, world, route_block=RB, is_causal=causal, layout=layout)
    out_f, lse_f = block_list_attention(q, k, v, bl, route_block=RB, is_causal=causal, return_lse=True)
    assert_half_close(out_r.float().cpu(), out_f.float().cpu(), "ring vs whole forward")
    torch.testing.assert_close(lse_r.cpu(), lse_f.cpu(), rtol=1e-4, atol=1e-3)
    # and against the oracle on two heads
    m = ao.token_mask(torch.from_numpy(blo.block_mask(router.cpu().numpy(), [3] * H, is_causal=causal,
                                                      sink_block=True)), RB, N, causal)
    for h in (0, 11):
        ref, _ = ao.masked_attention(q[:, h:h + 1].cpu().float(), k[:, h // 2:h // 2 + 1].cpu().float(),
                                     v[:, h // 2:h // 2 + 1].cpu().float(), m[:, h:h + 1])
        assert_half_close(out_r[:, h:h + 1].float().cpu(), ref.float(), f"ring head {h}")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, q_out):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "sparse-ai_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from datetime import timedelta
    from ultrametric import build_block_lists as bbl
    from ultrametric.ring import ring_block_list_attention
    from helpers import tree_router as tr
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        Z, H, Hkv, N, D, RB = 1, 4, 2, 2048, 128, 128
        gen = torch.Generator().manual_seed(9)
        q = torch.randn(Z, H, N, D, generator=gen).bfloat16()
        k = torch.randn(Z, Hkv, N, D, generator=gen).bfloat16()
        v = torch.randn(Z, Hkv, N, D, generator=gen).bfloat16()
        router = tr(Z, H, N // RB, 5).to(dev)
        bl = bbl(router, 2, is_causal=True, sink_block=True, arity=2)
        Nl = N // world
        rows = slice(rank * Nl, (rank + 1) * Nl)
        out, lse = ring_block_list_attention(q[:, :, rows].to(dev), k[:, :, rows].to(dev),
                                             v[:, :, rows].to(dev), bl, route_block=RB, is_causal=True)
        torch.cuda.synchronize()
        q_out.put((rank, "ok", out.cpu().float().numpy(), lse.cpu().numpy()))  # by value
    except Exception as e:
        q_out.put((rank, "error", repr(e), None))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_ring_over_nccl_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = dict((r, (s, a, b)) for r, s, a, b in (q.get(timeout=300) for _ in procs))
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    Z, H, Hkv, N, D, RB = 1, 4, 2, 2048, 128, 128
    gen = torch.Generator().manual_seed(9)
    qf = torch.randn(Z, H, N, D, generator=gen).bfloat16().to(DEV)
    kf = torch.randn(Z, Hkv, N, D, generator=gen).bfloat16().to(DEV)
    vf = torch.randn(Z, Hkv, N, D, generator=gen).bfloat16().to(DEV)
    router = tree_router(Z, H, N // RB, 5).to(DEV)
    bl = build_block_lists(router, 2, is_causal=True, sink_block=True, arity=2)
    ref, _ = block_list_attention(qf, kf, vf, bl, route_block=RB, is_causal=True, return_lse=True)
    for r in range(2):
        status, out, _ = res[r]
        assert status == "ok", out
        assert_half_close(torch.from_numpy(out), ref[:, :, r * N // 2:(r + 1) * N // 2].float().cpu(), f"rank {r}")

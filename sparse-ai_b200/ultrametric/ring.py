"""Sequence-sharded block-list attention forward for very long prefill (the KV ring).

The reference has no context parallelism (its forward's LSE output,
``src/ultrametric/block_list.py:467-470``, is the hook a ring needs).  Here each of P ranks
holds a contiguous chunk of ``N/P`` query rows and the matching K/V rows; the global block
lists are tiny and every rank holds all of them.  In P hops the K/V chunks rotate around
the ring (rank r sends to r+1 and receives from r-1 into a second buffer; with NCCL the
transfer runs beside this hop's compute): at hop j rank r attends its queries to chunk
``c = (r - j) mod P``, restricted to the kept block pairs that fall in that chunk, and
merges the partial (output, LSE) into an fp32 accumulator by log-sum-exp weights
(``sa_attention_lse_merge``).

Causality needs no kernel change: the diagonal chunk (c == r) runs causally, earlier
chunks lie entirely before this rank's queries, and later chunks hold no kept pair of a
causal list, so those hops are skipped.

``attn`` and ``merge`` can be replaced (same signatures) so that the schedule is testable
on CPU ranks; by default they are this package's CUDA entry points.
"""

from __future__ import annotations

import math
from typing import Callable, Optional

import torch

from . import _native as nat
from .block_list import BlockLists, _fwd


def chunk_lists(lists: torch.Tensor, counts: torch.Tensor, q_lo: int, q_hi: int, k_lo: int,
                k_hi: int) -> tuple[torch.Tensor, torch.Tensor]:
    """The lists of query blocks [q_lo, q_hi) restricted to key blocks [k_lo, k_hi) and
    re-based to that range (ascending, zero padded).  Lists are ascending, so the entries
    of a key range are one contiguous run of each row."""
    L = lists[:, :, q_lo:q_hi].long()
    cnt = counts[:, :, q_lo:q_hi].long()
    mc = max(L.shape[-1], 1)
    slot = torch.arange(L.shape[-1], device=L.device)
    valid = slot < cnt[..., None]
    start = ((L < k_lo) & valid).sum(-1)
    n = ((L >= k_lo) & (L < k_hi) & valid).sum(-1)
    idx = (start[..., None] + slot).clamp_max(mc - 1)
    sub = torch.gather(L, -1, idx) - k_lo
    sub = torch.where(slot < n[..., None], sub, torch.zeros_like(sub))
    return sub.to(torch.int32).contiguous(), n.to(torch.int32).contiguous()


def _attn_cuda(q, k, v, lists, counts, route_block, is_causal, scale):
    return _fwd(q, k, v, lists, counts, route_block, is_causal, scale, True, None)


class _CudaMerge:
    """fp32 accumulator + ``sa_attention_lse_merge``."""

    def __init__(self, q: torch.Tensor):
        Z, H, N, D = q.shape
        self.acc = torch.empty((Z, H, N, D), dtype=torch.float32, device=q.device)
        self.lse = torch.empty((Z, H, N), dtype=torch.float32, device=q.device)
        self.dtype = q.dtype

    def __call__(self, o, lse, first: bool, out: Optional[torch.Tensor]):
        Z, H, N, D = o.shape
        nat.check(nat.lib().sa_attention_lse_merge(
            nat.float_code(o.dtype), Z, H, N, D, o.data_ptr(), nat.strides(o), lse.data_ptr(),
            self.acc.data_ptr(), self.lse.data_ptr(), int(first), nat.ptr(out),
            nat.strides(out) if out is not None else None, nat.stream_of(o)), "lse merge")


def ring_hops(rank: int, world: int, is_causal: bool) -> list[tuple[int, int, bool]]:
    """(hop, visiting chunk, causal?) for the hops rank ``rank`` computes, in ring order."""
    hops = []
    for j in range(world):
        c = (rank - j) % world
        if is_causal and c > rank:
            continue  # a causal list holds no pair with a later chunk
        hops.append((j, c, is_causal and c == rank))
    return hops


def ring_block_list_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                              block_lists: BlockLists, *, route_block: int = 128,
                              is_causal: bool = False, sm_scale: Optional[float] = None,
                              group=None, attn: Optional[Callable] = None,
                              merge_factory: Optional[Callable] = None,
                              ) -> tuple[torch.Tensor, torch.Tensor]:
    """Block-list attention forward over a sequence split across the ranks of ``group``.

    q: (Z, H, N/P, D) this rank's query rows (chunk ``rank``); k, v: (Z, Hkv, N/P, D) the
    matching K/V rows; ``block_lists``: the global lists for all N/route_block query
    blocks.  N/P must be a multiple of ``route_block``.  Returns this rank's (out, lse)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    Z, H, Nl, D = q.shape
    if k.shape != v.shape or k.shape[0] != Z or k.shape[2] != Nl or k.shape[3] != D:
        raise ValueError("k and v must be (Z, Hkv, N/P, D) chunks matching q")
    if Nl % route_block:
        raise ValueError(f"the per-rank chunk ({Nl} rows) must be a multiple of route_block")
    nbl = Nl // route_block
    if block_lists.lists.shape[2] != nbl * world:
        raise ValueError(f"block_lists cover {block_lists.lists.shape[2]} query blocks, "
                         f"expected {nbl * world} (= N / route_block)")
    scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(D)
    attn = attn or _attn_cuda
    merge = (merge_factory or _CudaMerge)(q)
    hops = ring_hops(rank, world, is_causal)
    last_j = hops[-1][0]
    out = torch.empty_like(q)

    kv = torch.stack([k, v]).contiguous()
    nxt = torch.empty_like(kv)
    first = True
    for j in range(world):
        reqs = []
        if j < world - 1:  # rotate: send this chunk on, receive the next one
            ops = [dist.P2POp(dist.isend, kv, (rank + 1) % world, group),
                   dist.P2POp(dist.irecv, nxt, (rank - 1) % world, group)]
            reqs = dist.batch_isend_irecv(ops)
        hop = next((h for h in hops if h[0] == j), None)
        if hop is not None:
            _, c, causal = hop
            sub, cnt = chunk_lists(block_lists.lists, block_lists.counts, rank * nbl,
                                   (rank + 1) * nbl, c * nbl, (c + 1) * nbl)
            o_j, lse_j = attn(q, kv[0], kv[1], sub, cnt, route_block, causal, scale)
            merge(o_j, lse_j, first, out if j == last_j else None)
            first = False
        for rq in reqs:
            rq.wait()
        if j < world - 1:
            kv, nxt = nxt, kv
    return out, merge.lse


def ring_emulate(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_lists: BlockLists,
                 world: int, *, route_block: int = 128, is_causal: bool = False,
                 sm_scale: Optional[float] = None) -> tuple[torch.Tensor, torch.Tensor]:
    """The ring's per-rank hop computations and merges run one rank after another on one
    device (no transfer): same chunk lists, attention and merge calls as
    ``ring_block_list_attention``.  q, k, v are the full (Z, *, N, D) tensors."""
    Z, H, N, D = q.shape
    if N % world or (N // world) % route_block:
        raise ValueError("N must split into world chunks that are multiples of route_block")
    Nl = N // world
    nbl = Nl // route_block
    scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(D)
    outs, lses = [], []
    for rank in range(world):
        rows = slice(rank * Nl, (rank + 1) * Nl)
        qr = q[:, :, rows]
        merge = _CudaMerge(qr)
        out = torch.empty_like(qr)
        hops = ring_hops(rank, world, is_causal)
        for i, (_, c, causal) in enumerate(hops):
            kr, vr = k[:, :, c * Nl:(c + 1) * Nl], v[:, :, c * Nl:(c + 1) * Nl]
            sub, cnt = chunk_lists(block_lists.lists, block_lists.counts, rank * nbl,
                                   (rank + 1) * nbl, c * nbl, (c + 1) * nbl)
            o_j, lse_j = _attn_cuda(qr, kr, vr, sub, cnt, route_block, causal, scale)
            merge(o_j, lse_j, i == 0, out if i == len(hops) - 1 else None)
        outs.append(out)
        lses.append(merge.lse)
    return torch.cat(outs, dim=2), torch.cat(lses, dim=2)

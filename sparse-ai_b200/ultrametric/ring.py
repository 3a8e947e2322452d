"""Sequence-sharded block-list attention forward for very long prefill (the KV ring).

The reference has no context parallelism (its forward's LSE output,
``src/ultrametric/block_list.py:467-470``, is the hook a ring needs).  Here each of P ranks
holds a contiguous chunk of ``N/P`` query rows and the matching K/V rows; the global block
lists are tiny and every rank holds all of them.  At hop j rank r attends its queries to
chunk ``c = (r - j) mod P``, restricted to the kept block pairs that fall in that chunk,
and merges the partial (output, LSE) into an fp32 accumulator by log-sum-exp weights
(``sa_attention_lse_merge``).  Only the key blocks that rank r's lists reference leave
rank c (a sparse ring: for tree routes these are few -- the sink block and subtrees that
straddle a chunk boundary), so the exchange is small next to the compute.

Causality needs no kernel change: the diagonal chunk (c == r) runs causally, earlier
chunks lie entirely before this rank's queries, and later chunks hold no kept pair of a
causal list, so those hops are skipped.

With contiguous chunks a causal ring is unbalanced: rank r computes r + 1 hops and the last
rank carries the most work.  ``layout="zigzag"`` splits the sequence into 2P chunks and gives
rank r chunks r and 2P - 1 - r (one early, one late), stored one after the other in its local
q / k / v.  Every rank then holds the same causal work.  In local order the two chunks keep
their global order, so the diagonal hop still runs causally on local indices, and every other
hop is fully visible where its lists have entries.

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


def chunk_lists_multi(lists: torch.Tensor, counts: torch.Tensor, q_ranges, k_ranges
                      ) -> tuple[torch.Tensor, torch.Tensor]:
    """The lists of the query blocks in ``q_ranges`` (a list of [lo, hi) block ranges, taken
    in order as the local query blocks) restricted to the key blocks in ``k_ranges`` and
    re-based to the local key order (the ranges one after the other).  The ranges are
    ascending and disjoint, so the mapping keeps each row ascending."""
    L = torch.cat([lists[:, :, lo:hi] for lo, hi in q_ranges], dim=2).long()
    cnt = torch.cat([counts[:, :, lo:hi] for lo, hi in q_ranges], dim=2).long()
    mc = max(L.shape[-1], 1)
    slot = torch.arange(L.shape[-1], device=L.device)
    valid = slot < cnt[..., None]
    local = torch.full_like(L, -1)
    base = 0
    for lo, hi in k_ranges:
        inr = valid & (L >= lo) & (L < hi)
        local = torch.where(inr, L - lo + base, local)
        base += hi - lo
    keep = local >= 0
    n = keep.sum(-1)
    pos = torch.cumsum(keep.long(), -1) - 1
    sub = torch.zeros_like(L)
    sub.scatter_(-1, torch.where(keep, pos, torch.full_like(pos, mc - 1)).clamp_min(0),
                 torch.where(keep, local, torch.zeros_like(local)))
    # slots past n: zero (a masked scatter may have written the last slot)
    sub = torch.where(slot < n[..., None], sub, torch.zeros_like(sub))
    return sub.to(torch.int32).contiguous(), n.to(torch.int32).contiguous()


def rank_chunks(rank: int, world: int, layout: str) -> list[int]:
    """Chunk ids (in units of the layout's chunk size) that ``rank`` holds, in local order."""
    if layout == "zigzag":
        return [rank, 2 * world - 1 - rank]
    return [rank]


def _attn_cuda(q, k, v, lists, counts, route_block, is_causal, scale):
    return _fwd(q, k, v, lists, counts, route_block, is_causal, scale, True, None)


class _CudaMerge:
    """fp32 accumulator + ``sa_attention_lse_merge``."""

    def __init__(self, q: torch.Tensor):
        Z, H, N, D = q.shape
        self.acc = torch.empty((Z, H, N, D), dtype=torch.float32, device=q.device)
        self.lse = torch.empty((Z, H, N), dtype=torch.float32, device=q.device)
        self.dtype = q.dtype

    def finish(self, out: torch.Tensor) -> None:
        out.copy_(self.acc.to(out.dtype))

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


def reference_masks(lists: torch.Tensor, counts: torch.Tensor, owner, world: int) -> torch.Tensor:
    """(world, NB) bool: ref[r, kb] = some query block held by rank r lists key block kb.
    ``owner``: (NB,) rank of each query block, or an int (blocks per rank, contiguous)."""
    Z, H, NB, mc = lists.shape
    slot = torch.arange(mc, device=lists.device)
    valid = slot < counts.long()[..., None]
    if isinstance(owner, int):
        owner = torch.arange(NB, device=lists.device) // owner
    owner = owner.to(lists.device).view(1, 1, NB, 1)
    flat = torch.where(valid, owner * (NB + 1) + lists.long(), torch.full_like(lists, NB, dtype=torch.long))
    ref = torch.zeros(world * (NB + 1), dtype=torch.bool, device=lists.device)
    ref[flat.reshape(-1)] = True
    return ref.view(world, NB + 1)[:, :NB]


class RingPlan:
    """One rank's ring schedule for one set of block lists, built once (two small host
    reads) and reused by every call with those lists:

    * ``hops``: (rank whose K/V it reads, causal?, local lists, counts) for the hops this rank
      computes (lists in this rank's local query order against that rank's local key order);
    * ``exchange``: per hop j > 0, the local rows of this rank's K/V that rank r + j
      references (sent) and the local rows of rank r - j's K/V that this rank references
      (received).

    ``layout``: "contiguous" (rank r holds rows [r N/P, (r+1) N/P)) or "zigzag" (rank r holds
    chunks r and 2P - 1 - r of N / 2P rows, one after the other)."""

    def __init__(self, block_lists: BlockLists, world: int, rank: int, rows_per_rank: int,
                 route_block: int, is_causal: bool, layout: str = "contiguous"):
        if layout not in ("contiguous", "zigzag"):
            raise ValueError(f"unknown ring layout {layout!r}")
        nparts = len(rank_chunks(rank, world, layout))
        if rows_per_rank % (route_block * nparts):
            raise ValueError(f"the per-rank rows ({rows_per_rank}) must split into {nparts} chunk(s) "
                             f"that are multiples of route_block")
        nbc = rows_per_rank // route_block // nparts  # blocks per chunk
        lists, counts = block_lists.lists, block_lists.counts
        if lists.shape[2] != nbc * nparts * world:
            raise ValueError(f"block_lists cover {lists.shape[2]} query blocks, "
                             f"expected {nbc * nparts * world} (= N / route_block)")
        mc = int(counts.max()) if counts.numel() else 0  # sync-free lists are NB slots wide
        lists = lists[..., :max(mc, 1)]
        self.world, self.rank, self.rows, self.route_block = world, rank, rows_per_rank, route_block
        self.is_causal, self.layout = is_causal, layout
        ranges = lambda r: [(c * nbc, (c + 1) * nbc) for c in rank_chunks(r, world, layout)]
        self.hops = []
        for j in range(world):
            c = (rank - j) % world
            if layout == "contiguous":
                if is_causal and c > rank:
                    continue  # a causal list holds no pair with a later chunk
                sub, cnt = chunk_lists(lists, counts, rank * nbc, (rank + 1) * nbc, c * nbc, (c + 1) * nbc)
            else:
                sub, cnt = chunk_lists_multi(lists, counts, ranges(rank), ranges(c))
                if c != rank and int(cnt.sum()) == 0:
                    continue
            # only the diagonal hop needs the token-level causal mask: in local order the two
            # zigzag chunks keep their global order, and other hops' listed pairs are visible
            self.hops.append((c, is_causal and c == rank, sub, cnt))
        self.exchange = []
        if world > 1:
            # owner of each global query block, its local key position on the owning rank
            NB = lists.shape[2]
            owner = torch.empty(NB, dtype=torch.long)
            lpos = torch.empty(NB, dtype=torch.long)
            for r in range(world):
                for i, (lo, hi) in enumerate(ranges(r)):
                    owner[lo:hi] = r
                    lpos[lo:hi] = torch.arange(hi - lo) + i * nbc
            ref = reference_masks(lists, counts, owner.to(lists.device), world).cpu()
            dev = lists.device
            rows = torch.arange(route_block)
            to_rows = lambda b: (b.view(-1, 1) * route_block + rows).reshape(-1).to(dev)
            for j in range(1, world):
                dst, src = (rank + j) % world, (rank - j) % world
                mine = (owner == rank).nonzero().view(-1)    # global blocks this rank holds
                theirs = (owner == src).nonzero().view(-1)
                give = lpos[mine[ref[dst, mine]]]
                need = lpos[theirs[ref[rank, theirs]]]
                self.exchange.append((dst, to_rows(give) if give.numel() else None,
                                      src, to_rows(need) if need.numel() else None))


def _fwd_direct(q, k, v, lists, counts, route_block, is_causal, scale, out, lse, accumulate, ws):
    """The forward into (out, lse), or continuing from them, with the planner workspace ``ws``
    (heaviest-first work queue; None: static round-robin schedule)."""
    Z, H, N, D = q.shape
    wp, wn = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
    if accumulate:
        nat.check(nat.lib().sa_block_list_attention_fwd_accumulate(
            nat.float_code(q.dtype), Z, H, k.shape[1], N, D, route_block, q.data_ptr(), nat.strides(q),
            k.data_ptr(), nat.strides(k), v.data_ptr(), nat.strides(v), out.data_ptr(), nat.strides(out),
            lse.data_ptr(), lists.data_ptr(), lists.shape[-1], counts.data_ptr(), int(bool(is_causal)),
            float(scale), wp, wn, nat.stream_of(q)), "accumulating forward")
    else:
        nat.check(nat.lib().sa_block_list_attention_fwd(
            nat.float_code(q.dtype), Z, H, k.shape[1], N, D, route_block, q.data_ptr(), nat.strides(q),
            k.data_ptr(), nat.strides(k), v.data_ptr(), nat.strides(v), out.data_ptr(), nat.strides(out),
            lse.data_ptr(), lists.data_ptr(), lists.shape[-1], counts.data_ptr(), None, 0, None,
            int(bool(is_causal)), float(scale), wp, wn, nat.stream_of(q)), "forward")


def _accumulate_ok(q: torch.Tensor, route_block: int) -> bool:
    return q.dtype in (torch.bfloat16, torch.float16) and q.shape[-1] in (64, 128) and route_block % 128 == 0


def ring_block_list_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                              block_lists: BlockLists, *, route_block: int = 128,
                              is_causal: bool = False, sm_scale: Optional[float] = None,
                              group=None, plan: Optional[RingPlan] = None,
                              attn: Optional[Callable] = None,
                              merge_factory: Optional[Callable] = None,
                              layout: str = "contiguous",
                              ) -> tuple[torch.Tensor, torch.Tensor]:
    """Block-list attention forward over a sequence split across the ranks of ``group``.

    q: (Z, H, N/P, D) this rank's query rows (``layout`` "contiguous": chunk ``rank``;
    "zigzag": chunks ``rank`` and ``2P - 1 - rank`` of N/2P rows, in that order); k, v:
    (Z, Hkv, N/P, D) the matching K/V rows; ``block_lists``: the global lists for all
    N/route_block query blocks.  Chunks must be multiples of ``route_block``.  ``plan``: a
    ``RingPlan`` built once for these lists (else one is built here).  Returns this rank's
    (out, lse) in its local row order.

    Hop j pairs rank r with ranks r - j (whose chunk it attends) and r + j (which attends
    r's chunk).  Only the key blocks that the receiver's lists reference cross the link --
    all ranks hold the global lists, so sender and receiver agree on them without asking:
    they are gathered into one buffer, exchanged with send/recv (all hops' exchanges are
    posted at once and run beside the diagonal hop's compute), and put back at their rows
    of a chunk-sized buffer that the kernel reads through the hop's lists (rows it does not
    list are never read).  Hops after the first continue the forward from the previous
    output and LSE in place (``sa_block_list_attention_fwd_accumulate``); shapes outside
    the tensor-core path, and injected ``attn`` / ``merge_factory``, merge partials
    instead."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    Z, H, Nl, D = q.shape
    Hkv = k.shape[1]
    if k.shape != v.shape or k.shape[0] != Z or k.shape[2] != Nl or k.shape[3] != D:
        raise ValueError("k and v must be (Z, Hkv, N/P, D) chunks matching q")
    if plan is None:
        plan = RingPlan(block_lists, world, rank, Nl, route_block, is_causal, layout)
    elif (plan.world, plan.rank, plan.rows, plan.route_block, plan.is_causal) != (
            world, rank, Nl, route_block, is_causal):
        raise ValueError("plan was built for another ring layout")
    scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(D)
    accumulate = attn is None and merge_factory is None and _accumulate_ok(q, route_block)
    out = torch.empty_like(q)
    lse = torch.empty((Z, H, Nl), dtype=torch.float32, device=q.device)
    merge = None if accumulate else (merge_factory or _CudaMerge)(q)
    attn = attn or _attn_cuda

    recv, ops = {}, []
    for dst, give, src, need in plan.exchange:
        if give is not None:
            send = torch.stack([k.index_select(2, give), v.index_select(2, give)])
            ops.append(dist.P2POp(dist.isend, send, dst, group))
        if need is not None:
            buf = torch.empty((2, Z, Hkv, need.numel(), D), dtype=k.dtype, device=q.device)
            ops.append(dist.P2POp(dist.irecv, buf, src, group))
            recv[src] = (need, buf)
    reqs = dist.batch_isend_irecv(ops) if ops else []

    first = True
    chunk_k = chunk_v = None
    ws = None
    n_hops = len(plan.hops)
    for i, (c, causal, sub, cnt) in enumerate(plan.hops):
        last = i == n_hops - 1
        if c == rank:
            kc, vc = k, v
        elif c not in recv:  # none of this rank's lists reaches chunk c
            if last and merge is not None and not first:
                merge.finish(out)
            continue
        else:
            for rq in reqs:
                rq.wait()
            reqs = []
            need, buf = recv[c]
            if chunk_k is None:  # the kernel reads only listed rows; a dense stand-in reads all
                alloc = torch.empty_like if accumulate else torch.zeros_like
                chunk_k, chunk_v = alloc(k), alloc(v)
            chunk_k.index_copy_(2, need, buf[0])
            chunk_v.index_copy_(2, need, buf[1])
            kc, vc = chunk_k, chunk_v
        if accumulate:
            if ws is None:
                ws_bytes = int(nat.lib().sa_block_list_attention_fwd_workspace_bytes(
                    Z, H, Nl, D, route_block))
                ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=q.device)
            _fwd_direct(q, kc, vc, sub, cnt, route_block, causal, scale, out, lse, not first, ws)
        else:
            o_j, lse_j = attn(q, kc, vc, sub, cnt, route_block, causal, scale)
            merge(o_j, lse_j, first, out if last else None)
        first = False
    for rq in reqs:
        rq.wait()
    if merge is not None:
        lse = merge.lse
    if first:  # no hop attended anything (empty lists): zero rows, -inf LSE
        out.zero_()
        lse.fill_(float("-inf"))
    return out, lse


def ring_emulate(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_lists: BlockLists,
                 world: int, *, route_block: int = 128, is_causal: bool = False,
                 sm_scale: Optional[float] = None, layout: str = "contiguous"
                 ) -> tuple[torch.Tensor, torch.Tensor]:
    """The ring's per-rank hop computations and merges run one rank after another on one
    device (no transfer): same plans, lists, attention and merge calls as
    ``ring_block_list_attention``.  q, k, v are the full (Z, *, N, D) tensors; the result is
    in global row order."""
    Z, H, N, D = q.shape
    nparts = 2 if layout == "zigzag" else 1
    if N % (world * nparts) or (N // (world * nparts)) % route_block:
        raise ValueError("N must split into chunks that are multiples of route_block")
    Nl = N // world
    cs = Nl // nparts
    scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(D)
    out_all = torch.empty_like(q)
    lse_all = torch.empty((Z, H, N), dtype=torch.float32, device=q.device)
    local_rows = lambda r: torch.cat([torch.arange(c * cs, (c + 1) * cs)
                                      for c in rank_chunks(r, world, layout)]).to(q.device)
    for rank in range(world):
        rows = local_rows(rank)
        qr = q.index_select(2, rows)
        plan = RingPlan(block_lists, world, rank, Nl, route_block, is_causal, layout)
        acc = _accumulate_ok(qr, route_block)
        merge = None if acc else _CudaMerge(qr)
        out = torch.empty_like(qr)
        lse = torch.empty(qr.shape[:3], dtype=torch.float32, device=q.device)
        for i, (c, causal, sub, cnt) in enumerate(plan.hops):
            kr, vr = k.index_select(2, local_rows(c)), v.index_select(2, local_rows(c))
            if acc:
                # odd ranks without a planner workspace: both schedules stay exercised
                ws = None
                if rank % 2 == 0:
                    ws = torch.empty(max(int(nat.lib().sa_block_list_attention_fwd_workspace_bytes(
                        Z, H, Nl, D, route_block)), 256), dtype=torch.uint8, device=q.device)
                _fwd_direct(qr, kr, vr, sub, cnt, route_block, causal, scale, out, lse, i > 0, ws)
            else:
                o_j, lse_j = _attn_cuda(qr, kr, vr, sub, cnt, route_block, causal, scale)
                merge(o_j, lse_j, i == 0, out if i == len(plan.hops) - 1 else None)
        out_all.index_copy_(2, rows, out)
        lse_all.index_copy_(2, rows, lse if acc else merge.lse)
    return out_all, lse_all

"""Router outputs -> block lists for sparse-ai's LLaMA surgery prefill, in one C-ABI call.

``SurgicalLlamaAttention._block_list_prefill`` (src/llama_surgery/surgery.py:520-598 of
sparse-ai) turns its router's assignments into per-block routes with torch glue -- token
argmax, one-hot, a sum over each route block, argmax (surgery.py:543-547), or the argmax of
block-level assignments (:533-538) -- and then calls ``build_block_lists(block_route, r,
is_causal=True, sink_block=True, local_blocks=..., arity=p)``.
``build_block_lists_from_assignments`` does all of it on the device (the vote kernel and
the compaction kernel of ``sa_build_block_lists_from_assignments``), with no host sync, and
returns the same ``BlockLists`` (sync-free form: ``max_count = NB``) and, on request, the
block routes.

``RouteListCache`` is the cross-layer reuse of surgery.py:301-315 and :377-391: with
``surgical_route_stride = s > 1`` the anchor layers (index % s == 0) route themselves and
the layers between reuse their anchor's routes, here the anchor's lists, as long as the
heads, head dim, batch and sequence length agree.
"""

from __future__ import annotations

from typing import Optional, Sequence, Union

import torch

from . import _native as nat
from .block_list import BlockLists

DepthLike = Union[int, Sequence[int], torch.Tensor]


@torch.no_grad()
def build_block_lists_from_assignments(
    assignments: torch.Tensor,
    r: int,
    seq_len: Optional[int] = None,
    *,
    route_block: int = 128,
    block_assignments: Optional[torch.Tensor] = None,
    req_depth: Optional[DepthLike] = None,
    is_causal: bool = True,
    sink_block: bool = True,
    local_blocks: int = 0,
    arity: Optional[int] = None,
    return_routes: bool = False,
):
    """Block lists straight from router outputs.

    assignments        (B, H, S_a, levels, p) router outputs per token (probabilities or
                       logits: only their argmax over p matters), or per route block when
                       ``S_a == ceil(seq_len / route_block) != seq_len``.
    r                  levels that vote and must agree (``r`` of surgery.py:522).
    seq_len            tokens of the sequence (default ``S_a``); tokens past it do not vote.
    block_assignments  optional (B, H, NB, levels, p) block-level router outputs; when they
                       cover all NB blocks they are used instead (surgery.py:533-535).
    req_depth          optional per-head depths (<= r) for the match (default r everywhere).
    arity              branch count (default p); codes use base max(2, arity).
    Returns BlockLists(lists (B, H, NB, NB), counts, NB), plus the (B, H, NB, r) int32
    block routes when ``return_routes``."""
    if assignments.dim() != 5:
        raise ValueError(f"assignments must be (B, H, S, levels, p), got {tuple(assignments.shape)}")
    nat.require_cuda("build_block_lists_from_assignments", assignments)
    B, H, S_a, levels, p = assignments.shape
    S = S_a if seq_len is None else int(seq_len)
    rb = int(route_block)
    if rb < 1:
        raise ValueError(f"route_block must be >= 1, got {rb}")
    NB = -(-S // rb)
    if not 0 <= r <= levels:
        raise ValueError(f"r must be in [0, {levels}], got {r}")
    src, per_block = assignments, False
    if block_assignments is not None and block_assignments.shape[2] == NB:
        src, per_block = block_assignments, True
    elif S_a == NB and NB != S:
        per_block = True
    elif S_a < S:
        raise ValueError(f"assignments cover {S_a} tokens, fewer than seq_len={S}")
    if src.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        src = src.float()
    if src.stride(-1) == 0 or src.stride(-2) == 0:
        src = src.contiguous()
    tokens = NB if per_block else S
    tpb = 1 if per_block else rb
    if req_depth is None:
        depth = torch.full((H,), int(r), dtype=torch.int32, device=src.device)
    else:
        depth = torch.as_tensor(req_depth, dtype=torch.int32).reshape(-1).to(src.device)
        if depth.numel() != H:
            raise ValueError(f"req_depth has {depth.numel()} entries, expected {H} (one per head)")
    routes = torch.empty((B, H, NB, max(r, 1)), dtype=torch.int32, device=src.device)
    lists = torch.empty((B, H, NB, max(NB, 1)), dtype=torch.int32, device=src.device)
    counts = torch.empty((B, H, NB), dtype=torch.int32, device=src.device)
    if B * H * NB:
        nat.check(nat.lib().sa_build_block_lists_from_assignments(
            src.data_ptr(), nat.float_code(src.dtype), nat.strides(src), B, H, tokens, levels, p,
            tpb, int(r), depth.data_ptr(), int(arity if arity is not None else p),
            int(bool(is_causal)), int(bool(sink_block)), int(local_blocks), routes.data_ptr(),
            lists.data_ptr(), lists.shape[-1], counts.data_ptr(), nat.stream_of(src)),
            "build_block_lists_from_assignments")
    bl = BlockLists(lists[..., :NB], counts, NB)
    if return_routes:
        return bl, routes[..., :r]
    return bl


class RouteListCache:
    """Cross-layer reuse of block lists with ``surgical_route_stride`` (surgery.py:301-315,
    377-391): layer ``l`` with ``l % stride != 0`` reuses the lists of anchor layer
    ``(l // stride) * stride`` when the entry was made for the same heads, head dim, batch
    and sequence length; anchor layers always route themselves and store their lists."""

    def __init__(self, stride: int = 1):
        self.stride = max(1, int(stride))
        self._entries = {}

    def anchor(self, layer_idx: int) -> int:
        return (int(layer_idx) // self.stride) * self.stride

    def lookup(self, layer_idx: int, *, num_heads: int, head_dim: int, batch: int, seq_len: int):
        if self.stride <= 1 or layer_idx % self.stride == 0:
            return None
        e = self._entries.get((num_heads, head_dim, self.anchor(layer_idx)))
        if e is None or e["batch"] != batch or e["seq_len"] != seq_len:
            return None
        return e["lists"]

    def store(self, layer_idx: int, block_lists, *, num_heads: int, head_dim: int, batch: int,
              seq_len: int) -> None:
        if self.stride <= 1 or layer_idx % self.stride != 0:
            return
        self._entries[(num_heads, head_dim, int(layer_idx))] = {
            "lists": block_lists, "batch": batch, "seq_len": seq_len}

    def clear(self) -> None:
        self._entries.clear()

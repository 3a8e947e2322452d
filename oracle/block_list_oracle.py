"""Block-list construction oracle (numpy; TEST INFRASTRUCTURE ONLY).

Restates ``src/ultrametric/block_list.py`` of sparse-ai:

* ``depth_vector``        -- ``_depth_tensor`` (block_list.py:93-104)
* ``structural_masks``    -- ``_apply_structural_masks`` (block_list.py:107-118)
* ``block_mask``          -- ``block_mask_reference`` (block_list.py:334-358): pairwise
  prefix comparison, shares no code with the builder restatement below.
* ``build_block_lists``   -- ``build_block_lists`` (block_list.py:170-278), including the
  mixed-radix prefix code (block_list.py:224-229), its int64 wrap-around and the
  per-level fallback when the code would overflow (block_list.py:256-258), so that the
  sync-free ``arity=`` path is reproduced bit for bit even for ids >= arity.
* ``transpose_block_lists`` -- ``build_transposed_block_lists`` (block_list.py:281-327).
"""

from __future__ import annotations

import math

import numpy as np


def depth_vector(req_depth, num_heads: int, tree_depth: int) -> np.ndarray:
    """Per-head required depth as int64 (H,), validated like block_list.py:93-104."""
    if isinstance(req_depth, (int, np.integer)):
        depth = np.full((num_heads,), int(req_depth), dtype=np.int64)
    else:
        depth = np.asarray(req_depth, dtype=np.int64).reshape(-1)
        if depth.size != num_heads:
            raise ValueError(f"req_depth has {depth.size} entries, expected {num_heads} (one per head)")
    if depth.size and (depth.min() < 0 or depth.max() > tree_depth):
        raise ValueError(f"req_depth must be in [0, {tree_depth}], got {depth.tolist()}")
    return depth


def structural_masks(match: np.ndarray, *, is_causal: bool, sink_block: bool,
                     local_blocks: int) -> np.ndarray:
    """OR the local band and sink column, AND the causal triangle (block_list.py:107-118)."""
    nb = match.shape[-1]
    idx = np.arange(nb)
    match = match.copy()
    if local_blocks > 0:
        match |= np.abs(idx[:, None] - idx[None, :]) <= local_blocks
    if sink_block:
        match[..., 0] = True
    if is_causal:
        match &= idx[:, None] >= idx[None, :]
    return match


def block_mask(router: np.ndarray, req_depth, *, is_causal=False, sink_block=False,
               local_blocks=0) -> np.ndarray:
    """(Z, H, NB, NB) bool: query block i keeps key block j iff routes agree on the first
    req_depth[h] levels, then the structural rules (block_list.py:334-358)."""
    router = np.asarray(router)
    Z, H, NB, TD = router.shape
    depth = depth_vector(req_depth, H, TD)
    out = np.empty((Z, H, NB, NB), dtype=bool)
    for h in range(H):
        d = int(depth[h])
        if d == 0:
            out[:, h] = True
        else:
            rh = router[:, h, :, :d]
            out[:, h] = (rh[:, :, None, :] == rh[:, None, :, :]).all(-1)
    return structural_masks(out, is_causal=is_causal, sink_block=sink_block,
                            local_blocks=local_blocks)


def _compact(match: np.ndarray, width: int) -> tuple[np.ndarray, np.ndarray]:
    """Stable compaction of each row's True columns into ascending slots; zero padding."""
    counts = match.sum(-1).astype(np.int32)
    lead = match.shape[:-1]
    lists = np.zeros(lead + (width,), dtype=np.int32)
    flat_m = match.reshape(-1, match.shape[-1])
    flat_l = lists.reshape(-1, width)
    for r in range(flat_m.shape[0]):
        cols = np.nonzero(flat_m[r])[0]
        flat_l[r, :cols.size] = cols[:width]
    return lists, counts


def prefix_codes(router: np.ndarray, depth: np.ndarray, base: int) -> np.ndarray:
    """Mixed-radix code sum_{l < depth[h]} r_l * base**l with int64 wrap-around
    (block_list.py:224-229)."""
    Z, H, NB, TD = router.shape
    r = router.astype(np.int64).astype(np.uint64)
    code = np.zeros((Z, H, NB), dtype=np.uint64)
    power = np.uint64(1)
    with np.errstate(over="ignore"):
        for lvl in range(TD):
            keep = (lvl < depth).astype(np.uint64).reshape(1, H, 1)
            code = code + r[..., lvl] * power * keep
            power = power * np.uint64(base)
    return code.astype(np.int64)


def build_block_lists(router: np.ndarray, req_depth, *, is_causal=False, sink_block=False,
                      local_blocks=0, arity=None):
    """Return (lists, counts, max_count) exactly as block_list.py:170-278 does.

    ``arity`` given -> sync-free semantics: ids unchecked, ``base = max(2, arity)``,
    lists padded to NB columns.  Otherwise ids must be >= 0, ``base = max(id) + 1`` and
    ``max_count`` is the largest row count.
    """
    router = np.asarray(router)
    if router.ndim != 4:
        raise ValueError(f"router_indices must be (Z, H, NB, TD), got {tuple(router.shape)}")
    Z, H, NB, TD = router.shape
    sync_free = arity is not None
    if sync_free and isinstance(req_depth, (int, np.integer)):
        if not 0 <= int(req_depth) <= TD:
            raise ValueError(f"req_depth must be in [0, {TD}], got {req_depth}")
        depth = np.full((H,), int(req_depth), dtype=np.int64)
    else:
        depth = depth_vector(req_depth, H, TD)
    r = router.astype(np.int64)
    if sync_free:
        base = max(2, int(arity))
    else:
        if r.size and int(r.min()) < 0:
            raise ValueError("router_indices must be non-negative branch ids")
        base = max(2, int(r.max()) + 1) if r.size else 2

    if TD * math.log2(base) < 62:
        code = prefix_codes(r, depth, base)
        match = code[..., :, None] == code[..., None, :]
    else:
        keep = np.arange(TD)[None, :] < depth[:, None]           # (H, TD)
        eq = (r[:, :, :, None, :] == r[:, :, None, :, :]) | ~keep[None, :, None, None, :]
        match = eq.all(-1)
    match = structural_masks(match, is_causal=is_causal, sink_block=sink_block,
                             local_blocks=local_blocks)
    counts = match.sum(-1).astype(np.int32)
    max_count = NB if sync_free else (int(counts.max()) if counts.size else 0)
    lists, counts = _compact(match, max_count)
    return lists, counts, max_count


def transpose_block_lists(lists: np.ndarray, counts: np.ndarray, max_count: int,
                          num_key_blocks=None):
    """Key block -> ascending query blocks that list it (block_list.py:281-327)."""
    Z, H, NBQ = counts.shape
    NBK = NBQ if num_key_blocks is None else int(num_key_blocks)
    if NBQ == 0 or NBK == 0 or max_count == 0:
        return (np.zeros((Z, H, NBK, 0), dtype=np.int32), np.zeros((Z, H, NBK), dtype=np.int32), 0)
    match_qk = np.zeros((Z, H, NBQ, NBK), dtype=bool)
    for z in range(Z):
        for h in range(H):
            for qb in range(NBQ):
                c = int(counts[z, h, qb])
                for kb in lists[z, h, qb, :c]:
                    if 0 <= kb < NBK:
                        match_qk[z, h, qb, kb] = True
    match_kq = np.swapaxes(match_qk, -1, -2)
    q_counts = match_kq.sum(-1).astype(np.int32)
    max_q = int(q_counts.max()) if q_counts.size else 0
    k_lists, q_counts = _compact(match_kq, max_q)
    return k_lists, q_counts, max_q


def tree_router(Z: int, H: int, NB: int, TD: int) -> np.ndarray:
    """MSB-first binary path of each block index, padded to TD levels
    (tests/test_block_list.py:37-43 of the reference)."""
    depth = max(1, math.ceil(math.log2(max(NB, 2))))
    r = np.zeros((Z, H, NB, TD), dtype=np.int32)
    for d in range(min(depth, TD)):
        r[:, :, :, d] = (np.arange(NB) >> (depth - 1 - d)) % 2
    return r

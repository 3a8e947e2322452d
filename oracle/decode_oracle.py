"""Routed paged-decode oracle (torch on CPU; TEST INFRASTRUCTURE ONLY).

Restates ``_ultrametric_decode_reference`` (src/ultrametric/kernel_decode.py:129-185) of
sparse-ai: for request b and query head h, the logical pages whose routing vector (stored
at the PHYSICAL page id, kernel_decode.py:79) agrees with the query's on the first
``req_depth`` levels, plus logical page 0 when ``sink_block`` and the last
``local_blocks`` logical pages, are concatenated (tail tokens cut at ``context_lens[b]``)
and attended with an fp32 (here: selectable) softmax at scale 1/sqrt(D).  A request with
``context_lens[b] == 0`` yields zeros.

The only extension is GQA: K/V caches may hold ``Hkv`` heads, query head h reading cache
head ``h // (H // Hkv)``; with ``Hkv == H`` this is exactly the reference.
"""

from __future__ import annotations

import torch


def selected_pages(block_tables, context_lens, router_indices, q_router_indices, req_depth,
                   local_blocks, sink_block, page_size, b, h):
    """Logical page ids selected for (request b, head h), ascending."""
    tree_depth = q_router_indices.shape[-1]
    r = min(max(int(req_depth), 0), tree_depth)
    ctx = int(context_lens[b])
    if ctx <= 0:
        return []
    n_logical = (ctx + page_size - 1) // page_size
    phys = block_tables[b, :n_logical].long()
    if r > 0:
        match = (router_indices[phys, h, :r] == q_router_indices[b, h, :r].unsqueeze(0)).all(-1)
    else:
        match = torch.ones(n_logical, dtype=torch.bool)
    if sink_block:
        match[0] = True
    if local_blocks > 0:
        match[max(0, n_logical - local_blocks):] = True
    return torch.nonzero(match).flatten().tolist()


def ultrametric_decode_reference(q, k_cache, v_cache, block_tables, context_lens, router_indices,
                                 q_router_indices, req_depth, local_blocks=0, sink_block=False,
                                 compute_dtype=torch.float32, requests=None):
    """(B, H, D) output; ``requests`` restricts the work to a subset of b (others stay 0)."""
    B, H, D = q.shape
    hkv = k_cache.shape[1]
    group = H // hkv
    page = k_cache.shape[2]
    scale = 1.0 / (D ** 0.5)
    out = torch.zeros(B, H, D, dtype=compute_dtype)
    for b in (range(B) if requests is None else requests):
        ctx = int(context_lens[b])
        if ctx <= 0:
            continue
        for h in range(H):
            pages = selected_pages(block_tables, context_lens, router_indices, q_router_indices,
                                   req_depth, local_blocks, sink_block, page, b, h)
            if not pages:
                continue
            ks, vs = [], []
            for lp in pages:
                p = int(block_tables[b, lp])
                valid = min(page, ctx - lp * page)
                ks.append(k_cache[p, h // group, :valid].to(compute_dtype))
                vs.append(v_cache[p, h // group, :valid].to(compute_dtype))
            kc = torch.cat(ks, 0)
            vc = torch.cat(vs, 0)
            s = torch.matmul(kc, q[b, h].to(compute_dtype)) * scale
            out[b, h] = torch.matmul(torch.softmax(s, dim=-1), vc)
    return out


def routed_bytes(block_tables, context_lens, router_indices, q_router_indices, req_depth,
                 local_blocks, sink_block, page_size, num_heads, num_kv_heads, head_dim,
                 elem_bytes=2):
    """Algorithmic K+V bytes a routed decode must read: every (request, KV head, page) that
    at least one query head of the group selects, valid tokens only, K and V once each."""
    group = num_heads // num_kv_heads
    total = 0
    for b in range(block_tables.shape[0]):
        ctx = int(context_lens[b])
        for g in range(num_kv_heads):
            pages = set()
            for h in range(g * group, (g + 1) * group):
                pages.update(selected_pages(block_tables, context_lens, router_indices,
                                            q_router_indices, req_depth, local_blocks,
                                            sink_block, page_size, b, h))
            for lp in pages:
                valid = min(page_size, ctx - lp * page_size)
                total += 2 * valid * head_dim * elem_bytes
    return total

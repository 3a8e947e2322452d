"""Routed sparse PagedAttention decode on B200 (sm_100a): the drop-in for sparse-ai's
``src/ultrametric/kernel_decode.py`` (``ultrametric_decode``, :188-247 there).

One C-ABI call (``sa_ultrametric_decode``) selects the routed pages of every (request, KV
head) and streams only those pages.  For bf16/fp16 caches with head_dim 64 or 128 (and page
sizes 16, 32 or multiples of 64) it runs the sm_100a fast path (``csrc/decode_sm100.cu``):
a selection kernel builds per-KV-head page lists and cuts them into balanced chunks, a
persistent kernel streams each chunk's K/V tiles with TMA and serves every query head of
the GQA group from each loaded tile, and a combine kernel merges the chunk partials by
log-sum-exp.  Other shapes and fp32 take the general split-K kernel (``csrc/decode.cu``:
16-byte ``cp.async`` loads, per-split online softmax, log-sum-exp merge).  Differences
from the reference, all supersets: ``k_cache``/``v_cache`` may hold ``H // g`` KV heads
(native GQA; the reference needs them expanded to H); a request with
``context_lens[b] == 0`` gets zeros (the reference kernel leaves ``torch.empty`` memory
there, its CPU reference writes zeros).  There is no CPU or Triton path.
"""

from __future__ import annotations

import torch

from . import _native as nat

HAS_TRITON = True  # import compatibility with the reference module


def ultrametric_decode(
    q,
    k_cache,
    v_cache,
    block_tables,
    context_lens,
    router_indices,
    q_router_indices,
    req_depth,
    local_blocks: int = 0,
    sink_block: bool = False,
):
    """Decode one token per request against a routed paged KV cache.

    q (B, H, D); k_cache, v_cache (num_pages, Hkv, page_size, D); block_tables (B, L) int32
    physical page per logical page; context_lens (B,) int32; router_indices (num_pages, H, TD)
    routing vector per PHYSICAL page and head; q_router_indices (B, H, TD).  A logical page is
    attended by head h when its route agrees with the query's on the first ``req_depth``
    levels, or it is page 0 and ``sink_block``, or it is one of the last ``local_blocks``
    pages.  Returns (B, H, D) in q.dtype.
    """
    batch_size, num_heads, head_dim = q.shape
    tree_depth = int(q_router_indices.shape[-1])
    assert tree_depth >= 1, "tree_depth must be >= 1"
    nat.require_cuda("ultrametric_decode", q, k_cache, v_cache, block_tables, context_lens,
                     router_indices, q_router_indices)
    if k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError(f"k_cache/v_cache must be (num_pages, Hkv, page_size, D); got "
                         f"{tuple(k_cache.shape)}, {tuple(v_cache.shape)}")
    num_pages, hkv, page_size, d2 = k_cache.shape
    if d2 != head_dim or hkv == 0 or num_heads % hkv:
        raise ValueError("cache head_dim / heads incompatible with q")
    if not (q.dtype == k_cache.dtype == v_cache.dtype):
        raise ValueError("q, k_cache, v_cache must share dtype")
    bt = block_tables if block_tables.dtype == torch.int32 else block_tables.to(torch.int32)
    ctx = context_lens.to(torch.int32).contiguous()
    ri = router_indices if router_indices.dtype in (torch.int32, torch.int64) else router_indices.to(torch.int64)
    qri = q_router_indices if q_router_indices.dtype in (torch.int32, torch.int64) else q_router_indices.to(torch.int64)
    kc = k_cache if k_cache.stride(-1) == 1 else k_cache.contiguous()
    vc = v_cache if v_cache.stride(-1) == 1 else v_cache.contiguous()
    qq = q if q.stride(-1) == 1 else q.contiguous()
    out = torch.empty_like(qq)
    max_logical = bt.shape[1]
    ws_bytes = int(nat.lib().sa_ultrametric_decode_workspace_bytes(
        batch_size, num_heads, hkv, head_dim, max_logical))
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=q.device)
    nat.check(nat.lib().sa_ultrametric_decode(
        nat.float_code(q.dtype), batch_size, num_heads, hkv, head_dim, page_size, num_pages,
        qq.data_ptr(), nat.strides(qq), kc.data_ptr(), nat.strides(kc), vc.data_ptr(), nat.strides(vc),
        bt.data_ptr(), nat.strides(bt), max_logical, ctx.data_ptr(),
        ri.data_ptr(), nat.int_code(ri.dtype), nat.strides(ri),
        qri.data_ptr(), nat.int_code(qri.dtype), nat.strides(qri),
        tree_depth, int(req_depth), int(local_blocks), int(bool(sink_block)),
        out.data_ptr(), nat.strides(out), ws.data_ptr(), ws.numel(), nat.stream_of(q)),
        "ultrametric_decode")
    return out

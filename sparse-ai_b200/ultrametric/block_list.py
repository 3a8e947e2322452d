"""Block-list sparse attention on B200 (sm_100a): the drop-in for sparse-ai's
``src/ultrametric/block_list.py``.

Same names, arguments, defaults, return types and ``ValueError`` messages as the
reference (block_list.py:78-90, 170-327, 968-1083), so ``from ultrametric.block_list
import block_list_attention, build_block_lists`` in ``llama_surgery/surgery.py:530``
resolves here unchanged.  Behind it every operator is one C-ABI call into hand-written
CUDA (``libsparse_ai_b200.so``):

* ``build_block_lists``            -> ``sa_build_block_lists`` (one compaction kernel)
* ``build_transposed_block_lists`` -> ``sa_build_transposed_block_lists``
* ``block_list_attention``         -> ``sa_block_list_attention_fwd`` / ``_bwd``
  (tcgen05 + TMA + TMEM for bf16/fp16 with head_dim 64/128 and route_block % 128 == 0;
  CUDA-core kernels for fp32 and the remaining shapes)

Additions over the reference: native GQA (``k``/``v`` may have ``H // g`` heads), and
``build_block_lists_from_mask``.  ``block_m``, ``block_n``, ``num_warps`` and
``num_stages`` are accepted for signature compatibility; the sm_100a kernels fix their
own tiles.  There is no CPU or Triton path: non-CUDA tensors raise ``RuntimeError``.
"""

from __future__ import annotations

import warnings

import math
from typing import NamedTuple, Optional, Sequence, Union

import torch

from . import _native as nat

# Kept for import compatibility with the reference (__init__.py:25,53 there); the backend
# here is hand-written CUDA, not Triton.
HAS_TRITON = True

DepthLike = Union[int, Sequence[int], torch.Tensor]

__all__ = [
    "HAS_TRITON",
    "BlockLists",
    "build_block_lists",
    "build_block_lists_from_mask",
    "build_transposed_block_lists",
    "block_list_attention",
    "routed_block_attention",
]


class BlockLists(NamedTuple):
    """Active key route-blocks per query route-block (or transposed).

    lists:     (Z, H, NB, max_count) int32, ascending per row; slots >= counts are padding.
    counts:    (Z, H, NB) int32.
    max_count: int, row stride of ``lists``.
    """

    lists: torch.Tensor
    counts: torch.Tensor
    max_count: int


def _depth_list(req_depth: DepthLike, num_heads: int, tree_depth: int) -> list[int]:
    """Per-head depths on the host, validated like block_list.py:93-104."""
    if isinstance(req_depth, int):
        depth = [int(req_depth)] * num_heads
    else:
        depth = torch.as_tensor(req_depth, dtype=torch.int64).reshape(-1).tolist()
        if len(depth) != num_heads:
            raise ValueError(f"req_depth has {len(depth)} entries, expected {num_heads} (one per head)")
    if depth and (min(depth) < 0 or max(depth) > tree_depth):
        raise ValueError(f"req_depth must be in [0, {tree_depth}], got {depth}")
    return depth


@torch.no_grad()
def build_block_lists(
    router_indices: torch.Tensor,
    req_depth: DepthLike,
    *,
    is_causal: bool = False,
    sink_block: bool = False,
    local_blocks: int = 0,
    arity: Optional[int] = None,
) -> BlockLists:
    """Per-row ascending active key-block lists from per-block routing vectors.

    Query block i keeps key block j iff their routing vectors agree on the first
    ``req_depth[h]`` levels, OR |i - j| <= local_blocks, OR (sink_block and j == 0); AND
    j <= i when ``is_causal`` (block_list.py:37-38,107-118).  ``arity`` given -> sync-free:
    ids are not validated, ``max_count = NB`` and no device->host read happens.  Without
    it ids must be >= 0 and ``max_count`` is the exact maximum (one host read, as in the
    reference).  Bit-exact with the reference builder, including its mixed-radix code
    (block_list.py:224-229) and per-level fallback (:256-258).
    """
    if router_indices.dim() != 4:
        raise ValueError(f"router_indices must be (Z, H, NB, TD), got {tuple(router_indices.shape)}")
    nat.require_cuda("build_block_lists", router_indices)
    Z, H, NB, TD = router_indices.shape
    device = router_indices.device
    sync_free = arity is not None
    if sync_free and isinstance(req_depth, int):
        if not 0 <= req_depth <= TD:
            raise ValueError(f"req_depth must be in [0, {TD}], got {req_depth}")
        depth_dev = torch.full((H,), int(req_depth), dtype=torch.int32, device=device)
    else:
        depth_dev = torch.tensor(_depth_list(req_depth, H, TD), dtype=torch.int32, device=device)
    r = router_indices
    if r.dtype not in (torch.int32, torch.int64):
        r = r.to(torch.int64)
    if sync_free:
        base = max(2, int(arity))
    else:
        if r.numel() and int(r.min()) < 0:
            raise ValueError("router_indices must be non-negative branch ids")
        base = max(2, int(r.max()) + 1) if r.numel() else 2
    use_codes = TD * math.log2(base) < 62

    lists_full = torch.empty((Z, H, NB, max(NB, 1)), dtype=torch.int32, device=device)
    counts = torch.empty((Z, H, NB), dtype=torch.int32, device=device)
    if Z * H * NB:
        nat.check(nat.lib().sa_build_block_lists(
            r.data_ptr(), nat.int_code(r.dtype), nat.strides(r), Z, H, NB, TD,
            depth_dev.data_ptr(), base, int(use_codes), int(bool(is_causal)),
            int(bool(sink_block)), int(local_blocks), lists_full.data_ptr(), lists_full.shape[-1],
            counts.data_ptr(), nat.stream_of(r)), "build_block_lists")
    lists_full = lists_full[..., :NB]
    if sync_free:
        return BlockLists(lists_full, counts, NB)
    max_count = int(counts.max()) if counts.numel() else 0
    return BlockLists(lists_full[..., :max_count].contiguous(), counts, max_count)


@torch.no_grad()
def build_block_lists_from_mask(block_mask: torch.Tensor, *, sync_free: bool = True) -> BlockLists:
    """Compact a (Z, H, NB, NB) boolean block mask into ascending lists (superset API).

    Row i of head h lists the key blocks j with ``block_mask[z, h, i, j]`` in ascending
    order, zero padded (the compaction of block_list.py:269-278).  Runs on the
    transposition kernel: column j of the mask is handed over as an unordered "list" whose
    slot t holds t where ``mask[t, j]`` and the out-of-range id NB elsewhere (ignored), so
    the kernel's output row i is exactly the ascending j with ``mask[i, j]``.
    """
    if block_mask.dim() != 4 or block_mask.shape[-1] != block_mask.shape[-2]:
        raise ValueError(f"block_mask must be (Z, H, NB, NB), got {tuple(block_mask.shape)}")
    nat.require_cuda("build_block_lists_from_mask", block_mask)
    Z, H, NB, _ = block_mask.shape
    m_t = block_mask.to(torch.bool).transpose(-1, -2)
    rows = torch.arange(NB, dtype=torch.int32, device=m_t.device).expand(Z, H, NB, NB)
    cols_in = torch.where(m_t, rows, torch.full_like(rows, NB)).contiguous()
    counts_in = torch.full((Z, H, NB), NB, dtype=torch.int32, device=m_t.device)
    k_lists = torch.empty((Z, H, NB, max(NB, 1)), dtype=torch.int32, device=m_t.device)
    q_counts = torch.empty((Z, H, NB), dtype=torch.int32, device=m_t.device)
    if Z * H * NB:
        nat.check(nat.lib().sa_build_transposed_block_lists(
            cols_in.data_ptr(), NB, counts_in.data_ptr(), Z * H, NB, NB,
            k_lists.data_ptr(), k_lists.shape[-1], q_counts.data_ptr(), None,
            nat.stream_of(cols_in)), "build_block_lists_from_mask")
    k_lists = k_lists[..., :NB]
    if sync_free:
        return BlockLists(k_lists, q_counts, NB)
    mc = int(q_counts.max()) if q_counts.numel() else 0
    return BlockLists(k_lists[..., :mc].contiguous(), q_counts, mc)


@torch.no_grad()
def build_transposed_block_lists(
    block_lists: BlockLists,
    num_key_blocks: Optional[int] = None,
) -> BlockLists:
    """Key block -> ascending query blocks that attend to it (block_list.py:281-327).

    Returns ``BlockLists(k_lists, q_counts, max_q_count)`` with the exact maximum (one
    device->host read, as in the reference)."""
    lists, counts, max_count = block_lists
    Z, H, NB_Q = counts.shape
    NB_K = num_key_blocks if num_key_blocks is not None else NB_Q
    device = lists.device
    if NB_Q == 0 or NB_K == 0 or max_count == 0:
        return BlockLists(torch.zeros((Z, H, NB_K, 0), dtype=torch.int32, device=device),
                          torch.zeros((Z, H, NB_K), dtype=torch.int32, device=device), 0)
    nat.require_cuda("build_transposed_block_lists", lists, counts)
    lists = lists.to(torch.int32).contiguous()
    counts = counts.to(torch.int32).contiguous()
    k_lists = torch.empty((Z, H, NB_K, NB_Q), dtype=torch.int32, device=device)
    q_counts = torch.empty((Z, H, NB_K), dtype=torch.int32, device=device)
    nat.check(nat.lib().sa_build_transposed_block_lists(
        lists.data_ptr(), lists.shape[-1], counts.data_ptr(), Z * H, NB_Q, NB_K,
        k_lists.data_ptr(), NB_Q, q_counts.data_ptr(), None, nat.stream_of(lists)),
        "build_transposed_block_lists")
    max_q = int(q_counts.max()) if q_counts.numel() else 0
    return BlockLists(k_lists[..., :max_q].contiguous(), q_counts, max_q)


# ----------------------------------------------------------------------------------------
# attention
# ----------------------------------------------------------------------------------------

_SIMT_WARNED = set()


def _warn_if_simt(dtype, head_dim, route_block):
    """The tensor-core (tcgen05) kernels take bf16/fp16 with head_dim 64 or 128 and a route
    block that is a multiple of 128; other half-precision shapes run the CUDA-core kernels,
    several times slower.  Say so once per shape instead of falling off that cliff quietly."""
    if dtype not in (torch.float16, torch.bfloat16):
        return
    if head_dim in (64, 128) and route_block % 128 == 0:
        return
    key = (dtype, head_dim, route_block)
    if key in _SIMT_WARNED:
        return
    _SIMT_WARNED.add(key)
    warnings.warn(
        f"block_list_attention: {str(dtype).replace('torch.', '')} with head_dim={head_dim} and "
        f"route_block={route_block} runs on the CUDA-core kernels; the tensor-core path needs "
        f"head_dim 64 or 128 and route_block a multiple of 128", RuntimeWarning, stacklevel=3)


def _fwd(q, k, v, lists, counts, route_block, is_causal, scale, store_lse, soft_block_bias):
    Z, H, N, D = q.shape
    _warn_if_simt(q.dtype, D, route_block)
    out = torch.empty_like(q)
    lse = torch.empty((Z, H, N), dtype=torch.float32, device=q.device) if store_lse else None
    sb = soft_block_bias
    ws_bytes = int(nat.lib().sa_block_list_attention_fwd_workspace_bytes(Z, H, N, D, route_block))
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=q.device)
    nat.check(nat.lib().sa_block_list_attention_fwd(
        nat.float_code(q.dtype), Z, H, k.shape[1], N, D, route_block,
        q.data_ptr(), nat.strides(q), k.data_ptr(), nat.strides(k), v.data_ptr(), nat.strides(v),
        out.data_ptr(), nat.strides(out), nat.ptr(lse),
        lists.data_ptr(), lists.shape[-1], counts.data_ptr(),
        nat.ptr(sb), nat.float_code(sb.dtype) if sb is not None else 0,
        nat.strides(sb) if sb is not None else None,
        int(bool(is_causal)), float(scale), ws.data_ptr(), ws.numel(), nat.stream_of(q)),
        "block_list_attention forward")
    return out, lse


def _bwd(do, q, k, v, out, lse, lists, counts, route_block, is_causal, scale, soft_block_bias,
         deterministic=False):
    Z, H, N, D = q.shape
    do = do.contiguous() if do.stride(-1) != 1 else do
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    sb = soft_block_bias
    nb = -(-N // route_block)
    d_sb = (torch.empty((Z, H, nb, lists.shape[-1]), dtype=torch.float32, device=q.device)
            if sb is not None else None)
    ws_bytes = int(nat.lib().sa_block_list_attention_bwd_workspace_bytes(Z, H, k.shape[1], N, D,
                                                                          route_block))
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=q.device)
    # phase 0: the whole backward (the fused single-pass kernel where the shape allows);
    # deterministic: the dQ and dK/dV kernels (phases 1-3), whose sums are reproducible
    for phase in ((1, 2, 3) if deterministic else (0,)):
        nat.check(nat.lib().sa_block_list_attention_bwd_phase(
            phase, nat.float_code(q.dtype), Z, H, k.shape[1], N, D, route_block,
            q.data_ptr(), nat.strides(q), k.data_ptr(), nat.strides(k), v.data_ptr(), nat.strides(v),
            out.data_ptr(), nat.strides(out), do.data_ptr(), nat.strides(do), lse.data_ptr(),
            lists.data_ptr(), lists.shape[-1], counts.data_ptr(),
            nat.ptr(sb), nat.float_code(sb.dtype) if sb is not None else 0,
            nat.strides(sb) if sb is not None else None,
            int(bool(is_causal)), float(scale),
            dq.data_ptr(), nat.strides(dq), dk.data_ptr(), nat.strides(dk), dv.data_ptr(),
            nat.strides(dv), nat.ptr(d_sb), ws.data_ptr(), ws.numel(), nat.stream_of(q)),
            "block_list_attention backward")
    if d_sb is not None:
        d_sb = d_sb.to(sb.dtype)
    return dq, dk, dv, d_sb


class _BlockListAttentionFn(torch.autograd.Function):
    """Autograd of the block-list attention (block_list.py:883-961): the forward stores
    the LSE; the backward runs Delta, transposed lists, dQ and dK/dV on the device."""

    @staticmethod
    def forward(ctx, q, k, v, lists, counts, route_block, is_causal, scale, return_lse,
                soft_block_bias, deterministic=False):
        out, lse = _fwd(q, k, v, lists, counts, route_block, is_causal, scale, True, soft_block_bias)
        ctx.deterministic = deterministic
        saved = [q, k, v, out, lse, lists, counts]
        if soft_block_bias is not None:
            saved.append(soft_block_bias)
        ctx.save_for_backward(*saved)
        ctx.has_bias = soft_block_bias is not None
        ctx.route_block = route_block
        ctx.is_causal = is_causal
        ctx.scale = scale
        if return_lse:
            ctx.mark_non_differentiable(lse)
            return out, lse
        return out

    @staticmethod
    def backward(ctx, *grads):
        do = grads[0]
        saved = ctx.saved_tensors
        q, k, v, out, lse, lists, counts = saved[:7]
        sb = saved[7] if ctx.has_bias else None
        dq, dk, dv, d_sb = _bwd(do, q, k, v, out, lse, lists, counts, ctx.route_block,
                                ctx.is_causal, ctx.scale, sb, ctx.deterministic)
        return (dq if ctx.needs_input_grad[0] else None,
                dk if ctx.needs_input_grad[1] else None,
                dv if ctx.needs_input_grad[2] else None,
                None, None, None, None, None, None,
                d_sb if (ctx.has_bias and ctx.needs_input_grad[9]) else None, None)


def block_list_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    block_lists: BlockLists,
    *,
    route_block: int = 128,
    is_causal: bool = False,
    sm_scale: Optional[float] = None,
    block_m: Optional[int] = None,
    block_n: Optional[int] = None,
    num_warps: int = 4,
    num_stages: int = 3,
    return_lse: bool = False,
    soft_block_bias: Optional[torch.Tensor] = None,
    deterministic: bool = False,
):
    """Block-sparse attention over precomputed block lists, with sparse autograd.

    Args as block_list.py:968-1006: q (Z, H, N, D); k, v (Z, H, N, D) or, GQA, (Z, Hkv, N, D)
    with H % Hkv == 0; fp16/bf16 (tcgen05) or fp32 (exact CUDA-core path); D a power of two
    >= 16; lists from ``build_block_lists`` with NB = ceil(N / route_block); ``return_lse``
    adds the (Z, H, N) fp32 natural-log LSE (-inf for rows with no visible key);
    ``soft_block_bias`` (Z, H, NB, max_count) is an additive logit bias per (row block, slot)
    with an exact gradient (for STE router training).

    The backward of bf16/fp16 with head_dim 128 and route_block a multiple of 128 runs one
    fused kernel (dK, dV and dQ in one pass; dQ summed in fp32 by atomics, so its last bits
    can differ from run to run).  ``deterministic=True`` (an addition to the reference's
    signature) runs the separate dQ and dK/dV kernels instead, whose sums are reproducible.
    """
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4 or k.shape != v.shape or \
            q.shape[0] != k.shape[0] or q.shape[2:] != k.shape[2:] or \
            k.shape[1] == 0 or q.shape[1] % k.shape[1] != 0:
        raise ValueError(f"q, k, v must share shape (Z, H, N, D); got {q.shape}, {k.shape}, {v.shape}")
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError("q, k, v must share dtype")
    Z, H, N, D = q.shape
    if D < 16 or D & (D - 1):
        raise ValueError(f"head_dim must be a power of two >= 16, got {D}")
    if route_block < 16 or route_block & (route_block - 1):
        raise ValueError(f"route_block must be a power of two >= 16, got {route_block}")
    for bm in (block_m, block_n):
        if bm is not None and route_block % bm:
            raise ValueError(f"block_m ({block_m}) and block_n ({block_n}) must divide route_block ({route_block})")

    lists, counts, max_count = block_lists
    nb = -(-N // route_block)
    if tuple(counts.shape) != (Z, H, nb) or tuple(lists.shape[:3]) != (Z, H, nb):
        raise ValueError(f"block_lists built for {tuple(counts.shape)}, expected {(Z, H, nb)} "
                         f"(N={N}, route_block={route_block})")
    if lists.shape[-1] != max_count:
        raise ValueError("lists.shape[-1] must equal max_count")
    if soft_block_bias is not None and tuple(soft_block_bias.shape) != (Z, H, nb, max_count):
        raise ValueError(
            f"soft_block_bias must have shape {(Z, H, nb, max_count)}, got {tuple(soft_block_bias.shape)}")
    nat.require_cuda("block_list_attention", q, k, v, lists, counts, soft_block_bias)
    nat.float_code(q.dtype)

    lists = lists.to(torch.int32).contiguous()
    counts = counts.to(torch.int32).contiguous()
    scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(D)
    if q.stride(-1) != 1:
        q = q.contiguous()
    if k.stride(-1) != 1:
        k = k.contiguous()
    if v.stride(-1) != 1:
        v = v.contiguous()

    needs_grad = torch.is_grad_enabled() and (
        q.requires_grad or k.requires_grad or v.requires_grad
        or (soft_block_bias is not None and soft_block_bias.requires_grad))
    if needs_grad:
        return _BlockListAttentionFn.apply(q, k, v, lists, counts, int(route_block),
                                           bool(is_causal), float(scale), bool(return_lse),
                                           soft_block_bias, bool(deterministic))
    out, lse = _fwd(q, k, v, lists, counts, int(route_block), bool(is_causal), float(scale),
                    bool(return_lse), soft_block_bias)
    return (out, lse) if return_lse else out


def routed_block_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    router_indices: torch.Tensor,
    req_depth: DepthLike,
    *,
    route_block: int = 128,
    is_causal: bool = False,
    sink_block: bool = False,
    local_blocks: int = 0,
    sm_scale: Optional[float] = None,
    soft_block_bias: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Convenience wrapper: build the block lists, then run the kernel (block_list.py:1064-1083)."""
    bl = build_block_lists(router_indices, req_depth, is_causal=is_causal,
                           sink_block=sink_block, local_blocks=local_blocks)
    return block_list_attention(q, k, v, bl, route_block=route_block, is_causal=is_causal,
                                sm_scale=sm_scale, soft_block_bias=soft_block_bias)

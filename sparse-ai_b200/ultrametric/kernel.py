"""Quickstart and legacy entry points of sparse-ai's ``src/ultrametric/kernel.py``, re-based
on the sm_100a block-list kernels.

* ``block_sparse_attention`` (kernel.py:520-580 there): pad/trim routes, build exact lists,
  run the block-list forward, return ``(out, lse)``.  No CPU fallback: CUDA tensors only.
* ``ultrametric_attention_triton`` (kernel.py:420-517): the legacy padded-list kernel's
  signature; here a shim onto the block-list forward with route block min(128, N).
* ``CurriculumSparseAttention`` (kernel.py:583-671): the legacy autograd wrapper, as a shim
  onto the block-list autograd.
* ``routing_to_block_indices`` (kernel.py:152-191): per-token one-hot routes -> per-block
  routes (first token of each block), plain torch glue on the caller's device.
"""

from __future__ import annotations

import math

import torch

from .block_list import block_list_attention, build_block_lists

HAS_TRITON = True  # import compatibility with the reference; the backend is CUDA


def routing_to_block_indices(assignments: torch.Tensor, seq_len: int, block_size: int = 128) -> torch.Tensor:
    """(B, H, S, L, p) one-hot routing -> (B, H, ceil(S/block), L) int32, each block
    represented by its first token's argmax branch (kernel.py:152-191 of the reference)."""
    B, H, S, L, P = assignments.shape
    num_blocks = math.ceil(seq_len / block_size)
    branch_ids = assignments.argmax(dim=-1)
    if S < num_blocks * block_size:
        pad_len = num_blocks * block_size - S
        branch_ids = torch.nn.functional.pad(branch_ids, (0, 0, 0, pad_len), value=0)
    branch_ids = branch_ids.view(B, H, num_blocks, block_size, L)
    return branch_ids[:, :, :, 0, :].to(torch.int32)


def _pad_routes(router_indices: torch.Tensor, nb: int) -> torch.Tensor:
    Z, H, have, TD = router_indices.shape
    if have < nb:
        pad = torch.zeros((Z, H, nb - have, TD), dtype=router_indices.dtype, device=router_indices.device)
        return torch.cat([router_indices, pad], dim=2)
    if have > nb:
        return router_indices[:, :, :nb]
    return router_indices


def block_sparse_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    router_indices: torch.Tensor,
    req_depth: int = 2,
    p: int = 2,
    is_causal: bool = False,
    route_block: int = 128,
):
    """Quickstart API: routed block-sparse attention forward, returns ``(out, lse)``.

    Routes shorter than ceil(N / route_block) blocks are padded with branch 0, longer ones
    trimmed (kernel.py:557-566).  Lists are built exactly (host-validated ids), so this costs
    a couple of host reads; in a hot loop build lists once with ``arity=`` and call
    ``block_list_attention``.  ``p`` is informational, as in the reference."""
    Z, H, N, D = q.shape
    nb = -(-N // route_block)
    router_indices = _pad_routes(router_indices.to(torch.int64), nb)
    bl = build_block_lists(router_indices, req_depth, is_causal=is_causal)
    return block_list_attention(q, k, v, bl, route_block=route_block, is_causal=is_causal,
                                return_lse=True)


def ultrametric_attention_triton(q, k, v, router_indices, req_depth: int = 2, p: int = 2,
                                 is_causal: bool = False):
    """Legacy signature (kernel.py:420-517): routes per ``min(128, N)``-token block, returns
    ``(out, L)``.  Runs the block-list kernels."""
    N = q.shape[2]
    rb = 128 if N >= 128 else max(16, 1 << (max(N, 1) - 1).bit_length())
    TD = router_indices.shape[-1]
    if not 0 <= req_depth <= TD:
        raise AssertionError(f"req_depth ({req_depth}) must be in [0, {TD}]")
    nb = -(-N // rb)
    r = _pad_routes(router_indices.to(torch.int32), nb)
    bl = build_block_lists(r, req_depth, is_causal=is_causal)
    return block_list_attention(q, k, v, bl, route_block=rb, is_causal=is_causal, return_lse=True)


class CurriculumSparseAttention(torch.autograd.Function):
    """Legacy autograd entry (kernel.py:583-671): ``use_sparse_backend=True`` only."""

    @staticmethod
    def forward(ctx, q, k, v, router_indices, req_depth=2, p=2, use_sparse_backend=False):
        if not use_sparse_backend:
            raise NotImplementedError("CurriculumSparseAttention should only be called for use_sparse_backend=True")
        with torch.enable_grad():
            qd, kd, vd = (t.detach().requires_grad_(True) for t in (q, k, v))
            N = q.shape[2]
            rb = 128 if N >= 128 else max(16, 1 << (max(N, 1) - 1).bit_length())
            r = _pad_routes(router_indices.to(torch.int32), -(-N // rb))
            bl = build_block_lists(r, req_depth)
            out = block_list_attention(qd, kd, vd, bl, route_block=rb)
        ctx.save_for_backward(qd, kd, vd, out)
        return out.detach()

    @staticmethod
    def backward(ctx, do):
        qd, kd, vd, out = ctx.saved_tensors
        dq, dk, dv = torch.autograd.grad(out, (qd, kd, vd), do)
        return dq, dk, dv, None, None, None, None

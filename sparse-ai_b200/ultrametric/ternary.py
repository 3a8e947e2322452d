"""Ternary (2-bit) K/V for sparse-ai's LLaMA-surgery prefill, on the B200 kernels.

The reference quantises K/V rows to {-1, 0, +1} x a per-row scale (``TernaryQuantize``,
``src/llama_surgery/surgery.py:15-32``), packs 16 values per int32 (``pack_ternary`` /
``unpack_ternary``, :35-75) and attends with a Triton kernel that unpacks K/V tiles on the fly
(``ternary_ultrametric_attention_triton``, ``src/llama_surgery/kernel.py:348-418``, kernel
:147-249).  Here quantise + pack and unpack + dequantise are CUDA kernels
(``sa_ternary_quantize_pack``, ``sa_ternary_dequantize``), and the attention runs the
block-list forward over the dequantised fp16 K/V with lists built from the same rule (routes
matching on ``req_depth`` levels, sink block, local window, causal).

``shift_size`` (the Swin shift of the reference kernel's region mask) must be 0 here.
"""

from __future__ import annotations

import math

import torch

from . import _native as nat
from .block_list import block_list_attention, build_block_lists


def quantize_pack_ternary(x: torch.Tensor):
    """Rows of ``x`` (..., D), D a multiple of 16 -> (packed (..., D // 16) int32, scale (...)
    fp32): scale = mean |x| over the row, value +1 above scale / 2, -1 below -scale / 2, else 0
    (``TernaryQuantize`` then ``pack_ternary`` of the reference)."""
    nat.require_cuda("quantize_pack_ternary", x)
    D = x.shape[-1]
    if D % 16:
        raise AssertionError("Last dimension must be multiple of 16 for packing")
    xr = x.reshape(-1, D)
    if xr.stride(-1) != 1:
        xr = xr.contiguous()
    packed = torch.empty(xr.shape[0], D // 16, dtype=torch.int32, device=x.device)
    scale = torch.empty(xr.shape[0], dtype=torch.float32, device=x.device)
    nat.check(nat.lib().sa_ternary_quantize_pack(nat.float_code(xr.dtype), xr.shape[0], D, xr.data_ptr(),
                                                 xr.stride(0), packed.data_ptr(), scale.data_ptr(),
                                                 nat.stream_of(x)), "quantize_pack_ternary")
    return packed.view(*x.shape[:-1], D // 16), scale.view(x.shape[:-1])


def dequantize_ternary(packed: torch.Tensor, scale: torch.Tensor, dtype=torch.float16) -> torch.Tensor:
    """packed (..., D // 16) int32, scale (...) -> (..., D) values code x scale in ``dtype``."""
    nat.require_cuda("dequantize_ternary", packed, scale)
    W = packed.shape[-1]
    pr = packed.reshape(-1, W).to(torch.int32).contiguous()
    sc = scale.reshape(-1).to(torch.float32).contiguous()
    out = torch.empty(pr.shape[0], W * 16, dtype=dtype, device=packed.device)
    nat.check(nat.lib().sa_ternary_dequantize(nat.float_code(dtype), pr.shape[0], W * 16, pr.data_ptr(),
                                              sc.data_ptr(), out.data_ptr(), out.stride(0),
                                              nat.stream_of(packed)), "dequantize_ternary")
    return out.view(*packed.shape[:-1], W * 16)


def pack_ternary(x_ternary: torch.Tensor) -> torch.Tensor:
    """{-1, 0, +1} values (..., D) -> packed (..., D // 16) int32 (surgery.py:35-55)."""
    return quantize_pack_ternary(x_ternary)[0]


def unpack_ternary(packed: torch.Tensor, original_shape: tuple) -> torch.Tensor:
    """packed int32 -> fp32 {-1, 0, +1} of ``original_shape`` (surgery.py:57-75)."""
    ones = torch.ones(packed.shape[:-1], dtype=torch.float32, device=packed.device)
    return dequantize_ternary(packed, ones, torch.float32).view(original_shape)


class TernaryQuantize(torch.autograd.Function):
    """Forward: the row-wise ternary value x scale (surgery.py:15-28); backward: straight
    through (the identity, :30-32)."""

    @staticmethod
    def forward(ctx, x):
        packed, scale = quantize_pack_ternary(x.float())
        return dequantize_ternary(packed, scale, torch.float32)

    @staticmethod
    def backward(ctx, grad_output):
        return grad_output


def ternary_ultrametric_attention_triton(q, k_packed, v_packed, k_scale, v_scale, router_indices,
                                         local_window: int = 128, req_depth: int = 2,
                                         shift_size: int = 0, p: int = 2):
    """The reference's ternary prefill (kernel.py:348-418): q (Z, H, N, D) fp16, k_packed /
    v_packed (Z, H, N, D // 16) int32, k_scale / v_scale (Z, H, N), router_indices
    (Z, H, num_blocks, TD) per block of min(128, N) tokens.  Query block m attends key block
    n <= m when their routes agree on the first ``req_depth`` levels, n == 0, or
    m - n <= ceil(local_window / block); causal within blocks.  Returns fp16 (Z, H, N, D)."""
    if q.dtype != torch.float16:
        raise AssertionError(f"Triton kernel requires float16 Q, got {q.dtype}")
    if k_packed.dtype != torch.int32:
        raise AssertionError(f"Triton kernel requires int32 packed K, got {k_packed.dtype}")
    if shift_size:
        raise NotImplementedError("ternary attention: shift_size (Swin region mask) is not supported")
    Z, H, N, D = q.shape
    block = min(128, N)
    rb = 1 << max(4, (block - 1).bit_length())  # a power of two >= block: same block grid
    nb = -(-N // block)
    r = router_indices.to(torch.int32)
    if r.shape[2] < nb:
        pad = torch.zeros((Z, H, nb - r.shape[2], r.shape[3]), dtype=torch.int32, device=r.device)
        r = torch.cat([r, pad], dim=2)
    r = r[:, :, :nb].contiguous()
    lwb = math.ceil(local_window / block)
    bl = build_block_lists(r, req_depth, is_causal=True, sink_block=True, local_blocks=lwb, arity=p)
    k = dequantize_ternary(k_packed, k_scale, torch.float16)
    v = dequantize_ternary(v_packed, v_scale, torch.float16)
    if rb != block:  # N < 16: one block either way
        rb = block if block >= 16 else rb
    return block_list_attention(q, k, v, bl, route_block=rb if nb > 1 else max(rb, 16), is_causal=True)

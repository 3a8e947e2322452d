"""Masked dense attention oracle (torch on CPU; TEST INFRASTRUCTURE ONLY).

Restates the reference's ground truth for the prefill path of sparse-ai:

* ``token_mask``           -- ``token_mask_from_blocks`` (src/ultrametric/block_list.py:361-368)
* ``masked_attention``     -- ``masked_reference_attention`` (block_list.py:371-378) plus the
  log-sum-exp and the empty-row convention of the CPU quickstart path
  (src/ultrametric/kernel.py:574-580: softmax NaNs -> 0, lse = -inf) and of the kernel
  (block_list.py:463-470: zero output, -inf lse).
* ``masked_attention_chunked`` -- the query-chunked form used by the reference benchmark
  (benchmarks/benchmark_block_list.py:106-123) so N=8192 fits in host memory; GQA K/V are
  shared by ``H // Hkv`` query heads (the reference repeat-interleaves them).
* ``masked_attention_grads`` -- dQ, dK, dV and the soft-block-bias gradient by autograd of
  the masked reference (tests/test_block_list.py:287-292, 330-348 of the reference).
* ``masked_attention_grads_chunked`` -- the same gradients written out explicitly and
  query-chunked per GQA group, so the full N=8192 backward fits in host memory.
"""

from __future__ import annotations

import math
from typing import Optional

import torch


def token_mask(block_mask: torch.Tensor, route_block: int, seq_len: int,
               is_causal: bool = False) -> torch.Tensor:
    """Expand a (..., NB, NB) block mask to a (..., N, N) token mask (block_list.py:361-368)."""
    m = block_mask.repeat_interleave(route_block, dim=-2).repeat_interleave(route_block, dim=-1)
    m = m[..., :seq_len, :seq_len]
    if is_causal:
        m = m & torch.ones(seq_len, seq_len, dtype=torch.bool).tril()
    return m


def _expand_kv(x: torch.Tensor, num_heads: int) -> torch.Tensor:
    hkv = x.shape[1]
    if hkv == num_heads:
        return x
    return x.repeat_interleave(num_heads // hkv, dim=1)


def token_bias(bias: torch.Tensor, lists: torch.Tensor, counts: torch.Tensor,
               route_block: int, seq_len: int) -> torch.Tensor:
    """Scatter a (Z, H, NB, max_count) per-slot block bias to a (Z, H, N, N) token bias
    (the construction of tests/test_block_list.py:330-340 of the reference)."""
    Z, H, NB, _ = bias.shape
    full = torch.zeros(Z, H, NB, NB, dtype=bias.dtype)
    for z in range(Z):
        for h in range(H):
            for qb in range(NB):
                for t in range(int(counts[z, h, qb])):
                    full[z, h, qb, int(lists[z, h, qb, t])] = bias[z, h, qb, t]
    tb = full.repeat_interleave(route_block, dim=-2).repeat_interleave(route_block, dim=-1)
    return tb[..., :seq_len, :seq_len]


def masked_attention(q, k, v, mask, sm_scale: Optional[float] = None, bias=None,
                     compute_dtype=torch.float64):
    """Return (out, lse) of softmax(q k^T * scale + bias, masked) v in ``compute_dtype``.

    Rows with no visible key give out = 0 and lse = -inf."""
    D = q.shape[-1]
    scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(D)
    H = q.shape[1]
    qf = q.to(compute_dtype)
    kf = _expand_kv(k, H).to(compute_dtype)
    vf = _expand_kv(v, H).to(compute_dtype)
    s = torch.matmul(qf, kf.transpose(-2, -1)) * scale
    if bias is not None:
        s = s + bias.to(compute_dtype)
    s = s.masked_fill(~mask, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.softmax(s, dim=-1).nan_to_num(0.0)
    return torch.matmul(p, vf), lse


def masked_attention_chunked(q, k, v, block_mask, route_block: int, is_causal: bool,
                             sm_scale: Optional[float] = None, chunk: int = 1024,
                             compute_dtype=torch.float32, heads=None, row_ranges=None):
    """Query-chunked masked attention over (Z, H, N, D) q and (Z, Hkv, N, D) k/v
    (benchmarks/benchmark_block_list.py:106-123).  ``heads`` restricts to a head subset,
    ``row_ranges`` (a list of [start, end) query-row ranges) to some query rows; rows
    outside them are left zero.  Returns (out, lse) in ``compute_dtype`` for the selected
    heads."""
    Z, H, N, D = q.shape
    group = H // k.shape[1]
    scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(D)
    hs = list(range(H)) if heads is None else list(heads)
    out = torch.zeros(Z, len(hs), N, D, dtype=compute_dtype)
    lse = torch.zeros(Z, len(hs), N, dtype=compute_dtype)
    col_blk = torch.arange(N) // route_block
    cols = torch.arange(N)
    for z in range(Z):
        for hi, h in enumerate(hs):
            kf = k[z, h // group].to(compute_dtype)
            vf = v[z, h // group].to(compute_dtype)
            spans = row_ranges if row_ranges is not None else [(0, N)]
            starts = [(s0, min(e, s0 + chunk)) for b, e in spans for s0 in range(b, e, chunk)]
            for s0, e0 in starts:
                rows = torch.arange(s0, e0)
                sc = torch.matmul(q[z, h, s0:e0].to(compute_dtype), kf.T) * scale
                m = block_mask[z, h][rows // route_block][:, col_blk]
                if is_causal:
                    m = m & (rows[:, None] >= cols[None, :])
                sc = sc.masked_fill(~m, float("-inf"))
                lse[z, hi, s0:e0] = torch.logsumexp(sc, dim=-1)
                out[z, hi, s0:e0] = torch.matmul(torch.softmax(sc, dim=-1).nan_to_num(0.0), vf)
    return out, lse


def masked_attention_grads(q, k, v, mask, dout, sm_scale: Optional[float] = None,
                           block_bias=None, lists=None, counts=None, route_block=None,
                           compute_dtype=torch.float64):
    """Autograd of the masked reference.  Returns dict with out, dq, dk, dv and, when
    ``block_bias`` (Z, H, NB, max_count) is given, d_bias (the STE router gradient).
    GQA gradients are summed over each KV head's query-head group."""
    H = q.shape[1]
    N = q.shape[2]
    qf = q.detach().to(compute_dtype).requires_grad_(True)
    kf = k.detach().to(compute_dtype).requires_grad_(True)
    vf = v.detach().to(compute_dtype).requires_grad_(True)
    bias = None
    bf = None
    if block_bias is not None:
        bf = block_bias.detach().to(compute_dtype).requires_grad_(True)
        bias = _token_bias_differentiable(bf, lists, counts, route_block, N)
    out, _ = masked_attention(qf, kf, vf, mask, sm_scale=sm_scale, bias=bias,
                              compute_dtype=compute_dtype)
    out.backward(dout.to(compute_dtype))
    res = {"out": out.detach(), "dq": qf.grad, "dk": kf.grad, "dv": vf.grad}
    if bf is not None:
        res["d_bias"] = bf.grad
    return res


def _token_bias_differentiable(bf, lists, counts, route_block, seq_len):
    Z, H, NB, MC = bf.shape
    idx = torch.full((Z, H, NB, NB), MC, dtype=torch.long)
    for z in range(Z):
        for h in range(H):
            for qb in range(NB):
                for t in range(int(counts[z, h, qb])):
                    idx[z, h, qb, int(lists[z, h, qb, t])] = t
    padded = torch.cat([bf, torch.zeros(Z, H, NB, 1, dtype=bf.dtype)], dim=-1)
    full = torch.gather(padded, -1, idx)
    tb = full.repeat_interleave(route_block, dim=-2).repeat_interleave(route_block, dim=-1)
    return tb[..., :seq_len, :seq_len]


def block_list_backward_lowp(q, k, v, out, dout, lse, mask, sm_scale=None, io_dtype=torch.bfloat16):
    """Backward of the masked attention with the reference kernels' rounding points
    (src/ultrametric/block_list.py:565-580 dQ and :652-680 dK/dV): P and the scaled dS are
    rounded to the input dtype before their products, Delta uses the input-dtype output O
    (block_list.py:785); everything else in fp64.  GQA: dK/dV summed over each KV group."""
    H, D = q.shape[1], q.shape[-1]
    scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(D)
    f = torch.float64
    qf, kf, vf = q.to(f), _expand_kv(k, H).to(f), _expand_kv(v, H).to(f)
    dof = dout.to(f)
    s = torch.matmul(qf, kf.transpose(-2, -1)) * scale
    lse_safe = torch.where(torch.isinf(lse), torch.zeros_like(lse), lse).to(f)
    p = torch.where(mask, torch.exp(s - lse_safe[..., None]), torch.zeros_like(s))
    p_lp = p.to(io_dtype).to(f)
    dp = torch.matmul(dof, vf.transpose(-2, -1))
    delta = (dof * out.to(io_dtype).to(f)).sum(-1, keepdim=True)
    ds = torch.where(mask, p * (dp - delta), torch.zeros_like(p))
    ds_lp = (ds * scale).to(io_dtype).to(f)
    dq = torch.matmul(ds_lp, kf)
    dk = torch.matmul(ds_lp.transpose(-2, -1), qf)
    dv = torch.matmul(p_lp.transpose(-2, -1), dof)
    g = H // k.shape[1]
    if g > 1:
        Z, _, N, _ = dk.shape
        dk = dk.view(Z, k.shape[1], g, N, D).sum(2)
        dv = dv.view(Z, k.shape[1], g, N, D).sum(2)
    return {"dq": dq, "dk": dk, "dv": dv}


def masked_attention_grads_chunked(q, k, v, block_mask, route_block: int, is_causal: bool,
                                   dout, kv_heads, sm_scale: Optional[float] = None,
                                   chunk: int = 1024, io_dtype=None,
                                   compute_dtype=torch.float64):
    """Backward of the masked attention for whole GQA groups, query-chunked so N=8192 fits
    in host memory (the chunking of benchmarks/benchmark_block_list.py:106-123, applied to
    the gradients of block_list.py:494-681).

    For each KV head in ``kv_heads`` and its ``H // Hkv`` query heads: a forward pass per
    query chunk gives out and lse, then a second pass gives
        P = exp(S - lse), dP = dO V^T, Delta = rowsum(dO * O), dS = P * (dP - Delta),
        dQ = scale * dS K,  dK = scale * sum_heads dS^T Q,  dV = sum_heads P^T dO,
    and the unscaled per-block sums of dS (the soft-block-bias gradient before the slot
    gather, block_list.py:571-584).  With ``io_dtype`` set, P and scale*dS are rounded to it
    before their products and Delta uses O rounded to it, as the reference kernels do
    (block_list.py:565-580, 652-680, 785).  Returns a dict of tensors over the selected heads:
    out/lse/dq (Z, G*len(kv_heads), N, .), dk/dv (Z, len(kv_heads), N, D), dbias_blocks
    (Z, G*len(kv_heads), NB, NB), and ``heads``, the query heads in order."""
    Z, H, N, D = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    NB = -(-N // route_block)
    scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(D)
    f = compute_dtype
    heads = [g * G + j for g in kv_heads for j in range(G)]
    nh, nk = len(heads), len(kv_heads)
    res = {"heads": heads,
           "out": torch.zeros(Z, nh, N, D, dtype=f), "lse": torch.zeros(Z, nh, N, dtype=f),
           "dq": torch.zeros(Z, nh, N, D, dtype=f), "dk": torch.zeros(Z, nk, N, D, dtype=f),
           "dv": torch.zeros(Z, nk, N, D, dtype=f),
           "dbias_blocks": torch.zeros(Z, nh, NB, NB, dtype=f)}
    col_blk = torch.arange(N) // route_block
    cols = torch.arange(N)

    def rnd(x):
        return x.to(io_dtype).to(f) if io_dtype is not None else x

    for z in range(Z):
        for gi, g in enumerate(kv_heads):
            kf = k[z, g].to(f)
            vf = v[z, g].to(f)
            for j in range(G):
                hi = gi * G + j
                h = heads[hi]
                for s0 in range(0, N, chunk):
                    e0 = min(N, s0 + chunk)
                    rows = torch.arange(s0, e0)
                    qc = q[z, h, s0:e0].to(f)
                    doc = dout[z, h, s0:e0].to(f)
                    m = block_mask[z, h][rows // route_block][:, col_blk]
                    if is_causal:
                        m = m & (rows[:, None] >= cols[None, :])
                    s = (qc @ kf.T) * scale
                    s = s.masked_fill(~m, float("-inf"))
                    lse = torch.logsumexp(s, dim=-1)
                    lse_safe = torch.where(torch.isinf(lse), torch.zeros_like(lse), lse)
                    p = torch.where(m, torch.exp(s - lse_safe[:, None]), torch.zeros_like(s))
                    o = p @ vf
                    res["out"][z, hi, s0:e0] = o
                    res["lse"][z, hi, s0:e0] = lse
                    dp = doc @ vf.T
                    delta = (doc * rnd(o)).sum(-1, keepdim=True)
                    ds = torch.where(m, p * (dp - delta), torch.zeros_like(p))
                    ds_s = rnd(ds * scale)
                    res["dq"][z, hi, s0:e0] = ds_s @ kf
                    res["dk"][z, gi] += ds_s.T @ qc
                    res["dv"][z, gi] += rnd(p).T @ doc
                    # per-block sums of the unscaled dS: rows -> query blocks, cols -> key blocks
                    qb = rows // route_block
                    blk = torch.zeros(NB, N, dtype=f).index_add_(0, qb, ds)
                    res["dbias_blocks"][z, hi] += torch.zeros(NB, NB, dtype=f).index_add_(
                        1, col_blk, blk)
    return res

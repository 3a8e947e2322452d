"""CPU stand-ins for the two device operations of the sequence-sharded ring (TEST
INFRASTRUCTURE ONLY): attention of a query chunk to one K/V chunk over re-based block
lists, returning the normalised output and natural-log LSE like the forward kernel
(src/ultrametric/block_list.py:455-470 conventions), and the log-sum-exp merge of such
partials.  With them the ring schedule (``ultrametric.ring``) runs on gloo CPU ranks.
"""

from __future__ import annotations

import torch

from .attention_oracle import masked_attention, token_mask


def lists_to_mask(lists: torch.Tensor, counts: torch.Tensor, nb_k: int) -> torch.Tensor:
    """(Z, H, NBq, mc) lists + counts -> (Z, H, NBq, nb_k) boolean block mask."""
    Z, H, NBq, mc = lists.shape
    m = torch.zeros(Z, H, NBq, nb_k, dtype=torch.bool)
    for z in range(Z):
        for h in range(H):
            for qb in range(NBq):
                for t in range(int(counts[z, h, qb])):
                    m[z, h, qb, int(lists[z, h, qb, t])] = True
    return m


def chunk_attention(q, k, v, lists, counts, route_block, is_causal, scale):
    """q (Z, H, Nq, D) against one K/V chunk (Z, Hkv, Nk, D) over chunk-local lists; fp64
    math, outputs cast to q's dtype (out) and fp32 (lse)."""
    Z, H, Nq, D = q.shape
    Nk = k.shape[2]
    nb_k = -(-Nk // route_block)
    bm = lists_to_mask(lists.cpu(), counts.cpu(), nb_k)
    tm = bm.repeat_interleave(route_block, -2).repeat_interleave(route_block, -1)[..., :Nq, :Nk]
    if is_causal:
        tm = tm & torch.ones(Nq, Nk, dtype=torch.bool).tril()
    out, lse = masked_attention(q, k, v, tm, sm_scale=scale)
    return out.to(q.dtype), lse.to(torch.float32)


class LseMergeCPU:
    """fp32 accumulator merged by log-sum-exp weights, the interface of the CUDA merge."""

    def __init__(self, q: torch.Tensor):
        Z, H, N, D = q.shape
        self.acc = torch.zeros(Z, H, N, D, dtype=torch.float64)
        self.lse = torch.full((Z, H, N), float("-inf"), dtype=torch.float64)

    def finish(self, out):
        out.copy_(self.acc.to(out.dtype))

    def __call__(self, o, lse, first: bool, out):
        lj = lse.to(torch.float64)
        la = torch.full_like(lj, float("-inf")) if first else self.lse
        acc = torch.zeros_like(self.acc) if first else self.acc
        lnew = torch.logaddexp(la, lj)
        safe = torch.where(torch.isinf(lnew), torch.zeros_like(lnew), lnew)
        wa = torch.where(torch.isinf(la), torch.zeros_like(la), torch.exp(la - safe))
        wj = torch.where(torch.isinf(lj), torch.zeros_like(lj), torch.exp(lj - safe))
        self.acc = acc * wa[..., None] + o.to(torch.float64) * wj[..., None]
        self.lse = lnew
        if out is not None:
            out.copy_(self.acc.to(out.dtype))

"""The query-chunked oracles used at the benchmark sizes agree with the dense ones (CPU).

``masked_attention_grads_chunked`` writes the backward out by hand (per GQA group and query
chunk); here it is checked against autograd of the dense masked reference, including the
per-block dS sums that the soft-block-bias gradient gathers, and ``row_ranges`` of the
chunked forward against the full forward."""

import torch

from helpers import random_router
from oracle import attention_oracle as ao
from oracle import block_list_oracle as blo


def _case(seed=3, Z=1, H=4, Hkv=2, N=320, D=32, RB=64, depth=1, causal=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(Z, H, N, D, generator=g)
    k = torch.randn(Z, Hkv, N, D, generator=g)
    v = torch.randn(Z, Hkv, N, D, generator=g)
    do = torch.randn(Z, H, N, D, generator=g)
    NB = -(-N // RB)
    router = random_router(Z, H, NB, 4, 2, seed=seed).numpy()
    bm = torch.from_numpy(blo.block_mask(router, depth, is_causal=causal, sink_block=True))
    return q, k, v, do, bm, RB, causal


def test_chunked_grads_match_autograd():
    q, k, v, do, bm, RB, causal = _case()
    N = q.shape[2]
    lists, counts, mc = blo.build_block_lists(
        random_router(1, 4, bm.shape[2], 4, 2, seed=3).numpy(), 1, is_causal=True, sink_block=True)
    lists, counts = torch.from_numpy(lists), torch.from_numpy(counts)
    mask = ao.token_mask(bm, RB, N, causal)
    ref = ao.masked_attention_grads(q, k, v, mask, do, block_bias=torch.zeros(lists.shape),
                                    lists=lists, counts=counts, route_block=RB)
    got = ao.masked_attention_grads_chunked(q, k, v, bm, RB, causal, do, kv_heads=[0, 1], chunk=96)
    assert got["heads"] == [0, 1, 2, 3]
    for name in ("out", "dq", "dk", "dv"):
        assert (got[name] - ref[name]).abs().max() < 1e-9, name
    # d_bias[z, h, qb, t] = block sum of dS at (qb, lists[qb, t]) for t < counts[qb]
    blocks = got["dbias_blocks"]
    for h in range(4):
        for qb in range(bm.shape[2]):
            for t in range(int(counts[0, h, qb])):
                kb = int(lists[0, h, qb, t])
                assert abs(blocks[0, h, qb, kb] - ref["d_bias"][0, h, qb, t]) < 1e-9


def test_chunked_grads_low_precision_rounding_matches_lowp_oracle():
    q, k, v, do, bm, RB, causal = _case(seed=4, N=256, D=32)
    qb, kb, vb, dob = (t.bfloat16() for t in (q, k, v, do))
    N = q.shape[2]
    mask = ao.token_mask(bm, RB, N, causal)
    exact = ao.masked_attention_grads_chunked(qb, kb, vb, bm, RB, causal, dob, kv_heads=[0, 1])
    lowp = ao.block_list_backward_lowp(qb, kb, vb, exact["out"], dob, exact["lse"], mask)
    got = ao.masked_attention_grads_chunked(qb, kb, vb, bm, RB, causal, dob, kv_heads=[0, 1],
                                            io_dtype=torch.bfloat16)
    for name in ("dq", "dk", "dv"):
        assert (got[name] - lowp[name]).abs().max() < 1e-9, name


def test_chunked_forward_row_ranges():
    q, k, v, do, bm, RB, causal = _case(seed=5, N=384)
    full, full_lse = ao.masked_attention_chunked(q, k, v, bm, RB, causal, chunk=100)
    part, part_lse = ao.masked_attention_chunked(q, k, v, bm, RB, causal, chunk=100,
                                                 row_ranges=[(0, 50), (300, 384)], heads=[1, 3])
    for rs in ((0, 50), (300, 384)):
        assert torch.allclose(part[:, :, rs[0]:rs[1]], full[:, [1, 3], rs[0]:rs[1]])
        assert torch.allclose(part_lse[:, :, rs[0]:rs[1]], full_lse[:, [1, 3], rs[0]:rs[1]])

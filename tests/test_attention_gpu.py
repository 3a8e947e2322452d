"""GPU parity of the block-list attention forward/backward against the CPU oracle and the
reference's own outputs (tests/golden/forward.npz, backward.npz).

Tolerances (written here, from the north star): fp32 within 1e-5 relative (normwise) of
the fp64 oracle; bf16/fp16 outputs and gradients within 2e-2 abs + 1e-2 rel elementwise.
The fp32 golden fixtures (the reference's Triton kernels run in fp32 under its CPU
interpreter) are matched at the reference's own fp32 tolerance, 1e-4 abs.
"""

import math

import numpy as np
import pytest
import torch

from helpers import (assert_fp32_close, assert_half_close, block_mask_from_lists, lse_close,
                     random_router, randn, tree_router)
from oracle import attention_oracle as ao
from oracle import block_list_oracle as blo
from ultrametric import (BlockLists, block_list_attention, block_sparse_attention,
                         build_block_lists, build_block_lists_from_mask)

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _t(a):
    return torch.from_numpy(np.asarray(a))


def _bl_from(lists, counts):
    return BlockLists(_t(lists).to(DEV), _t(counts).to(DEV), lists.shape[-1])


def oracle_fwd(q, k, v, bl, rb, causal, bias=None, scale=None):
    N = q.shape[2]
    bm = block_mask_from_lists(bl.lists, bl.counts)
    mask = ao.token_mask(bm, rb, N, causal)
    tb = ao.token_bias(bias.cpu().float(), bl.lists.cpu(), bl.counts.cpu(), rb, N) if bias is not None else None
    return ao.masked_attention(q.cpu(), k.cpu(), v.cpu(), mask, sm_scale=scale, bias=tb)


# ---------------------------------------------------------------------------------------
# reference fixtures (fp32)
# ---------------------------------------------------------------------------------------

def test_forward_fixtures_fp32(golden):
    g = golden("forward")
    for i in range(6):
        key = f"f{i:02d}"
        N, rb, depth, causal, sink, local = (int(x) for x in g[key + "_meta"])
        q, k, v = (_t(g[f"{key}_{n}"]).float().to(DEV) for n in "qkv")
        bl = _bl_from(g[key + "_lists"], g[key + "_counts"])
        out, lse = block_list_attention(q, k, v, bl, route_block=rb, is_causal=bool(causal),
                                        return_lse=True)
        assert (out.cpu() - _t(g[key + "_out"])).abs().max() < 1e-4, key
        lse_close(lse, _t(g[key + "_lse"]), 1e-4)
        ref, ref_lse = oracle_fwd(q, k, v, bl, rb, bool(causal))
        assert_fp32_close(out, ref, key)
        out2 = block_list_attention(q, k, v, bl, route_block=rb, is_causal=bool(causal))
        assert torch.equal(out, out2), "storing the LSE changed the output"


def test_forward_fixture_bias_and_empty_row(golden):
    g = golden("forward")
    q, k, v = (_t(g[f"fb_{n}"]).float().to(DEV) for n in "qkv")
    bias = _t(g["fb_bias"]).float().to(DEV)
    bl = _bl_from(g["fb_lists"], g["fb_counts"])
    out, lse = block_list_attention(q, k, v, bl, route_block=32, is_causal=True, return_lse=True,
                                    soft_block_bias=bias)
    assert (out.cpu() - _t(g["fb_out"])).abs().max() < 1e-4
    lse_close(lse, _t(g["fb_lse"]), 1e-4)
    assert (out[0, 1, 64:96] == 0).all() and torch.isinf(lse[0, 1, 64:96]).all()


def test_quickstart_fixture(golden):
    g = golden("forward")
    q, k, v = (_t(g[f"qs_{n}"]).float().to(DEV) for n in "qkv")
    router = _t(g["qs_router"]).to(DEV)
    for causal in (0, 1):
        out, L = block_sparse_attention(q, k, v, router, req_depth=2, is_causal=bool(causal))
        assert out.shape == q.shape and L.shape == q.shape[:3]
        assert (out.cpu() - _t(g[f"qs{causal}_out"])).abs().max() < 1e-4
        lse_close(L, _t(g[f"qs{causal}_lse"]), 1e-4)


def test_backward_fixtures_fp32(golden):
    g = golden("backward")
    for i in range(3):
        key = f"g{i:02d}"
        N, rb, depth, causal, sink, local = (int(x) for x in g[key + "_meta"])
        q, k, v, do = (_t(g[f"{key}_{n}"]).float().to(DEV) for n in ("q", "k", "v", "do"))
        bl = _bl_from(g[key + "_lists"], g[key + "_counts"])
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        out = block_list_attention(qq, kk, vv, bl, route_block=rb, is_causal=bool(causal))
        out.backward(do)
        for name, t in (("dq", qq), ("dk", kk), ("dv", vv)):
            assert (t.grad.cpu() - _t(g[f"{key}_{name}"])).abs().max() < 1e-4, (key, name)


def test_soft_bias_gradient_fixtures(golden):
    g = golden("backward")
    for causal in (0, 1):
        key = f"s{causal}"
        q, k, v, do = (_t(g[f"{key}_{n}"]).float().to(DEV) for n in ("q", "k", "v", "do"))
        bl = _bl_from(g[key + "_lists"], g[key + "_counts"])
        raw = torch.zeros(bl.lists.shape, device=DEV, requires_grad=True)
        ste = raw - raw.detach()
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        out = block_list_attention(qq, kk, vv, bl, route_block=32, is_causal=bool(causal),
                                   soft_block_bias=ste)
        out.backward(do)
        assert (raw.grad.cpu() - _t(g[key + "_dbias"])).abs().max() < 1e-4
        for name, t in (("dq", qq), ("dk", kk), ("dv", vv)):
            assert (t.grad.cpu() - _t(g[f"{key}_{name}"])).abs().max() < 1e-4, (key, name)


# ---------------------------------------------------------------------------------------
# BASELINE config C1 (fp32 correctness config, 1e-5 relative)
# ---------------------------------------------------------------------------------------

def c1_inputs(seed=0):
    B, H, N, D, RB = 1, 4, 1024, 64, 64
    gen = torch.Generator().manual_seed(seed)
    q, k, v = (randn((B, H, N, D), gen) for _ in range(3))
    NB = N // RB
    m = torch.zeros(B, H, NB, NB, dtype=torch.bool)
    for h in range(H):
        for i in range(NB):
            for j in range(i + 1):
                if j == i or j == 0:
                    m[0, h, i, j] = True
                else:
                    m[0, h, i, j] = bool(torch.rand(1, generator=gen).item() < 0.25)
    return q, k, v, m, RB


def test_c1_fp32_forward_1e5_relative():
    q, k, v, m, RB = c1_inputs()
    bl = build_block_lists_from_mask(m.to(DEV))
    out, lse = block_list_attention(q.to(DEV), k.to(DEV), v.to(DEV), bl, route_block=RB,
                                    is_causal=True, return_lse=True)
    ref, ref_lse = ao.masked_attention(q, k, v, ao.token_mask(m, RB, q.shape[2], True))
    assert_fp32_close(out, ref, "C1")
    lse_close(lse, ref_lse, 1e-5)


# ---------------------------------------------------------------------------------------
# tcgen05 shapes: bf16 / fp16, head_dim 64/128, route_block 128/256, GQA, tails, bias
# ---------------------------------------------------------------------------------------

TC_CASES = [
    # (Z, H, Hkv, N, D, RB, depth, causal, sink, local, dtype)
    (1, 2, 2, 128, 128, 128, 0, False, False, 0, torch.bfloat16),
    (1, 4, 2, 512, 128, 128, 1, True, True, 0, torch.bfloat16),
    (2, 4, 1, 1000, 64, 128, 2, True, False, 1, torch.float16),
    (1, 4, 4, 700, 128, 256, 1, False, True, 0, torch.bfloat16),
    (1, 8, 2, 2048, 128, 128, [1, 2, 3, 4, 5, 6, 7, 8], True, True, 0, torch.bfloat16),
    (1, 2, 2, 300, 64, 128, 1, False, False, 0, torch.bfloat16),
]


@pytest.mark.parametrize("Z,H,Hkv,N,D,RB,depth,causal,sink,local,dtype", TC_CASES)
def test_tcgen05_forward_vs_oracle(Z, H, Hkv, N, D, RB, depth, causal, sink, local, dtype):
    gen = torch.Generator().manual_seed(N + D)
    q = randn((Z, H, N, D), gen).to(dtype)
    k = randn((Z, Hkv, N, D), gen).to(dtype)
    v = randn((Z, Hkv, N, D), gen).to(dtype)
    NB = -(-N // RB)
    router = random_router(Z, H, NB, 8, 2, seed=N).to(DEV)
    bl = build_block_lists(router, depth, is_causal=causal, sink_block=sink, local_blocks=local, arity=2)
    out, lse = block_list_attention(q.to(DEV), k.to(DEV), v.to(DEV), bl, route_block=RB,
                                    is_causal=causal, return_lse=True)
    ref, ref_lse = oracle_fwd(q.float(), k.float(), v.float(), bl, RB, causal)
    assert_half_close(out, ref, "out")
    lse_close(lse, ref_lse, 2e-2)
    out2 = block_list_attention(q.to(DEV), k.to(DEV), v.to(DEV), bl, route_block=RB, is_causal=causal)
    assert torch.equal(out, out2), "storing the LSE changed the output"


@pytest.mark.parametrize("D,dtype,causal", [(128, torch.bfloat16, False), (64, torch.float16, False),
                                             (128, torch.float16, True), (64, torch.bfloat16, True)])
def test_tcgen05_forward_one_tile_items(D, dtype, causal):
    """Lists of 0-3 blocks per query block in a pattern that gives runs of one-tile work items
    (finished by one softmax group alone, alternating groups) between longer items (both
    groups, merged) and empty ones."""
    Z, H, Hkv, RB, NB = 1, 4, 2, 128, 40
    N = NB * RB - 37  # a ragged tail
    gen = torch.Generator().manual_seed(D + 3)
    q = randn((Z, H, N, D), gen).to(dtype)
    k = randn((Z, Hkv, N, D), gen).to(dtype)
    v = randn((Z, Hkv, N, D), gen).to(dtype)
    m = torch.zeros(Z, H, NB, NB, dtype=torch.bool)
    for h in range(H):
        for i in range(NB):
            n = (1, 1, 1, 2, 1, 0, 3, 1, 1)[(i * 5 + h) % 9]
            hi = i + 1 if causal else NB
            cols = torch.randperm(hi, generator=gen)[:n]
            if causal and n > 0:
                cols[0] = i  # keep the diagonal so that causal rows see a key
            m[0, h, i, cols] = True
    bl = build_block_lists_from_mask(m.to(DEV))
    out, lse = block_list_attention(q.to(DEV), k.to(DEV), v.to(DEV), bl, route_block=RB,
                                    is_causal=causal, return_lse=True)
    ref, ref_lse = oracle_fwd(q.float(), k.float(), v.float(), bl, RB, causal)
    assert_half_close(out, ref, "out")
    lse_close(lse, ref_lse, 2e-2)


def test_tcgen05_forward_bias_empty_rows_and_strides():
    Z, H, N, D, RB = 1, 4, 640, 128, 128
    gen = torch.Generator().manual_seed(5)
    # (Z, N, H, D) storage viewed as (Z, H, N, D): non-contiguous heads, as HF layouts give
    q = randn((Z, N, H, D), gen).to(torch.bfloat16).to(DEV).transpose(1, 2)
    k = randn((Z, N, H, D), gen).to(torch.bfloat16).to(DEV).transpose(1, 2)
    v = randn((Z, N, H, D), gen).to(torch.bfloat16).to(DEV).transpose(1, 2)
    router = random_router(Z, H, 5, 4, 2, seed=3).to(DEV)
    bl = build_block_lists(router, 1, is_causal=True, sink_block=True)
    counts = bl.counts.clone()
    counts[0, 2, 3] = 0
    bl = BlockLists(bl.lists, counts, bl.max_count)
    bias = randn(bl.lists.shape, gen).to(DEV)
    out, lse = block_list_attention(q, k, v, bl, route_block=RB, is_causal=True, return_lse=True,
                                    soft_block_bias=bias)
    ref, ref_lse = oracle_fwd(q.float(), k.float(), v.float(), bl, RB, True, bias=bias)
    assert_half_close(out, ref, "out")
    lse_close(lse, ref_lse, 2e-2)
    assert (out[0, 2, 384:512] == 0).all() and torch.isinf(lse[0, 2, 384:512]).all()


@pytest.mark.parametrize("t,causal,sink", [(6, False, False), (4, True, True), (1, True, True)])
def test_c2_full_size_forward_head_subset(t, causal, sink):
    """BASELINE C2 at full size (N=8192, H=32/8, D=128, RB=128, bf16); the oracle checks a
    head subset (query-chunked fp32 masked attention)."""
    Z, H, Hkv, N, D, RB = 1, 32, 8, 8192, 128, 128
    gen = torch.Generator().manual_seed(0)
    q = randn((Z, H, N, D), gen).to(torch.bfloat16)
    k = randn((Z, Hkv, N, D), gen).to(torch.bfloat16)
    v = randn((Z, Hkv, N, D), gen).to(torch.bfloat16)
    router = tree_router(Z, H, N // RB, 6)
    bl = build_block_lists(router.to(DEV), t, is_causal=causal, sink_block=sink, arity=2)
    out, lse = block_list_attention(q.to(DEV), k.to(DEV), v.to(DEV), bl, route_block=RB,
                                    is_causal=causal, return_lse=True)
    heads = [0, 5, 31]
    bm = torch.from_numpy(blo.block_mask(router.numpy(), t, is_causal=causal, sink_block=sink))
    ref, ref_lse = ao.masked_attention_chunked(q.float(), k.float(), v.float(), bm, RB, causal,
                                               heads=heads, chunk=2048)
    assert_half_close(out[:, heads], ref, "C2 out")
    lse_close(lse[:, heads], ref_lse, 2e-2)


# ---------------------------------------------------------------------------------------
# backward on half precision (tcgen05-sized shapes)
# ---------------------------------------------------------------------------------------

BWD_CASES = [
    (1, 4, 2, 512, 128, 128, 1, True, True, 0, torch.bfloat16, False),
    (1, 2, 2, 300, 64, 128, 1, False, False, 1, torch.float16, True),
    (1, 4, 4, 384, 128, 128, [0, 1, 2, 3], True, True, 0, torch.bfloat16, True),
]


@pytest.mark.parametrize("Z,H,Hkv,N,D,RB,depth,causal,sink,local,dtype,with_bias", BWD_CASES)
def test_backward_half_vs_oracle(Z, H, Hkv, N, D, RB, depth, causal, sink, local, dtype, with_bias):
    gen = torch.Generator().manual_seed(7 + N)
    q = randn((Z, H, N, D), gen).to(dtype)
    k = randn((Z, Hkv, N, D), gen).to(dtype)
    v = randn((Z, Hkv, N, D), gen).to(dtype)
    do = randn((Z, H, N, D), gen).to(dtype)
    NB = -(-N // RB)
    router = random_router(Z, H, NB, 6, 2, seed=N).to(DEV)
    bl = build_block_lists(router, depth, is_causal=causal, sink_block=sink, local_blocks=local)
    qq, kk, vv = (t.to(DEV).requires_grad_(True) for t in (q, k, v))
    raw = torch.zeros(bl.lists.shape, device=DEV, requires_grad=True) if with_bias else None
    ste = (raw - raw.detach()) if with_bias else None
    out = block_list_attention(qq, kk, vv, bl, route_block=RB, is_causal=causal, soft_block_bias=ste)
    out.backward(do.to(DEV))
    bm = block_mask_from_lists(bl.lists, bl.counts)
    mask = ao.token_mask(bm, RB, N, causal)
    res = ao.masked_attention_grads(q.float(), k.float(), v.float(), mask, do.float(),
                                    block_bias=torch.zeros(bl.lists.shape) if with_bias else None,
                                    lists=bl.lists.cpu(), counts=bl.counts.cpu(), route_block=RB)
    assert_half_close(out, res["out"], "out")
    # gradients: per-tensor scale-aware (sums over many keys), 2e-2 abs + 1e-2 rel
    for name, t in (("dq", qq), ("dk", kk), ("dv", vv)):
        assert_half_close(t.grad, res[name], name)
    if with_bias:
        ref_db = res["d_bias"]
        err = (raw.grad.cpu().double() - ref_db).abs().max().item()
        assert err <= 2e-2 * max(1.0, ref_db.abs().max().item()), f"d_bias err {err}"


def test_backward_split_heavy_sink_column():
    """Causal + sink lists at N=2048 with 4 query heads per KV head: the sink key block is
    listed by every query block of the group, so the dK/dV planner splits that item into
    chunks whose fp32 partials are reduced separately; gradients must still match."""
    Z, H, Hkv, N, D, RB = 1, 4, 1, 2048, 128, 128
    gen = torch.Generator().manual_seed(31)
    q = randn((Z, H, N, D), gen).bfloat16()
    k = randn((Z, Hkv, N, D), gen).bfloat16()
    v = randn((Z, Hkv, N, D), gen).bfloat16()
    do = randn((Z, H, N, D), gen).bfloat16()
    router = tree_router(Z, H, N // RB, 4).to(DEV)
    bl = build_block_lists(router, [1, 1, 2, 1], is_causal=True, sink_block=True, arity=2)
    qq, kk, vv = (t.to(DEV).requires_grad_(True) for t in (q, k, v))
    out, lse = block_list_attention(qq, kk, vv, bl, route_block=RB, is_causal=True, return_lse=True)
    out.backward(do.to(DEV))
    mask = ao.token_mask(block_mask_from_lists(bl.lists, bl.counts), RB, N, True)
    res = ao.masked_attention_grads(q.float(), k.float(), v.float(), mask, do.float())
    assert_half_close(out, res["out"], "out")
    # The sink keys' dK/dV sum 8192 terms whose P / dS the reference kernels round to bf16
    # before the products (block_list.py:571-580, 666-680): compare with an oracle that
    # rounds at the same points, and with exact math at 2x the tolerance.
    lowp = ao.block_list_backward_lowp(q, k, v, out.detach().cpu(), do, lse.detach().cpu(), mask)
    for name, t in (("dq", qq), ("dk", kk), ("dv", vv)):
        assert_half_close(t.grad, lowp[name], name + " vs reference rounding")
        assert_half_close(t.grad, res[name], name + " vs exact", abs_tol=4e-2, rel_tol=2e-2)


# ---------------------------------------------------------------------------------------
# the fused single-pass backward (head_dim 128) against the oracle and the two-kernel path
# ---------------------------------------------------------------------------------------

FUSED_CASES = [
    # Z, H, Hkv, N, RB, depth, causal, sink, local, with_bias, empty_rows
    (1, 4, 1, 1024, 128, 1, True, True, 0, False, False),
    (2, 4, 2, 1000, 256, 1, True, True, 1, True, False),   # route block of two key tiles, tail
    (1, 2, 2, 320, 128, 2, False, False, 0, False, True),  # partial last sub-tile, empty rows
    (1, 8, 2, 768, 128, [0, 1, 2, 3, 1, 1, 2, 0], True, False, 0, True, False),
]


@pytest.mark.parametrize("Z,H,Hkv,N,RB,depth,causal,sink,local,with_bias,empty_rows", FUSED_CASES)
def test_fused_backward(Z, H, Hkv, N, RB, depth, causal, sink, local, with_bias, empty_rows):
    D = 128
    gen = torch.Generator().manual_seed(100 + N)
    q = randn((Z, H, N, D), gen).bfloat16()
    k = randn((Z, Hkv, N, D), gen).bfloat16()
    v = randn((Z, Hkv, N, D), gen).bfloat16()
    do = randn((Z, H, N, D), gen).bfloat16()
    NB = -(-N // RB)
    router = random_router(Z, H, NB, 6, 2, seed=N + 1).to(DEV)
    bl = build_block_lists(router, depth, is_causal=causal, sink_block=sink, local_blocks=local)
    if empty_rows:  # some query blocks list no key block: their dQ rows must come out zero
        counts = bl.counts.clone()
        counts[:, :, 1] = 0
        bl = BlockLists(bl.lists, counts, bl.max_count)
    grads = {}
    for det in (False, True):
        qq, kk, vv = (t.to(DEV).requires_grad_(True) for t in (q, k, v))
        raw = torch.zeros(bl.lists.shape, device=DEV, requires_grad=True) if with_bias else None
        ste = (raw - raw.detach()) if with_bias else None
        out = block_list_attention(qq, kk, vv, bl, route_block=RB, is_causal=causal,
                                   soft_block_bias=ste, deterministic=det)
        out.backward(do.to(DEV))
        grads[det] = {"out": out.detach(), "dq": qq.grad, "dk": kk.grad, "dv": vv.grad,
                      "db": raw.grad if with_bias else None}
    mask = ao.token_mask(block_mask_from_lists(bl.lists, bl.counts), RB, N, causal)
    res = ao.masked_attention_grads(q.float(), k.float(), v.float(), mask, do.float(),
                                    block_bias=torch.zeros(bl.lists.shape) if with_bias else None,
                                    lists=bl.lists.cpu(), counts=bl.counts.cpu(), route_block=RB)
    g = grads[False]
    for name in ("dq", "dk", "dv"):
        assert_half_close(g[name], res[name], f"fused {name}")
        # same math as the two-kernel path, up to bf16 rounding of the stored gradients
        assert_half_close(g[name], grads[True][name].float(), f"fused vs two-kernel {name}")
    if empty_rows:
        assert (g["dq"][:, :, RB:2 * RB] == 0).all()
    if with_bias:
        err = (g["db"].cpu().double() - res["d_bias"]).abs().max().item()
        assert err <= 2e-2 * max(1.0, res["d_bias"].abs().max().item()), f"d_bias err {err}"
    assert _native_status() == 0


def _native_status():
    from ultrametric import _native as nat
    return nat.read_device_status()


@pytest.mark.parametrize("RB,empty,with_bias", [(128, False, True), (256, False, False), (128, True, False)])
def test_forward_uniform_one_entry_items(RB, empty, with_bias):
    """Every query block lists exactly one key block (or none): the forward planner finds every
    work item of the same weight, and the kernel's scheduler then takes the items two per queue
    atomic and decodes them on two lanes -- with a soft bias, with two key tiles per list entry
    (route block 256), and with every item empty.  256 items, so most come from the queue."""
    Z, H, Hkv, D, N = 1, 16, 4, 128, 2048
    NB = N // RB
    gen = torch.Generator().manual_seed(RB + 11)
    q = randn((Z, H, N, D), gen).to(torch.bfloat16)
    k = randn((Z, Hkv, N, D), gen).to(torch.bfloat16)
    v = randn((Z, Hkv, N, D), gen).to(torch.bfloat16)
    m = torch.zeros(Z, H, NB, NB, dtype=torch.bool)
    if not empty:
        cols = torch.randint(0, NB, (H, NB), generator=gen)
        for h in range(H):
            m[0, h, torch.arange(NB), cols[h]] = True
    bl = build_block_lists_from_mask(m.to(DEV))
    bias = randn(bl.lists.shape, gen).to(DEV) if with_bias else None
    out, lse = block_list_attention(q.to(DEV), k.to(DEV), v.to(DEV), bl, route_block=RB,
                                    is_causal=False, return_lse=True, soft_block_bias=bias)
    if empty:
        assert (out == 0).all() and torch.isneginf(lse).all()
        return
    ref, ref_lse = oracle_fwd(q.float(), k.float(), v.float(), bl, RB, False, bias=bias)
    assert_half_close(out, ref, "out")
    lse_close(lse, ref_lse, 2e-2)

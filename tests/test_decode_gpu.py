"""GPU parity of the routed paged decode against the reference's outputs
(tests/golden/decode.npz: its Triton kernel under the CPU interpreter and its
``_ultrametric_decode_reference``) and the CPU oracle (GQA, bf16, C3-shaped cases).

fp32: 1e-5 relative (normwise) to the fp64 oracle and 1e-4 abs to the reference kernel;
bf16: 2e-2 abs + 1e-2 rel."""

import numpy as np
import pytest
import torch

from helpers import assert_fp32_close, assert_half_close, randn
from oracle import decode_oracle as dor
from ultrametric import ultrametric_decode

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _t(a):
    return torch.from_numpy(np.asarray(a))


@pytest.mark.parametrize("td", [1, 3, 5, 6, 7, 10])
def test_decode_reference_fixtures(golden, td):
    g = golden("decode")
    key = f"d{td:02d}"
    rd, local, sink = (int(x) for x in g[key + "_meta"])
    q, k, v = (_t(g[f"{key}_{n}"]).float() for n in "qkv")
    bt, ctx, ri, qri = (_t(g[f"{key}_{n}"]) for n in ("bt", "ctx", "ri", "qri"))
    out = ultrametric_decode(q.to(DEV), k.to(DEV), v.to(DEV), bt.to(DEV), ctx.to(DEV), ri.to(DEV),
                             qri.to(DEV), rd, local_blocks=local, sink_block=bool(sink))
    assert out.shape == q.shape
    assert (out.cpu() - _t(g[key + "_out_kernel"])).abs().max() < 1e-4
    ref = dor.ultrametric_decode_reference(q, k, v, bt, ctx, ri, qri, rd, local_blocks=local,
                                           sink_block=bool(sink), compute_dtype=torch.float64)
    assert_fp32_close(out, ref, key)


def test_decode_zero_context_and_no_match(golden):
    g = golden("decode")
    q, k, v = (_t(g[f"dz_{n}"]).float() for n in "qkv")
    bt, ctx, ri, qri = (_t(g[f"dz_{n}"]) for n in ("bt", "ctx", "ri", "qri"))
    out = ultrametric_decode(q.to(DEV), k.to(DEV), v.to(DEV), bt.to(DEV), ctx.to(DEV), ri.to(DEV),
                             qri.to(DEV), 1)
    assert (out.cpu() - _t(g["dz_out_ref"])).abs().max() < 1e-5
    assert (out[0] == 0).all()


def make_paged(B, H, Hkv, D, page, ctx_lo, ctx_hi, TD, seed, dtype=torch.bfloat16, shared_routes=True):
    gen = torch.Generator().manual_seed(seed)
    ctx = torch.randint(ctx_lo, ctx_hi + 1, (B,), generator=gen, dtype=torch.int32)
    n_log = (ctx + page - 1) // page
    maxL = int(n_log.max())
    total = int(n_log.sum()) + 3
    perm = torch.randperm(total, generator=gen).to(torch.int32)
    bt = torch.zeros(B, maxL, dtype=torch.int32)
    off = 0
    logical_of = torch.zeros(total, dtype=torch.int64)
    for b in range(B):
        n = int(n_log[b])
        bt[b, :n] = perm[off:off + n]
        logical_of[perm[off:off + n].long()] = torch.arange(n)
        off += n
    q = randn((B, H, D), gen).to(dtype)
    kc = randn((total, Hkv, page, D), gen).to(dtype)
    vc = randn((total, Hkv, page, D), gen).to(dtype)
    bits = ((logical_of.view(-1, 1) >> torch.arange(TD - 1, -1, -1).view(1, -1)) & 1).to(torch.int32)
    if shared_routes:
        ri = bits.view(total, 1, TD).expand(total, H, TD).contiguous()
        leaf = torch.randint(0, 1 << TD, (B,), generator=gen)
        qb = ((leaf.view(-1, 1) >> torch.arange(TD - 1, -1, -1).view(1, -1)) & 1).to(torch.int32)
        qri = qb.view(B, 1, TD).expand(B, H, TD).contiguous()
    else:
        ri = torch.randint(0, 2, (total, H, TD), generator=gen, dtype=torch.int32)
        qri = torch.randint(0, 2, (B, H, TD), generator=gen, dtype=torch.int32)
    return q, kc, vc, bt, ctx, ri, qri


@pytest.mark.parametrize("B,H,Hkv,D,page,lo,hi,TD,rd,local,sink,shared,dtype", [
    (4, 8, 2, 128, 64, 100, 3000, 9, 2, 1, True, True, torch.bfloat16),
    (3, 4, 4, 64, 16, 1, 500, 6, 3, 2, False, False, torch.bfloat16),
    (2, 8, 1, 128, 32, 700, 900, 5, 1, 0, True, False, torch.float16),
    (5, 6, 2, 32, 8, 20, 200, 5, 2, 1, True, False, torch.float32),
])
def test_decode_gqa_vs_oracle(B, H, Hkv, D, page, lo, hi, TD, rd, local, sink, shared, dtype):
    q, kc, vc, bt, ctx, ri, qri = make_paged(B, H, Hkv, D, page, lo, hi, TD, seed=B * 7 + D, dtype=dtype,
                                             shared_routes=shared)
    out = ultrametric_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), ctx.to(DEV), ri.to(DEV),
                             qri.to(DEV), rd, local_blocks=local, sink_block=sink)
    ref = dor.ultrametric_decode_reference(q.float(), kc.float(), vc.float(), bt, ctx, ri, qri, rd,
                                           local_blocks=local, sink_block=sink,
                                           compute_dtype=torch.float64)
    if dtype == torch.float32:
        assert_fp32_close(out, ref, "decode fp32")
    else:
        assert_half_close(out, ref, "decode")


@pytest.mark.parametrize("B,H,Hkv,D,page,lo,hi,TD,rd,local,sink,shared,dtype", [
    (3, 16, 1, 128, 128, 1, 1000, 6, 2, 1, True, False, torch.bfloat16),  # 16 heads per KV head
    (2, 4, 2, 64, 256, 300, 1200, 5, 1, 0, True, True, torch.float16),   # tiles inside a page
    (6, 8, 8, 128, 16, 1, 400, 6, 3, 2, False, True, torch.bfloat16),    # 4 pages per tile
    (5, 8, 4, 64, 32, 1, 700, 6, 2, 1, True, False, torch.bfloat16),     # 2 pages per tile
    (4, 12, 4, 128, 64, 1, 5000, 7, 2, 3, True, False, torch.bfloat16),  # 3 heads per KV head
    (3, 8, 2, 128, 48, 10, 900, 5, 2, 1, True, False, torch.bfloat16),   # general path (page 48)
])
def test_decode_fast_path_shapes(B, H, Hkv, D, page, lo, hi, TD, rd, local, sink, shared, dtype):
    """Shapes of the tensor-core path: group sizes 1..16, page sizes 16..256 (several pages
    per 64-token tile, several tiles per page, partial last pages), and one shape that
    takes the general path, all against the fp64 oracle."""
    q, kc, vc, bt, ctx, ri, qri = make_paged(B, H, Hkv, D, page, lo, hi, TD, seed=B * 11 + page,
                                             dtype=dtype, shared_routes=shared)
    out = ultrametric_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), ctx.to(DEV), ri.to(DEV),
                             qri.to(DEV), rd, local_blocks=local, sink_block=sink)
    ref = dor.ultrametric_decode_reference(q.float(), kc.float(), vc.float(), bt, ctx, ri, qri, rd,
                                           local_blocks=local, sink_block=sink,
                                           compute_dtype=torch.float64)
    assert_half_close(out, ref, "decode")


def test_decode_nonfinite_cache_past_context():
    """Cache slots past a request's context length hold inf / NaN (stale memory); the
    result must not see them (the reference loads them masked to 0)."""
    B, H, Hkv, D, page, TD = 3, 8, 2, 128, 64, 6
    q, kc, vc, bt, ctx, ri, qri = make_paged(B, H, Hkv, D, page, 70, 300, TD, seed=5,
                                             shared_routes=True)
    kc2, vc2 = kc.clone(), vc.clone()
    for b in range(B):
        n = int(ctx[b])
        last = int(bt[b, (n - 1) // page])
        r = n - ((n - 1) // page) * page
        if r < page:
            kc2[last, :, r:] = float("nan")
            vc2[last, :, r:] = float("inf")
    out = ultrametric_decode(q.to(DEV), kc2.to(DEV), vc2.to(DEV), bt.to(DEV), ctx.to(DEV),
                             ri.to(DEV), qri.to(DEV), 2, local_blocks=1, sink_block=True)
    ref = dor.ultrametric_decode_reference(q.float(), kc.float(), vc.float(), bt, ctx, ri, qri, 2,
                                           local_blocks=1, sink_block=True,
                                           compute_dtype=torch.float64)
    assert torch.isfinite(out).all()
    assert_half_close(out, ref, "decode")


def test_decode_c3_shape_subset():
    """BASELINE C3 per-request shape (H=32/8, D=128, page 64, ctx in [2048, 32768],
    req_depth 4, sink + last page) with 16 of the 64 requests to bound host memory; the
    oracle checks 4 of them."""
    B, H, Hkv, D, page, TD = 16, 32, 8, 128, 64, 9
    q, kc, vc, bt, ctx, ri, qri = make_paged(B, H, Hkv, D, page, 2048, 32768, TD, seed=0)
    out = ultrametric_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), ctx.to(DEV), ri.to(DEV),
                             qri.to(DEV), 4, local_blocks=1, sink_block=True)
    reqs = [0, 5, 11, 15]
    ref = dor.ultrametric_decode_reference(q.float(), kc.float(), vc.float(), bt, ctx, ri, qri, 4,
                                           local_blocks=1, sink_block=True, requests=reqs,
                                           compute_dtype=torch.float64)
    assert_half_close(out[reqs], ref[reqs], "C3 decode")

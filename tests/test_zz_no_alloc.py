"""The decode entry point that allocates nothing (``sa_ultrametric_decode_noalloc``).

It serves callers that cannot allocate device memory when they decode -- e.g. a serving
loop whose memory is carved up front by its own pool and that binds only the C ABI, so it
has no allocator to call for the split-K workspace.  The entry point takes that workspace
from a fixed device array inside the library instead.

This file is collected last on purpose.  Both tests call the library through the C ABI
(ctypes), the way such a caller would; the first compares the no-alloc entry point with
``sa_ultrametric_decode`` (caller workspace) on two calls in a row, which also checks that
the shared array's leftover contents from the first call do not leak into the second.  It
runs on the bf16 fast path (D=128, page 64) and on the general split-K path (fp32, and
bf16 with D=32), both of which keep their partials in the shared array.
"""

import ctypes

import pytest
import torch

from helpers import assert_fp32_close, assert_half_close
from ultrametric import _native as nat

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(seed, B=6, H=8, Hkv=2, D=128, page=64, TD=6, dtype=torch.bfloat16):
    gen = torch.Generator().manual_seed(seed)
    ctx = torch.randint(1, 3000, (B,), generator=gen, dtype=torch.int32)
    ctx[0] = 0  # a request with no context
    n_log = (ctx + page - 1) // page
    maxL = int(n_log.max())
    total = int(n_log.sum()) + 2
    perm = torch.randperm(total, generator=gen).to(torch.int32)
    bt = torch.zeros(B, maxL, dtype=torch.int32)
    off = 0
    for b in range(B):
        n = int(n_log[b])
        bt[b, :n] = perm[off:off + n]
        off += n
    t = dict(
        q=torch.randn(B, H, D, generator=gen).to(dtype),
        kc=torch.randn(total, Hkv, page, D, generator=gen).to(dtype),
        vc=torch.randn(total, Hkv, page, D, generator=gen).to(dtype),
        bt=bt, ctx=ctx,
        ri=torch.randint(0, 2, (total, H, TD), generator=gen, dtype=torch.int32),
        qri=torch.randint(0, 2, (B, H, TD), generator=gen, dtype=torch.int32),
    )
    return {k: v.to(DEV) for k, v in t.items()}


def _common_args(t, out, req_depth=2, local_blocks=1, sink=1):
    q, kc, vc, bt, ctx, ri, qri = (t[k] for k in ("q", "kc", "vc", "bt", "ctx", "ri", "qri"))
    B, H, D = q.shape
    P, Hkv, page, _ = kc.shape
    sa_dtype = {torch.bfloat16: nat.SA_BF16, torch.float16: nat.SA_F16, torch.float32: nat.SA_F32}[q.dtype]
    return [sa_dtype, B, H, Hkv, D, page, P,
            q.data_ptr(), nat.strides(q), kc.data_ptr(), nat.strides(kc),
            vc.data_ptr(), nat.strides(vc), bt.data_ptr(), nat.strides(bt), bt.shape[1],
            ctx.data_ptr(), ri.data_ptr(), nat.SA_I32, nat.strides(ri),
            qri.data_ptr(), nat.SA_I32, nat.strides(qri), ri.shape[-1], req_depth, local_blocks,
            sink, out.data_ptr(), nat.strides(out)]


def _with_workspace(t):
    out = torch.empty_like(t["q"])
    q = t["q"]
    need = nat.lib().sa_ultrametric_decode_workspace_bytes(q.shape[0], q.shape[1], t["kc"].shape[1],
                                                           q.shape[2], t["bt"].shape[1])
    ws = torch.empty(max(need, 256), dtype=torch.uint8, device=DEV)
    args = _common_args(t, out) + [ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream]
    nat.check(nat.lib().sa_ultrametric_decode(*args), "sa_ultrametric_decode")
    return out


def _no_alloc(t):
    out = torch.empty_like(t["q"])
    args = _common_args(t, out) + [torch.cuda.current_stream().cuda_stream]
    nat.check(nat.lib().sa_ultrametric_decode_noalloc(*args), "sa_ultrametric_decode_noalloc")
    return out


@pytest.mark.parametrize("dtype,D,page", [
    (torch.bfloat16, 128, 64),  # fast path (decode_sm100.cu)
    (torch.float32, 128, 64),   # general split-K path (decode.cu), fp32
    (torch.bfloat16, 32, 16),   # general split-K path, a head_dim the fast path does not take
])
def test_no_alloc_decode_matches_workspace_decode_twice(dtype, D, page):
    for seed in (11, 12):  # two calls in a row, different inputs
        t = _inputs(seed, D=D, page=page, dtype=dtype)
        ref = _with_workspace(t)
        got = _no_alloc(t)
        torch.cuda.synchronize()
        what = f"no-alloc decode ({dtype}, D={D}, call with seed {seed})"
        if dtype == torch.float32:
            assert_fp32_close(got, ref, what)
        else:
            assert_half_close(got, ref.float(), what)
        assert (got[0] == 0).all()
    assert nat.read_device_status() == 0


def test_no_alloc_decode_rejects_oversized_requests():
    t = _inputs(3)
    out = torch.empty_like(t["q"])
    args = _common_args(t, out) + [torch.cuda.current_stream().cuda_stream]
    # pretend a batch of 200k requests: its workspace exceeds the fixed array
    args[1] = 200_000
    rc = nat.lib().sa_ultrametric_decode_noalloc(*args)
    assert rc == nat.SA_EWORKSPACE
    assert b"fixed" in nat.lib().sa_last_error()

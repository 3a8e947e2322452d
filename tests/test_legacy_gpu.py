"""GPU parity of the legacy entry points of sparse-ai's ``src/ultrametric/kernel.py``,
which here are shims onto the block-list kernels:

* ``ultrametric_attention_triton`` (kernel.py:420-517): fp16, per-``min(128, N)``-block
  routes matched on the first ``req_depth`` levels (kernel.py:123-149: no sink, no local
  band), optional causal mask; returns ``(out, L)`` with L the natural-log LSE;
* ``CurriculumSparseAttention`` (kernel.py:583-671): the same forward (non-causal) with
  its backward.

Checked against the CPU oracle (masked dense attention in fp32) at the half-precision
tolerance of this build: 2e-2 abs + 1e-2 rel.
"""

import math

import pytest
import torch

from helpers import assert_half_close, lse_close, random_router
from oracle import attention_oracle as ao
from oracle import block_list_oracle as blo
from ultrametric.kernel import CurriculumSparseAttention, ultrametric_attention_triton

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(Z, H, N, D, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(Z, H, N, D, generator=g).half() for _ in range(3)]


def _oracle(q, k, v, routes, depth, causal, rb):
    N = q.shape[2]
    bm = torch.from_numpy(blo.block_mask(routes.numpy(), depth, is_causal=causal))
    mask = ao.token_mask(bm, rb, N, causal)
    return ao.masked_attention(q.float(), k.float(), v.float(), mask), mask


@pytest.mark.parametrize("N,depth,causal", [(512, 2, False), (512, 1, True), (384, 3, True),
                                            (64, 1, False)])
def test_ultrametric_attention_triton_shim(N, depth, causal):
    Z, H, D = 1, 2, 64
    q, k, v = _inputs(Z, H, N, D, seed=N + depth)
    rb = 128 if N >= 128 else N
    nb = -(-N // rb)
    routes = random_router(Z, H, nb, 4, 2, seed=depth)
    out, lse = ultrametric_attention_triton(q.to(DEV), k.to(DEV), v.to(DEV), routes.to(DEV),
                                            req_depth=depth, p=2, is_causal=causal)
    (ref, ref_lse), _ = _oracle(q, k, v, routes, depth, causal, rb)
    assert out.dtype == torch.float16 and out.shape == q.shape
    assert_half_close(out, ref, f"legacy forward N={N} depth={depth}")
    lse_close(lse, ref_lse, 2e-2)


def test_ultrametric_attention_triton_pads_short_routes():
    # fewer route blocks than ceil(N / 128): the missing blocks route to branch 0
    Z, H, N, D = 1, 1, 512, 64
    q, k, v = _inputs(Z, H, N, D, seed=5)
    routes = random_router(Z, H, 2, 3, 2, seed=9)
    out, _ = ultrametric_attention_triton(q.to(DEV), k.to(DEV), v.to(DEV), routes.to(DEV),
                                          req_depth=2)
    padded = torch.cat([routes, torch.zeros(Z, H, 2, 3, dtype=torch.int32)], dim=2)
    (ref, _), _ = _oracle(q, k, v, padded, 2, False, 128)
    assert_half_close(out, ref, "legacy forward with padded routes")


def test_ultrametric_attention_triton_rejects_bad_depth():
    q = torch.zeros(1, 1, 128, 64, dtype=torch.float16, device=DEV)
    routes = torch.zeros(1, 1, 1, 2, dtype=torch.int32, device=DEV)
    with pytest.raises(AssertionError):
        ultrametric_attention_triton(q, q, q, routes, req_depth=3)


def test_curriculum_sparse_attention_grads():
    Z, H, N, D, depth = 1, 2, 256, 64, 1
    q, k, v = _inputs(Z, H, N, D, seed=21)
    g = torch.Generator().manual_seed(22)
    do = torch.randn(Z, H, N, D, generator=g).half()
    routes = random_router(Z, H, 2, 3, 2, seed=23)
    qd, kd, vd = (t.to(DEV).requires_grad_(True) for t in (q, k, v))
    out = CurriculumSparseAttention.apply(qd, kd, vd, routes.to(DEV), depth, 2, True)
    out.backward(do.to(DEV))
    _, mask = _oracle(q, k, v, routes, depth, False, 128)
    ref = ao.masked_attention_grads(q.float(), k.float(), v.float(), mask, do.float())
    assert_half_close(out, ref["out"], "curriculum out")
    for name, got in (("dq", qd.grad), ("dk", kd.grad), ("dv", vd.grad)):
        assert_half_close(got, ref[name], f"curriculum {name}")

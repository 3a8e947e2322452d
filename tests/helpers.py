"""Seeded input generators and tolerance checks shared by the tests.

Inputs are drawn on the CPU with ``torch.Generator`` (q, k, v, then dO) and copied to the
device, so the CPU oracle and the kernels see identical values."""

from __future__ import annotations

import math

import numpy as np
import torch

# Tolerances stated by the north star of this build:
#   fp32 outputs within 1e-5 relative (normwise: max|err| / max|ref|) of the fp64 oracle;
#   bf16/fp16 outputs and gradients within 2e-2 absolute + 1e-2 relative (elementwise).
FP32_REL = 1e-5
HALF_ABS = 2e-2
HALF_REL = 1e-2


def randn(shape, gen, dtype=torch.float32):
    return torch.randn(*shape, generator=gen).to(dtype)


def random_router(Z, H, NB, TD, p, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, p, (Z, H, NB, TD), generator=g, dtype=torch.int32)


def tree_router(Z, H, NB, TD):
    depth = max(1, math.ceil(math.log2(max(NB, 2))))
    r = torch.zeros(Z, H, NB, TD, dtype=torch.int32)
    for d in range(min(depth, TD)):
        r[:, :, :, d] = (torch.arange(NB) >> (depth - 1 - d)) % 2
    return r


def block_mask_from_lists(lists, counts, NBK=None):
    Z, H, NB = counts.shape
    NBK = NB if NBK is None else NBK
    m = torch.zeros(Z, H, NB, NBK, dtype=torch.bool)
    lists = lists.cpu()
    counts = counts.cpu()
    for z in range(Z):
        for h in range(H):
            for i in range(NB):
                c = int(counts[z, h, i])
                if c:
                    m[z, h, i, lists[z, h, i, :c].long()] = True
    return m


def assert_fp32_close(out, ref, what=""):
    out = out.detach().double().cpu()
    ref = ref.detach().double().cpu()
    scale = ref.abs().max().item()
    err = (out - ref).abs().max().item()
    assert err <= FP32_REL * max(scale, 1e-30), f"{what}: max err {err:.3e} vs scale {scale:.3e}"


def assert_half_close(out, ref, what="", abs_tol=HALF_ABS, rel_tol=HALF_REL):
    out = out.detach().double().cpu()
    ref = ref.detach().double().cpu()
    assert torch.isfinite(out).all(), f"{what}: non-finite values"
    bad = (out - ref).abs() > abs_tol + rel_tol * ref.abs()
    if bad.any():
        idx = bad.nonzero()[0].tolist()
        raise AssertionError(f"{what}: {int(bad.sum())} elements out of tolerance, first at {idx}: "
                             f"{out[tuple(idx)].item():.5f} vs {ref[tuple(idx)].item():.5f}; "
                             f"max err {(out - ref).abs().max().item():.3e}")


def lse_close(lse, ref, tol):
    lse = lse.detach().double().cpu()
    ref = ref.detach().double().cpu()
    fin = torch.isfinite(ref)
    assert torch.equal(fin, torch.isfinite(lse)), "lse: -inf pattern differs"
    if fin.any():
        err = (lse[fin] - ref[fin]).abs().max().item()
        assert err < tol, f"lse max err {err:.3e}"

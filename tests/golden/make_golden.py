"""Generate the golden fixtures in this folder by running the sparse-ai reference itself.

Run once, in a container that has the reference checkout (its path is the first argument,
the folder holding ``src/ultrametric``):

    TRITON_INTERPRET=1 python tests/golden/make_golden.py <reference-root>

``TRITON_INTERPRET=1`` makes the reference's own Triton kernels run on the CPU in fp32
(the reference's test strategy, tests/test_block_list.py:27-29 there), so the fixtures
hold outputs of:

* ``build_block_lists`` (sync path, sync-free ``arity=`` path, per-level overflow path),
  cross-checked inside this script against a direct launch of ``_build_block_lists_kernel``;
* ``build_transposed_block_lists``;
* ``block_list_attention`` forward (+ LSE, + soft block bias) and backward (dQ, dK, dV,
  d_soft_block_bias) -- the Triton kernels themselves;
* ``block_sparse_attention`` on its CPU fallback path (the reference's CPU path);
* ``ultrametric_decode`` (Triton kernel) and ``_ultrametric_decode_reference``.

Inputs are drawn with torch's seeded CPU generator and rounded to fp16 so they are exact
in the stored fp16 arrays; outputs are stored in fp32.  Nothing at test time reads the
reference: tests load the ``.npz`` files only.
"""

from __future__ import annotations

import math
import os
import sys

import numpy as np


def main(ref_root: str, out_dir: str) -> None:
    assert os.environ.get("TRITON_INTERPRET") == "1", "run with TRITON_INTERPRET=1"
    sys.path.insert(0, os.path.join(ref_root, "src"))
    import torch
    from ultrametric import block_list as bl_mod
    from ultrametric.block_list import (block_list_attention, block_mask_reference,
                                        build_block_lists, build_transposed_block_lists)
    from ultrametric.kernel import block_sparse_attention
    from ultrametric.kernel_decode import _ultrametric_decode_reference, ultrametric_decode

    def rand_router(Z, H, NB, TD, p, seed):
        g = torch.Generator().manual_seed(seed)
        return torch.randint(0, p, (Z, H, NB, TD), generator=g, dtype=torch.int32)

    def tree_router(Z, H, NB, TD):
        depth = max(1, math.ceil(math.log2(max(NB, 2))))
        r = torch.zeros(Z, H, NB, TD, dtype=torch.int32)
        for d in range(depth):
            r[:, :, :, d] = (torch.arange(NB) >> (depth - 1 - d)) % 2
        return r

    def halfrand(shape, gen):
        return torch.randn(*shape, generator=gen).half().float()

    # ------------------------------------------------------------------ builder
    builder = {}
    n = 0

    def add_builder(router, depth, kw, arity=None):
        nonlocal n
        b = build_block_lists(router, depth, arity=arity, **kw)
        key = f"b{n:03d}"
        n += 1
        d = np.asarray(depth if not isinstance(depth, int) else [depth] * router.shape[1],
                       dtype=np.int64)
        builder[key + "_router"] = router.numpy().astype(np.int64)
        builder[key + "_depth"] = d
        builder[key + "_depth_is_int"] = np.array(isinstance(depth, int))
        builder[key + "_flags"] = np.array([int(kw["is_causal"]), int(kw["sink_block"]),
                                            int(kw["local_blocks"]), -1 if arity is None else arity],
                                           dtype=np.int64)
        builder[key + "_lists"] = b.lists.numpy()
        builder[key + "_counts"] = b.counts.numpy()
        builder[key + "_max_count"] = np.array(b.max_count)
        t = build_transposed_block_lists(b, num_key_blocks=router.shape[2])
        builder[key + "_tlists"] = t.lists.numpy()
        builder[key + "_tcounts"] = t.counts.numpy()
        builder[key + "_tmax_count"] = np.array(t.max_count)
        # The fused Triton compaction kernel (run by the interpreter) must agree.
        if router.shape[2] <= 1024 and arity is not None and isinstance(depth, int):
            Z, H, NB, TD = router.shape
            base = max(2, arity)
            levels = torch.arange(TD)
            keep = (levels < depth).view(1, 1, 1, TD)
            if TD * math.log2(base) < 62:
                code = (router.to(torch.int64) * keep * torch.pow(base, levels)).sum(-1).contiguous()
                lf = torch.zeros((Z, H, NB, NB), dtype=torch.int32)
                cn = torch.empty((Z, H, NB), dtype=torch.int32)
                bl_mod._build_block_lists_kernel[(NB, Z * H)](
                    code, lf, cn, *code.stride(), *lf.stride(), *cn.stride(), H, NB,
                    IS_CAUSAL=kw["is_causal"], SINK_BLOCK=kw["sink_block"],
                    LOCAL_BLOCKS=kw["local_blocks"], BLOCK_NB=1 << (NB - 1).bit_length())
                assert torch.equal(cn, b.counts), "triton compaction != torch builder"
                assert torch.equal(lf, b.lists), "triton compaction lists differ"

    for p in (2, 3):
        for causal in (False, True):
            for sink, local in ((False, 0), (True, 0), (False, 1), (True, 2)):
                kw = dict(is_causal=causal, sink_block=sink, local_blocks=local)
                add_builder(rand_router(2, 3, 7, 4, p, seed=p), [0, 2, 4], kw)
    for p in (2, 3):
        for causal in (False, True):
            for depth in (0, 1, 3, [0, 2]):
                kw = dict(is_causal=causal, sink_block=True, local_blocks=0)
                add_builder(rand_router(2, 2, 9, 3, p, seed=7), depth, kw, arity=p)
    # sync-free with ids >= arity: the reference's mixed-radix codes may collide
    kw = dict(is_causal=False, sink_block=False, local_blocks=0)
    add_builder(rand_router(1, 2, 12, 3, 5, seed=11), 3, kw, arity=2)
    add_builder(rand_router(1, 2, 12, 3, 5, seed=12), [2, 3], kw, arity=3)
    # per-level path: TD * log2(base) >= 62
    add_builder(rand_router(1, 2, 10, 40, 3, seed=5), [20, 40], dict(is_causal=True, sink_block=False, local_blocks=1))
    add_builder(rand_router(1, 1, 10, 40, 3, seed=6), 30, dict(is_causal=False, sink_block=True, local_blocks=0), arity=3)
    # tree routing (known-answer shapes) and a C2-like per-head threshold case
    for r in range(5):
        add_builder(tree_router(1, 1, 16, 4), r, dict(is_causal=False, sink_block=False, local_blocks=0))
    add_builder(tree_router(1, 4, 64, 6), [1, 2, 4, 6], dict(is_causal=True, sink_block=True, local_blocks=0))
    add_builder(tree_router(1, 2, 64, 6), 6, dict(is_causal=True, sink_block=True, local_blocks=1), arity=2)
    # larger NB through the fused kernel cross-check
    add_builder(rand_router(1, 2, 200, 8, 2, seed=3), 3, dict(is_causal=True, sink_block=True, local_blocks=2), arity=2)
    np.savez_compressed(os.path.join(out_dir, "builder.npz"), **builder)

    # ------------------------------------------------------------------ forward
    fwd = {}
    cases = [
        # (N, rb, bm, bn, depth, causal, sink, local) -- tests/test_block_list.py:190-196
        (200, 64, 32, 32, 1, False, False, 0),
        (200, 64, 32, 32, 2, True, False, 0),
        (256, 64, 64, 32, 2, True, True, 0),
        (192, 64, 32, 64, 1, False, False, 1),
        (160, 32, 32, 32, 0, True, False, 0),
        (300, 128, 64, 64, 2, True, True, 1),
    ]
    for i, (N, rb, bm, bn, depth, causal, sink, local) in enumerate(cases):
        gen = torch.Generator().manual_seed(1000 + i)
        Z, H, D = 1, 2, 32
        q, k, v = (halfrand((Z, H, N, D), gen) for _ in range(3))
        NB = math.ceil(N / rb)
        router = rand_router(Z, H, NB, 3, 2, seed=N)
        kw = dict(is_causal=causal, sink_block=sink, local_blocks=local)
        b = build_block_lists(router, depth, **kw)
        out, lse = block_list_attention(q, k, v, b, route_block=rb, is_causal=causal,
                                        block_m=bm, block_n=bn, return_lse=True)
        key = f"f{i:02d}"
        for nm, t in (("q", q), ("k", k), ("v", v)):
            fwd[f"{key}_{nm}"] = t.half().numpy()
        fwd[f"{key}_router"] = router.numpy()
        fwd[f"{key}_meta"] = np.array([N, rb, depth, int(causal), int(sink), local])
        fwd[f"{key}_lists"] = b.lists.numpy()
        fwd[f"{key}_counts"] = b.counts.numpy()
        fwd[f"{key}_out"] = out.numpy()
        fwd[f"{key}_lse"] = lse.numpy()
    # forward with a non-zero soft block bias and an empty row (count 0)
    gen = torch.Generator().manual_seed(77)
    Z, H, N, D, rb = 1, 2, 128, 32, 32
    q, k, v = (halfrand((Z, H, N, D), gen) for _ in range(3))
    router = rand_router(Z, H, 4, 3, 2, seed=9)
    b = build_block_lists(router, 1, is_causal=True, sink_block=True)
    counts = b.counts.clone()
    counts[0, 1, 2] = 0  # an empty query block: zero output, -inf lse
    b = bl_mod.BlockLists(b.lists, counts, b.max_count)
    bias = halfrand((Z, H, 4, b.max_count), gen)
    out, lse = block_list_attention(q, k, v, b, route_block=rb, is_causal=True, block_m=32,
                                    block_n=32, return_lse=True, soft_block_bias=bias)
    for nm, t in (("q", q), ("k", k), ("v", v), ("bias", bias)):
        fwd[f"fb_{nm}"] = t.half().numpy()
    fwd["fb_lists"] = b.lists.numpy()
    fwd["fb_counts"] = b.counts.numpy()
    fwd["fb_out"] = out.numpy()
    fwd["fb_lse"] = lse.numpy()
    # quickstart on the CPU fallback (the reference's CPU path), routes padded 2 -> 3 blocks
    gen = torch.Generator().manual_seed(3)
    Z, H, N, D = 2, 2, 300, 32
    q, k, v = (halfrand((Z, H, N, D), gen) for _ in range(3))
    router = rand_router(Z, H, 2, 4, 2, seed=5)
    os.environ["TRITON_INTERPRET"] = "0"
    import ultrametric.kernel as kmod
    saved = kmod.HAS_TRITON
    kmod.HAS_TRITON = False
    for causal in (False, True):
        out, L = block_sparse_attention(q, k, v, router, req_depth=2, is_causal=causal)
        fwd[f"qs{int(causal)}_out"] = out.numpy()
        fwd[f"qs{int(causal)}_lse"] = L.numpy()
    kmod.HAS_TRITON = saved
    os.environ["TRITON_INTERPRET"] = "1"
    for nm, t in (("q", q), ("k", k), ("v", v)):
        fwd[f"qs_{nm}"] = t.half().numpy()
    fwd["qs_router"] = router.numpy()
    np.savez_compressed(os.path.join(out_dir, "forward.npz"), **fwd)

    # ------------------------------------------------------------------ backward
    bwd = {}
    bcases = [
        (128, 64, 32, 32, 1, False, False, 0),
        (100, 32, 16, 16, 2, True, True, 0),
        (96, 32, 32, 16, 1, False, False, 1),
    ]
    for i, (N, rb, bm, bn, depth, causal, sink, local) in enumerate(bcases):
        gen = torch.Generator().manual_seed(2000 + i)
        Z, H, D = 1, 2, 16
        q0, k0, v0, do = (halfrand((Z, H, N, D), gen) for _ in range(4))
        router = rand_router(Z, H, math.ceil(N / rb), 3, 2, seed=N)
        kw = dict(is_causal=causal, sink_block=sink, local_blocks=local)
        b = build_block_lists(router, depth, **kw)
        q, k, v = (t.clone().requires_grad_(True) for t in (q0, k0, v0))
        out = block_list_attention(q, k, v, b, route_block=rb, is_causal=causal, block_m=bm, block_n=bn)
        out.backward(do)
        key = f"g{i:02d}"
        for nm, t in (("q", q0), ("k", k0), ("v", v0), ("do", do)):
            bwd[f"{key}_{nm}"] = t.half().numpy()
        bwd[f"{key}_meta"] = np.array([N, rb, depth, int(causal), int(sink), local])
        bwd[f"{key}_lists"] = b.lists.numpy()
        bwd[f"{key}_counts"] = b.counts.numpy()
        bwd[f"{key}_out"] = out.detach().numpy()
        bwd[f"{key}_dq"] = q.grad.numpy()
        bwd[f"{key}_dk"] = k.grad.numpy()
        bwd[f"{key}_dv"] = v.grad.numpy()
    for causal in (False, True):
        gen = torch.Generator().manual_seed(99 + int(causal))
        Z, H, N, D, rb = 1, 2, 96, 16, 32
        q0, k0, v0, do = (halfrand((Z, H, N, D), gen) for _ in range(4))
        router = rand_router(Z, H, 3, 3, 2, seed=17)
        b = build_block_lists(router, 1, is_causal=causal, sink_block=True)
        raw = halfrand((Z, H, 3, b.max_count), gen).requires_grad_(True)
        ste = raw - raw.detach()
        q, k, v = (t.clone().requires_grad_(True) for t in (q0, k0, v0))
        out = block_list_attention(q, k, v, b, route_block=rb, is_causal=causal, block_m=16,
                                   block_n=16, soft_block_bias=ste)
        out.backward(do)
        key = f"s{int(causal)}"
        for nm, t in (("q", q0), ("k", k0), ("v", v0), ("do", do)):
            bwd[f"{key}_{nm}"] = t.half().numpy()
        bwd[f"{key}_lists"] = b.lists.numpy()
        bwd[f"{key}_counts"] = b.counts.numpy()
        bwd[f"{key}_dq"] = q.grad.numpy()
        bwd[f"{key}_dk"] = k.grad.numpy()
        bwd[f"{key}_dv"] = v.grad.numpy()
        bwd[f"{key}_dbias"] = raw.grad.numpy()
    np.savez_compressed(os.path.join(out_dir, "backward.npz"), **bwd)

    # ------------------------------------------------------------------ decode
    dec = {}
    for td in (1, 3, 5, 6, 7, 10):
        gen = torch.Generator().manual_seed(100 + td)
        B, H, D, num_blocks, page = 2, 4, 16, 6, 8
        rd = min(3, td)
        q = halfrand((B, H, D), gen)
        kc = halfrand((num_blocks, H, page, D), gen)
        vc = halfrand((num_blocks, H, page, D), gen)
        bt = torch.arange(num_blocks, dtype=torch.int32).unsqueeze(0).repeat(B, 1)
        bt[1] = torch.randperm(num_blocks, generator=gen).to(torch.int32)
        ctx = torch.tensor([40, 35], dtype=torch.int32)
        ri = torch.randint(0, 2, (num_blocks, H, td), generator=gen, dtype=torch.int32)
        qri = torch.randint(0, 2, (B, H, td), generator=gen, dtype=torch.int32)
        out_k = ultrametric_decode(q, kc, vc, bt, ctx, ri, qri, req_depth=rd, local_blocks=1,
                                   sink_block=True)
        out_r = _ultrametric_decode_reference(q, kc, vc, bt, ctx, ri, qri, req_depth=rd,
                                              local_blocks=1, sink_block=True)
        key = f"d{td:02d}"
        for nm, t in (("q", q), ("k", kc), ("v", vc)):
            dec[f"{key}_{nm}"] = t.half().numpy()
        dec[f"{key}_bt"] = bt.numpy()
        dec[f"{key}_ctx"] = ctx.numpy()
        dec[f"{key}_ri"] = ri.numpy()
        dec[f"{key}_qri"] = qri.numpy()
        dec[f"{key}_meta"] = np.array([rd, 1, 1])
        dec[f"{key}_out_kernel"] = out_k.numpy()
        dec[f"{key}_out_ref"] = out_r.numpy()
    # zero-length context and no sink/local: the reference function's zeros
    gen = torch.Generator().manual_seed(5)
    B, H, D, num_blocks, page = 3, 2, 16, 8, 4
    q = halfrand((B, H, D), gen)
    kc = halfrand((num_blocks, H, page, D), gen)
    vc = halfrand((num_blocks, H, page, D), gen)
    bt = torch.stack([torch.randperm(num_blocks, generator=gen) for _ in range(B)]).to(torch.int32)
    ctx = torch.tensor([0, 13, 32], dtype=torch.int32)
    ri = torch.randint(0, 3, (num_blocks, H, 4), generator=gen, dtype=torch.int32)
    qri = torch.randint(0, 3, (B, H, 4), generator=gen, dtype=torch.int32)
    out_r = _ultrametric_decode_reference(q, kc, vc, bt, ctx, ri, qri, req_depth=1)
    for nm, t in (("q", q), ("k", kc), ("v", vc)):
        dec[f"dz_{nm}"] = t.half().numpy()
    dec["dz_bt"] = bt.numpy()
    dec["dz_ctx"] = ctx.numpy()
    dec["dz_ri"] = ri.numpy()
    dec["dz_qri"] = qri.numpy()
    dec["dz_meta"] = np.array([1, 0, 0])
    dec["dz_out_ref"] = out_r.numpy()
    np.savez_compressed(os.path.join(out_dir, "decode.npz"), **dec)
    print("wrote", sorted(os.listdir(out_dir)))


if __name__ == "__main__":
    main(sys.argv[1], os.path.dirname(os.path.abspath(__file__)))

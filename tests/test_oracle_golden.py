"""Pin the CPU oracle against outputs of the reference itself (tests/golden/*.npz).

The fixtures were produced by tests/golden/make_golden.py, which ran sparse-ai's
``build_block_lists`` / ``build_transposed_block_lists`` / Triton kernels (under the
Triton CPU interpreter) / CPU quickstart path / decode reference.  Bit-exact for lists;
fp32 kernels of the reference vs the fp64 oracle within the reference's own fp32
tolerance (1e-4 abs, tests/test_block_list.py:217,295 there).
"""

import math

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ao
from oracle import block_list_oracle as blo
from oracle import decode_oracle as do


def _builder_keys(g):
    return sorted({k.split("_")[0] for k in g})


def test_builder_golden_bit_exact(golden):
    g = golden("builder")
    keys = _builder_keys(g)
    assert len(keys) >= 40
    for key in keys:
        router = g[key + "_router"]
        depth = g[key + "_depth"]
        causal, sink, local, arity = (int(x) for x in g[key + "_flags"])
        dep = int(depth[0]) if bool(g[key + "_depth_is_int"]) else depth.tolist()
        lists, counts, mc = blo.build_block_lists(
            router, dep, is_causal=bool(causal), sink_block=bool(sink), local_blocks=local,
            arity=None if arity < 0 else arity)
        assert mc == int(g[key + "_max_count"]), key
        np.testing.assert_array_equal(counts, g[key + "_counts"], err_msg=key)
        np.testing.assert_array_equal(lists, g[key + "_lists"], err_msg=key)
        tl, tc, tmc = blo.transpose_block_lists(lists, counts, mc, router.shape[2])
        assert tmc == int(g[key + "_tmax_count"]), key
        np.testing.assert_array_equal(tc, g[key + "_tcounts"], err_msg=key)
        np.testing.assert_array_equal(tl, g[key + "_tlists"], err_msg=key)


def test_builder_mask_oracle_agrees_with_builder(golden):
    """The pairwise mask oracle and the builder restatement agree wherever ids < arity."""
    g = golden("builder")
    for key in _builder_keys(g):
        router = g[key + "_router"]
        causal, sink, local, arity = (int(x) for x in g[key + "_flags"])
        if arity >= 0 and router.max() >= arity:
            continue  # deliberately-invalid ids: only the code path defines the result
        depth = g[key + "_depth"].tolist()
        m = blo.block_mask(router, depth, is_causal=bool(causal), sink_block=bool(sink),
                           local_blocks=local)
        np.testing.assert_array_equal(m.sum(-1), g[key + "_counts"], err_msg=key)


def test_builder_code_collisions_are_reproduced(golden):
    """Sync-free builds with ids >= arity differ from the pairwise mask; the restated
    mixed-radix code reproduces the reference's (colliding) result exactly."""
    g = golden("builder")
    differs = 0
    for key in _builder_keys(g):
        router = g[key + "_router"]
        arity = int(g[key + "_flags"][3])
        if arity >= 0 and router.max() >= arity:
            m = blo.block_mask(router, g[key + "_depth"].tolist())
            differs += int((m.sum(-1) != g[key + "_counts"]).any())
    assert differs >= 1


def test_invalid_depth_raises():
    r = np.zeros((1, 2, 4, 3), dtype=np.int64)
    with pytest.raises(ValueError):
        blo.build_block_lists(r, 4)
    with pytest.raises(ValueError):
        blo.build_block_lists(r, [1, 2, 3])
    with pytest.raises(ValueError):
        blo.build_block_lists(r, 4, arity=2)
    with pytest.raises(ValueError):
        blo.build_block_lists(-np.ones((1, 1, 2, 2), dtype=np.int64), 1)


def test_tree_known_answers():
    NB = 16
    r = blo.tree_router(1, 1, NB, 4)
    for d in range(5):
        _, counts, _ = blo.build_block_lists(r, d)
        assert (counts == NB // 2 ** d).all()
    lists, counts, _ = blo.build_block_lists(r, 4)
    assert (lists[0, 0, :, 0] == np.arange(NB)).all()


def _t(a):
    return torch.from_numpy(np.asarray(a))


def test_forward_oracle_matches_reference_kernel(golden):
    g = golden("forward")
    for i in range(6):
        key = f"f{i:02d}"
        N, rb, depth, causal, sink, local = (int(x) for x in g[key + "_meta"])
        q, k, v = (_t(g[f"{key}_{n}"]).float() for n in "qkv")
        bm = blo.block_mask(g[key + "_router"], depth, is_causal=bool(causal),
                            sink_block=bool(sink), local_blocks=local)
        mask = ao.token_mask(_t(bm), rb, N, bool(causal))
        out, lse = ao.masked_attention(q, k, v, mask)
        assert (out - _t(g[key + "_out"]).double()).abs().max() < 1e-4, key
        assert (lse - _t(g[key + "_lse"]).double()).abs().max() < 1e-4, key


def test_forward_oracle_bias_and_empty_row(golden):
    g = golden("forward")
    q, k, v = (_t(g[f"fb_{n}"]).float() for n in "qkv")
    bias = _t(g["fb_bias"]).float()
    lists, counts = _t(g["fb_lists"]), _t(g["fb_counts"])
    Z, H, N, D = q.shape
    rb = 32
    NB = counts.shape[-1]
    bm = torch.zeros(Z, H, NB, NB, dtype=torch.bool)
    for h in range(H):
        for qb in range(NB):
            for t in range(int(counts[0, h, qb])):
                bm[0, h, qb, int(lists[0, h, qb, t])] = True
    mask = ao.token_mask(bm, rb, N, True)
    tb = ao.token_bias(bias, lists, counts, rb, N)
    out, lse = ao.masked_attention(q, k, v, mask, bias=tb)
    ref_out, ref_lse = _t(g["fb_out"]).double(), _t(g["fb_lse"]).double()
    assert (out - ref_out).abs().max() < 1e-4
    fin = torch.isfinite(ref_lse)
    assert torch.equal(fin, torch.isfinite(lse))
    assert (lse[fin] - ref_lse[fin]).abs().max() < 1e-4
    assert (ref_out[0, 1, 64:96] == 0).all() and torch.isinf(ref_lse[0, 1, 64:96]).all()


def test_quickstart_cpu_path_golden(golden):
    g = golden("forward")
    q, k, v = (_t(g[f"qs_{n}"]).float() for n in "qkv")
    router = g["qs_router"].astype(np.int64)
    Z, H, N, D = q.shape
    full = np.concatenate([router, np.zeros((Z, H, 1, router.shape[-1]), np.int64)], axis=2)
    for causal in (0, 1):
        bm = blo.block_mask(full, 2, is_causal=bool(causal))
        out, lse = ao.masked_attention(q, k, v, ao.token_mask(_t(bm), 128, N, bool(causal)))
        assert (out - _t(g[f"qs{causal}_out"]).double()).abs().max() < 1e-4
        assert (lse - _t(g[f"qs{causal}_lse"]).double()).abs().max() < 1e-4


def test_backward_oracle_matches_reference_kernels(golden):
    g = golden("backward")
    for i in range(3):
        key = f"g{i:02d}"
        N, rb, depth, causal, sink, local = (int(x) for x in g[key + "_meta"])
        q, k, v, dout = (_t(g[f"{key}_{n}"]).float() for n in ("q", "k", "v", "do"))
        lists, counts = _t(g[key + "_lists"]), _t(g[key + "_counts"])
        NB = counts.shape[-1]
        bm = torch.zeros(1, 2, NB, NB, dtype=torch.bool)
        for h in range(2):
            for qb in range(NB):
                for t in range(int(counts[0, h, qb])):
                    bm[0, h, qb, int(lists[0, h, qb, t])] = True
        mask = ao.token_mask(bm, rb, N, bool(causal))
        res = ao.masked_attention_grads(q, k, v, mask, dout)
        for name in ("dq", "dk", "dv"):
            assert (res[name] - _t(g[f"{key}_{name}"]).double()).abs().max() < 1e-4, (key, name)


def test_soft_bias_gradient_oracle(golden):
    g = golden("backward")
    for causal in (0, 1):
        key = f"s{causal}"
        q, k, v, dout = (_t(g[f"{key}_{n}"]).float() for n in ("q", "k", "v", "do"))
        lists, counts = _t(g[key + "_lists"]), _t(g[key + "_counts"])
        Z, H, N, D = q.shape
        NB, MC = counts.shape[-1], lists.shape[-1]
        bm = torch.zeros(Z, H, NB, NB, dtype=torch.bool)
        for h in range(H):
            for qb in range(NB):
                for t in range(int(counts[0, h, qb])):
                    bm[0, h, qb, int(lists[0, h, qb, t])] = True
        mask = ao.token_mask(bm, 32, N, bool(causal))
        res = ao.masked_attention_grads(q, k, v, mask, dout, block_bias=torch.zeros(Z, H, NB, MC),
                                        lists=lists, counts=counts, route_block=32)
        assert (res["d_bias"] - _t(g[key + "_dbias"]).double()).abs().max() < 1e-4
        for name in ("dq", "dk", "dv"):
            assert (res[name] - _t(g[f"{key}_{name}"]).double()).abs().max() < 1e-4


def test_decode_oracle_matches_reference(golden):
    g = golden("decode")
    for td in (1, 3, 5, 6, 7, 10):
        key = f"d{td:02d}"
        rd, local, sink = (int(x) for x in g[key + "_meta"])
        args = [_t(g[f"{key}_{n}"]) for n in ("q", "k", "v", "bt", "ctx", "ri", "qri")]
        args[:3] = [a.float() for a in args[:3]]
        out = do.ultrametric_decode_reference(*args, rd, local_blocks=local, sink_block=bool(sink),
                                              compute_dtype=torch.float64)
        assert (out - _t(g[key + "_out_ref"]).double()).abs().max() < 1e-5, key
        assert (out - _t(g[key + "_out_kernel"]).double()).abs().max() < 1e-4, key
    args = [_t(g[f"dz_{n}"]) for n in ("q", "k", "v", "bt", "ctx", "ri", "qri")]
    args[:3] = [a.float() for a in args[:3]]
    out = do.ultrametric_decode_reference(*args, 1, compute_dtype=torch.float64)
    assert (out - _t(g["dz_out_ref"]).double()).abs().max() < 1e-5
    assert (out[0] == 0).all()

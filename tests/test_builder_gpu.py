"""GPU parity of the compaction kernels (bit-exact).

* every builder fixture produced by the reference (tests/golden/builder.npz): sync path,
  sync-free ``arity=`` path (incl. ids >= arity, where the reference's mixed-radix codes
  collide), per-level overflow path, tree routing, per-head thresholds;
* the transposed lists of each fixture;
* larger seeded cases at the BASELINE sizes (C2: NB=64, C5: NB=1024) against the numpy
  oracle;
* known answers of tests/test_block_list.py:131-183 of the reference.
"""

import numpy as np
import pytest
import torch

from helpers import random_router, tree_router
from oracle import block_list_oracle as blo
from ultrametric import (BlockLists, build_block_lists, build_block_lists_from_mask,
                         build_transposed_block_lists)

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _keys(g):
    return sorted({k.split("_")[0] for k in g})


def test_builder_matches_reference_fixtures(golden):
    g = golden("builder")
    for key in _keys(g):
        router = torch.from_numpy(g[key + "_router"]).to(DEV)
        causal, sink, local, arity = (int(x) for x in g[key + "_flags"])
        depth = g[key + "_depth"]
        dep = int(depth[0]) if bool(g[key + "_depth_is_int"]) else depth.tolist()
        for rdtype in (torch.int64, torch.int32):
            bl = build_block_lists(router.to(rdtype), dep, is_causal=bool(causal), sink_block=bool(sink),
                                   local_blocks=local, arity=None if arity < 0 else arity)
            assert bl.lists.dtype == torch.int32 and bl.counts.dtype == torch.int32
            assert bl.max_count == int(g[key + "_max_count"]), key
            np.testing.assert_array_equal(bl.counts.cpu().numpy(), g[key + "_counts"], err_msg=key)
            np.testing.assert_array_equal(bl.lists.cpu().numpy(), g[key + "_lists"], err_msg=key)
        t = build_transposed_block_lists(bl, num_key_blocks=router.shape[2])
        assert t.max_count == int(g[key + "_tmax_count"]), key
        np.testing.assert_array_equal(t.counts.cpu().numpy(), g[key + "_tcounts"], err_msg=key)
        np.testing.assert_array_equal(t.lists.cpu().numpy(), g[key + "_tlists"], err_msg=key)


@pytest.mark.parametrize("Z,H,NB,TD,depth,causal,sink,local", [
    (1, 32, 64, 6, [1, 2, 3, 4, 5, 6] * 5 + [1, 2], True, True, 0),    # C2 thresholds
    (1, 32, 64, 6, 6, False, False, 0),                                 # C2 98.4% row
    (1, 16, 1024, 10, 7, True, True, 1),                                # C5
    (2, 3, 300, 9, [2, 5, 9], False, True, 3),
])
def test_builder_large_vs_oracle(Z, H, NB, TD, depth, causal, sink, local):
    router = tree_router(Z, H, NB, TD)
    lists, counts, mc = blo.build_block_lists(router.numpy(), depth, is_causal=causal,
                                              sink_block=sink, local_blocks=local, arity=2)
    bl = build_block_lists(router.to(DEV), depth, is_causal=causal, sink_block=sink,
                           local_blocks=local, arity=2)
    assert bl.max_count == mc == NB
    np.testing.assert_array_equal(bl.counts.cpu().numpy(), counts)
    np.testing.assert_array_equal(bl.lists.cpu().numpy(), lists)
    rnd = random_router(Z, H, NB, TD, 3, seed=NB)
    l2, c2, m2 = blo.build_block_lists(rnd.numpy(), depth, is_causal=causal, sink_block=sink,
                                       local_blocks=local)
    b2 = build_block_lists(rnd.to(DEV), depth, is_causal=causal, sink_block=sink, local_blocks=local)
    assert b2.max_count == m2
    np.testing.assert_array_equal(b2.counts.cpu().numpy(), c2)
    np.testing.assert_array_equal(b2.lists.cpu().numpy(), l2)
    if NB <= 300:
        tl, tc, tm = blo.transpose_block_lists(l2, c2, m2, NB)
        t = build_transposed_block_lists(b2)
        assert t.max_count == tm
        np.testing.assert_array_equal(t.counts.cpu().numpy(), tc)
        np.testing.assert_array_equal(t.lists.cpu().numpy(), tl)


def test_known_answers():
    router = random_router(1, 2, 9, 3, 2, seed=1).to(DEV)
    for causal in (False, True):
        bl = build_block_lists(router, 3, is_causal=causal)
        for h in range(2):
            for i in range(9):
                c = int(bl.counts[0, h, i])
                assert i in bl.lists[0, h, i, :c].tolist()
    r = random_router(1, 2, 5, 3, 2).to(DEV)
    assert torch.all(build_block_lists(r, 0).counts == 5)
    assert torch.equal(build_block_lists(r, 0, is_causal=True).counts[0, 0].cpu(),
                       torch.arange(1, 6, dtype=torch.int32))
    NB = 16
    tr = tree_router(1, 1, NB, 4).to(DEV)
    assert torch.all(build_block_lists(tr, 4).counts == 1)
    for d in range(5):
        assert torch.all(build_block_lists(tr, d).counts == NB // 2 ** d)


def test_sync_free_padding_is_zero():
    r = random_router(2, 2, 9, 3, 2, seed=7).to(DEV)
    b = build_block_lists(r, 1, is_causal=True, sink_block=True, arity=2)
    assert b.max_count == 9 and b.lists.shape[-1] == 9
    for z in range(2):
        for h in range(2):
            for i in range(9):
                c = int(b.counts[z, h, i])
                assert (b.lists[z, h, i, c:] == 0).all()


def test_mask_entry_point():
    g = torch.Generator().manual_seed(0)
    m = torch.rand(2, 3, 37, 37, generator=g) < 0.3
    bl = build_block_lists_from_mask(m.to(DEV), sync_free=False)
    lists, counts = blo._compact(m.numpy(), int(m.sum(-1).max()))
    np.testing.assert_array_equal(bl.counts.cpu().numpy(), counts)
    np.testing.assert_array_equal(bl.lists.cpu().numpy(), lists)
    assert bl.max_count == int(m.sum(-1).max())


def test_empty_and_degenerate_shapes():
    r = torch.zeros(1, 2, 0, 3, dtype=torch.int32, device=DEV)
    b = build_block_lists(r, 1)
    assert b.max_count == 0 and b.lists.shape == (1, 2, 0, 0)
    t = build_transposed_block_lists(BlockLists(torch.zeros(1, 1, 3, 0, dtype=torch.int32, device=DEV),
                                                torch.zeros(1, 1, 3, dtype=torch.int32, device=DEV), 0))
    assert t.max_count == 0 and t.lists.shape == (1, 1, 3, 0)

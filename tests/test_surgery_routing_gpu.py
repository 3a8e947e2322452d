"""GPU parity of ``build_block_lists_from_assignments`` (sa_build_block_lists_from_assignments:
the per-block vote kernel + the compaction kernel) against the reference's own outputs
(tests/golden/surgery_routing.npz, from sparse-ai's ``_block_list_prefill``) and the CPU
oracle at the C4 size.  Integer work: block routes, lists and counts must be bit-exact."""

import numpy as np
import pytest
import torch

from oracle import block_list_oracle as blo
from oracle import surgery_oracle as so
from ultrametric import _native as nat
from ultrametric.surgery_routing import build_block_lists_from_assignments

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("key", [f"s{i:02d}" for i in range(8)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_reference_fixtures(golden, key, dtype):
    g = golden("surgery_routing")
    S, rb, r, p, local, causal, sink, arity, block = (int(x) for x in g[key + "_meta"])
    a = torch.from_numpy(g[key + "_assign"])
    if dtype == torch.bfloat16:
        # bf16 rounding can create new ties inside a token's branches; keep the fp32 argmax
        # by scaling the winner up before the cast
        win = torch.nn.functional.one_hot(a.argmax(-1), p).bool()
        a = torch.where(win, a + 1.0, a)
    a = a.to(dtype).to(DEV)
    if block:
        tok = a.repeat_interleave(rb, dim=2)[:, :, :S]
        bl, route = build_block_lists_from_assignments(tok, r, S, route_block=rb, block_assignments=a,
                                                       local_blocks=local, arity=arity,
                                                       is_causal=bool(causal), sink_block=bool(sink),
                                                       return_routes=True)
    else:
        bl, route = build_block_lists_from_assignments(a, r, S, route_block=rb, local_blocks=local,
                                                       arity=arity, is_causal=bool(causal),
                                                       sink_block=bool(sink), return_routes=True)
    assert np.array_equal(route.cpu().numpy(), g[key + "_route"]), key
    assert np.array_equal(bl.counts.cpu().numpy(), g[key + "_counts"]), key
    assert np.array_equal(bl.lists.cpu().numpy(), g[key + "_lists"]), key


def test_c4_size_vs_oracle_strided_and_per_head_depth():
    """C4's routing per layer (batch 4, 4 heads, N=32768, levels 8, p=2, r=4, per-head depth
    3/4/4/4, route block 128, one local block) from router outputs stored (B, S, H, L, p)
    and viewed as (B, H, S, L, p); and a partial last block (S = 32768 - 77)."""
    g = torch.Generator().manual_seed(44)
    for S in (32768, 32768 - 77):
        raw = torch.randn(4, S, 4, 8, 2, generator=g).to(torch.bfloat16)
        a = raw.permute(0, 2, 1, 3, 4)  # non-contiguous view
        depth = [3, 4, 4, 4]
        bl, route = build_block_lists_from_assignments(raw.to(DEV).permute(0, 2, 1, 3, 4),
                                                       4, route_block=128, req_depth=depth,
                                                       local_blocks=1, arity=2, return_routes=True)
        want_route = so.majority_routes(a.float().numpy(), 4, 128)
        assert np.array_equal(route.cpu().numpy(), want_route)
        lists, counts, _ = blo.build_block_lists(want_route, depth, is_causal=True, sink_block=True,
                                                 local_blocks=1, arity=2)
        assert np.array_equal(bl.counts.cpu().numpy(), counts)
        assert np.array_equal(bl.lists.cpu().numpy(), lists)
    assert nat.read_device_status() == 0


def test_three_branch_ties_and_r_zero():
    # p = 3, level 0 votes 11 : 11 : 10 in every block: the tie goes to the lowest branch id
    S, rb = 96, 32
    a = torch.zeros(1, 2, S, 2, 3)
    a[..., 0, :] = torch.nn.functional.one_hot((torch.arange(S) % 32) // 11, 3).float().view(1, 1, S, 3)
    a[..., 1, :] = torch.nn.functional.one_hot(torch.full((S,), 2), 3).float().view(1, 1, S, 3)
    bl, route = build_block_lists_from_assignments(a.to(DEV), 2, route_block=rb, arity=3,
                                                   return_routes=True)
    want = so.majority_routes(a.numpy(), 2, rb)
    assert np.array_equal(route.cpu().numpy(), want)
    # r = 0: every earlier block matches (dense causal)
    bl0 = build_block_lists_from_assignments(a.to(DEV), 0, route_block=rb, arity=3)
    assert bl0.counts.cpu().tolist() == [[[1, 2, 3], [1, 2, 3]]]

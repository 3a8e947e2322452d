"""The surgery routing oracle against the reference's own outputs
(tests/golden/surgery_routing.npz, made by tests/golden/make_golden_surgery.py running
``SurgicalLlamaAttention._block_list_prefill`` of sparse-ai): block routes and lists
bit-exact, including vote ties, partial last blocks, three branches and block-level
assignments; and the cross-layer list cache of surgery.py:301-315 / 377-391."""

import numpy as np
import pytest

from oracle import block_list_oracle as blo
from oracle import surgery_oracle as so

CASES = [f"s{i:02d}" for i in range(8)]


@pytest.mark.parametrize("key", CASES)
def test_oracle_routes_and_lists_match_reference(golden, key):
    g = golden("surgery_routing")
    S, rb, r, p, local, causal, sink, arity, block = (int(x) for x in g[key + "_meta"])
    a = g[key + "_assign"]
    route = so.block_level_routes(a, r) if block else so.majority_routes(a, r, rb, S)
    assert np.array_equal(route, g[key + "_route"]), key
    lists, counts, _ = blo.build_block_lists(route, r, is_causal=bool(causal), sink_block=bool(sink),
                                             local_blocks=local, arity=arity)
    assert np.array_equal(counts, g[key + "_counts"]), key
    assert np.array_equal(lists, g[key + "_lists"]), key


def test_vote_ties_go_to_lowest_branch():
    a = np.zeros((1, 1, 4, 1, 3), dtype=np.float32)
    a[0, 0, [0, 1], 0, 2] = 1.0  # two tokens vote 2
    a[0, 0, [2, 3], 0, 1] = 1.0  # two vote 1
    assert so.majority_routes(a, 1, 4)[0, 0, 0, 0] == 1


def test_route_cache_reuses_anchor_lists():
    from ultrametric.surgery_routing import RouteListCache
    cache = RouteListCache(stride=3)
    assert cache.anchor(0) == 0 and cache.anchor(4) == 3 and cache.anchor(5) == 3
    key = dict(num_heads=2, head_dim=32, batch=1, seq_len=100)
    assert cache.lookup(1, **key) is None
    cache.store(0, "lists-0", **key)
    assert cache.lookup(1, **key) == "lists-0"
    assert cache.lookup(2, **key) == "lists-0"
    assert cache.lookup(0, **key) is None       # an anchor layer always routes itself
    assert cache.lookup(3, **key) is None       # a new anchor
    assert cache.lookup(1, num_heads=2, head_dim=32, batch=1, seq_len=101) is None  # length changed
    cache.store(4, "not-an-anchor", **key)      # only anchors are stored
    assert cache.lookup(5, **key) is None
    assert RouteListCache(stride=1).lookup(1, **key) is None

"""GPU checks of the paged K/V cache writer (``sa_paged_kv_append``) and of decoding from the
cache it fills: K/V rows and tail-page routes land exactly where the block tables say
(byte-exact copies), context lengths advance, an unassigned page is skipped with a status
bit, and ``ultrametric_decode`` over the cache matches the CPU oracle (2e-2 abs + 1e-2 rel)."""

import pytest
import torch

from helpers import assert_half_close
from oracle import decode_oracle as dor
from ultrametric import _native as nat
from ultrametric.paged import PagedKVCache

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _cache(page=64, Hkv=2, H=8, D=128, TD=6, reqs=3):
    return PagedKVCache(num_pages=64, num_kv_heads=Hkv, page_size=page, head_dim=D, num_heads=H,
                        tree_depth=TD, max_requests=reqs, max_pages_per_request=16, device=DEV)


def test_prefill_append_decode_matches_oracle():
    g = torch.Generator().manual_seed(3)
    c = _cache()
    Hkv, H, D, TD, page = 2, 8, 128, 6, 64
    lens = [70, 128, 5]
    dense_k, dense_v = [], []
    for rid, S in enumerate(lens):
        c.add_request(rid)
        k = torch.randn(S, Hkv, D, generator=g).bfloat16()
        v = torch.randn(S, Hkv, D, generator=g).bfloat16()
        routes = torch.randint(0, 2, (-(-S // page), H, TD), generator=g, dtype=torch.int32)
        c.prefill(rid, k.to(DEV), v.to(DEV), routes.to(DEV))
        dense_k.append(k)
        dense_v.append(v)
    # several decode steps: append one token per request (with its tail-page route), decode
    for step in range(70):
        kn = torch.randn(3, Hkv, D, generator=g).bfloat16()
        vn = torch.randn(3, Hkv, D, generator=g).bfloat16()
        tr = torch.randint(0, 2, (3, H, TD), generator=g, dtype=torch.int32)
        c.append(range(3), kn.to(DEV), vn.to(DEV), tr.to(DEV))
        for rid in range(3):
            dense_k[rid] = torch.cat([dense_k[rid], kn[rid:rid + 1]])
            dense_v[rid] = torch.cat([dense_v[rid], vn[rid:rid + 1]])
        lens = [n + 1 for n in lens]
        # the new token's page got this step's route
        for rid in range(3):
            phys = c.alloc.pages[rid][(lens[rid] - 1) // page]
            assert torch.equal(c.router[phys].cpu(), tr[rid])
    torch.cuda.synchronize()
    assert c.context_lens.cpu().tolist() == lens
    # every token's K/V row sits at (block_tables[rid][pos // page], pos % page), byte-exact
    for rid in range(3):
        pages = c.alloc.pages[rid]
        got_k = torch.cat([c.k_cache[p].cpu().transpose(0, 1) for p in pages])[:lens[rid]]
        got_v = torch.cat([c.v_cache[p].cpu().transpose(0, 1) for p in pages])[:lens[rid]]
        assert torch.equal(got_k, dense_k[rid]) and torch.equal(got_v, dense_v[rid])
    q = torch.randn(3, H, D, generator=g).bfloat16()
    qr = torch.randint(0, 2, (3, H, TD), generator=g, dtype=torch.int32)
    out = c.decode(q.to(DEV), qr.to(DEV), 2, range(3), local_blocks=1, sink_block=True)
    ref = dor.ultrametric_decode_reference(q.float(), c.k_cache.float().cpu(), c.v_cache.float().cpu(),
                                           c.block_tables.cpu(), c.context_lens.cpu(), c.router.cpu(),
                                           qr, 2, local_blocks=1, sink_block=True,
                                           compute_dtype=torch.float64)
    assert_half_close(out, ref, "decode from the paged cache")
    assert nat.read_device_status() == 0


def test_append_without_page_is_skipped_and_flagged():
    c = _cache(reqs=1)
    c.add_request(0)
    # bypass the allocator: block table row 0 is empty (page id 0 is valid, so point it out of range)
    c.block_tables[0, 0] = 10_000
    k = torch.zeros(1, 2, 128, dtype=torch.bfloat16, device=DEV)
    nat.check(nat.lib().sa_paged_kv_append(
        nat.SA_BF16, 1, 2, 128, 64, c.k_cache.shape[0], k.data_ptr(), nat.strides(k), k.data_ptr(),
        nat.strides(k), c.block_tables.data_ptr(), nat.strides(c.block_tables), c.block_tables.shape[1],
        c.context_lens.data_ptr(), c.k_cache.data_ptr(), nat.strides(c.k_cache), c.v_cache.data_ptr(),
        nat.strides(c.v_cache), None, 0, None, 8, 6, c.router.data_ptr(), nat.SA_I32,
        nat.strides(c.router), torch.cuda.current_stream().cuda_stream), "append")
    torch.cuda.synchronize()
    assert c.context_lens.cpu().tolist() == [0]
    assert nat.read_device_status(reset=True) == 2
    assert nat.read_device_status() == 0

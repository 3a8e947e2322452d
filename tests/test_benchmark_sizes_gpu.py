"""Parity at the sizes bench.py measures: the exact C2, C3 and C5 inputs of the benchmark
(built by bench.py's own constructors), checked against the CPU oracle.

* C2 backward at full size (N=8192, H=32/8, D=128, RB=128, bf16, the seeded per-head
  threshold mix, causal + sink): dQ / dK / dV of two whole GQA groups (8 query heads), with
  and without the zero-valued straight-through soft-block bias (whose gradient is checked
  too), and the 98.4 % sweep point (threshold 6, non-causal, no sink).
* C3: the full 64-request decode batch, checked on 8 requests spread over it.
* C5: the N=131072 forward on one GPU, two heads, three query-row windows.

Tolerances (from the north star): bf16 outputs and gradients within 2e-2 abs + 1e-2 rel.
For the gradients that yardstick is an oracle with the reference kernels' rounding points
(P and scale*dS rounded to bf16 before their products, Delta from the bf16 output:
src/ultrametric/block_list.py:565-580, 652-680, 785).  The sink key block is listed by all
64 query blocks of the 4 heads of a group, so its dK/dV sum 32768 rounded terms; against
exact arithmetic the gradients are held to twice the tolerance (4e-2 abs + 2e-2 rel).
"""

import pytest
import torch

import bench
from helpers import assert_half_close, lse_close
from oracle import attention_oracle as ao
from oracle import block_list_oracle as blo
from oracle import decode_oracle as dor
from ultrametric import BlockLists, block_list_attention, build_block_lists

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _c2_block_mask(router, t_heads, causal, sink):
    return torch.from_numpy(blo.block_mask(router.cpu().numpy(), t_heads, is_causal=causal,
                                           sink_block=sink))


@pytest.mark.parametrize("mix,with_bias", [("seeded", False), ("seeded", True), ("98.4%", False)])
def test_c2_full_size_backward(mix, with_bias):
    C2 = bench.C2
    if mix == "seeded":
        t_heads, causal, sink = bench.c2_thresholds(0), True, True
    else:
        t_heads, causal, sink = [6] * C2["H"], False, False
    prob = bench.C2Problem(torch.device(DEV), 0, t_heads, causal=causal, sink=sink)
    RB = C2["RB"]
    bl = BlockLists(prob.lists, prob.counts, prob.lists.shape[-1])
    q, k, v = (t.detach().clone().requires_grad_(True) for t in (prob.q, prob.k, prob.v))
    raw = torch.zeros(bl.lists.shape, device=DEV, requires_grad=True) if with_bias else None
    ste = (raw - raw.detach()) if with_bias else None
    out = block_list_attention(q, k, v, bl, route_block=RB, is_causal=causal, soft_block_bias=ste)
    out.backward(prob.do)
    torch.cuda.synchronize()

    kv_heads = [0, 5]
    bm = _c2_block_mask(prob.router, t_heads, causal, sink)
    args = (prob.h_q, prob.h_k, prob.h_v, bm, RB, causal, prob.h_do)
    exact = ao.masked_attention_grads_chunked(*args, kv_heads=kv_heads, chunk=1024,
                                              compute_dtype=torch.float32)
    lowp = ao.masked_attention_grads_chunked(*args, kv_heads=kv_heads, chunk=1024,
                                             io_dtype=torch.bfloat16, compute_dtype=torch.float32)
    heads = exact["heads"]
    assert_half_close(out[:, heads], exact["out"], "C2 out")
    for name, got, sel in (("dq", q.grad, heads), ("dk", k.grad, kv_heads), ("dv", v.grad, kv_heads)):
        g = got[:, sel]
        assert_half_close(g, lowp[name], f"C2 {name} vs reference rounding")
        assert_half_close(g, exact[name], f"C2 {name} vs exact", abs_tol=4e-2, rel_tol=2e-2)
    if with_bias:
        # d_bias[z, h, qb, t] = unscaled dS summed over the block pair (qb, lists[qb, t])
        lists = prob.lists.cpu()[:, heads].long()
        counts = prob.counts.cpu()[:, heads]
        want = torch.gather(exact["dbias_blocks"], -1, lists)
        slot = torch.arange(lists.shape[-1]).view(1, 1, 1, -1)
        want = torch.where(slot < counts.unsqueeze(-1), want, torch.zeros_like(want))
        got = raw.grad.cpu()[:, heads].double()
        err = (got - want.double()).abs().max().item()
        assert err <= 2e-2 * max(1.0, want.abs().max().item()), f"C2 d_bias err {err}"
    assert int(bench_status()) == 0


def bench_status():
    from ultrametric import _native as nat
    return nat.read_device_status()


def test_c3_full_batch_decode():
    c3 = bench.make_c3(torch.device(DEV), 0)
    out = bench.c3_decode(c3)
    torch.cuda.synchronize()
    reqs = [0, 9, 18, 27, 36, 45, 54, 63]
    sub = bench.c3_host_subset(c3, reqs)
    ref = dor.ultrametric_decode_reference(sub["q"].float(), sub["kc"].float(), sub["vc"].float(),
                                           sub["bt"], sub["ctx"], sub["ri"], sub["qri"],
                                           bench.C3["req_depth"],
                                           local_blocks=bench.C3["local_blocks"],
                                           sink_block=bench.C3["sink_block"],
                                           compute_dtype=torch.float64)
    assert out.shape == (64, 32, 128)
    assert torch.isfinite(out).all()
    assert_half_close(out[reqs], ref, "C3 decode (64-request batch)")
    assert int(bench_status()) == 0


def test_c5_full_length_forward():
    c5 = bench.make_c5(torch.device(DEV))
    C5 = bench.C5
    N, RB = C5["N"], C5["RB"]
    out, lse = block_list_attention(c5["q"], c5["k"], c5["v"], c5["bl"], route_block=RB,
                                    is_causal=True, return_lse=True)
    torch.cuda.synchronize()
    assert int(c5["bl"].counts.sum()) == 5624 * C5["H"]
    heads = [0, 9]
    bm = torch.from_numpy(blo.block_mask(c5["router"][:, heads].numpy(), C5["t"], is_causal=True,
                                         sink_block=True))
    ranges = [(0, 1024), (65536, 66560), (N - 1024, N)]
    g = C5["H"] // C5["Hkv"]
    q = c5["q"][:, heads].float().cpu()
    kv_idx = [h // g for h in heads]
    k = c5["k"][:, kv_idx].float().cpu()
    v = c5["v"][:, kv_idx].float().cpu()
    # the sliced K/V hold one KV head per selected query head (group size 1 here)
    ref, ref_lse = ao.masked_attention_chunked(q, k, v, bm, RB, True, chunk=1024,
                                               row_ranges=ranges)
    for a, b in ranges:
        assert_half_close(out[:, heads, a:b], ref[:, :, a:b], f"C5 out rows {a}:{b}")
        lse_close(lse[:, heads, a:b], ref_lse[:, :, a:b], 2e-2)
    assert int(bench_status()) == 0

"""Benchmark of the B200 block-sparse attention path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload: block-sparse prefill forward+backward, bf16,
B=1, 32 query heads / 8 KV heads (GQA), D=128, N=8192, route block 128 (64x64 block grid),
tree routing of depth 6 with a per-head LCA threshold drawn from {1..6} (seeded), causal,
sink block kept.  A step = build the block lists + forward + backward (Delta/transposed
lists, dQ, dK/dV), each a C-ABI launch timed with CUDA events on the launching stream;
L2 is flushed (a 256 MiB write) between steps, outside the events.  ``value`` is kept-block
TFLOP/s: kept (query block, key block) pairs x (4 + 10) * RB^2 * D / step time.

Also reported: ``e2e`` (same metric through the public ``block_list_attention`` autograd API
with pinned host buffers, H2D of q/k/v/dO and D2H of out/dq/dk/dv inside the timed region),
the 50 / 90 / 98.4 % sparsity sweep with dense SDPA beside it, the C3 routed paged decode
(tok/s and GB/s of routed bytes), the roofline of the dominant kernel, sampled SM clocks,
and the reference's CPU path (masked dense fp32 attention) timed on a bounded head sample.

Multi-GPU (torchrun, one rank per GPU): each rank runs its own C2 head group and its own 64
decode requests, no data-path collective (weak scaling); times are the max over ranks.
``--impl reference`` times the reference's CPU path alone (rank 0; other ranks exit).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "sparse-ai_b200"))

import torch  # noqa: E402

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# C2 configuration
C2 = dict(Z=1, H=32, Hkv=8, N=8192, D=128, RB=128, TD=6)


# ---------------------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------------------

def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def tree_router(Z, H, NB, TD):
    depth = max(1, math.ceil(math.log2(max(NB, 2))))
    r = torch.zeros(Z, H, NB, TD, dtype=torch.int32)
    for d in range(min(depth, TD)):
        r[:, :, :, d] = (torch.arange(NB) >> (depth - 1 - d)) % 2
    return r


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.samples = []
        if self.proc is None:
            return False
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)
        return False

    def summary(self):
        if not getattr(self, "samples", None):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[5 + i] == "Active"})
        loaded = [x for x in sm if x > 500] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


def max_over_ranks(values, world, device):
    """Elementwise max over the ranks of per-rank device timings (ms): with weak scaling the
    job takes as long as its slowest rank.  A no-op for one rank."""
    vals = [float(v) for v in values]
    if world <= 1:
        return vals
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus and world > 1:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    return world, rank, local


# ---------------------------------------------------------------------------------------
# the reference's CPU path (bounded sample), used by cpu_baseline and --impl reference
# ---------------------------------------------------------------------------------------

def c2_masks(t_heads, causal, sink):
    from oracle import block_list_oracle as blo
    H, NB, TD = C2["H"], C2["N"] // C2["RB"], C2["TD"]
    router = tree_router(1, H, NB, TD).numpy()
    return torch.from_numpy(blo.block_mask(router, t_heads, is_causal=causal, sink_block=sink))


def c2_thresholds(seed=0):
    g = torch.Generator().manual_seed(1000 + seed)
    return torch.randint(1, 7, (C2["H"],), generator=g).tolist()


def cpu_reference_sample(heads=(0, 1), causal=True, sink=True, seed=0, t_heads=None):
    """Masked dense fp32 attention forward + autograd backward on the CPU for a head subset
    of C2 (query-chunked, benchmarks/benchmark_block_list.py:106-123 of the reference).
    Returns (seconds, n_heads)."""
    from oracle import attention_oracle as ao
    N, D, RB = C2["N"], C2["D"], C2["RB"]
    t_heads = t_heads if t_heads is not None else c2_thresholds(seed)
    bm = c2_masks(t_heads, causal, sink)
    gen = torch.Generator().manual_seed(seed)
    group = C2["H"] // C2["Hkv"]
    kv_heads = sorted({h // group for h in heads})
    q = torch.randn(1, len(heads), N, D, generator=gen).bfloat16().float().requires_grad_(True)
    k = torch.randn(1, len(kv_heads), N, D, generator=gen).bfloat16().float().requires_grad_(True)
    v = torch.randn(1, len(kv_heads), N, D, generator=gen).bfloat16().float().requires_grad_(True)
    do = torch.randn(1, len(heads), N, D, generator=gen).bfloat16().float()
    bm_sub = bm[:, list(heads)]
    t0 = time.perf_counter()
    outs = []
    for hi, h in enumerate(heads):
        kh = kv_heads.index(h // group)
        o, _ = ao.masked_attention_chunked(q[:, hi:hi + 1], k[:, kh:kh + 1], v[:, kh:kh + 1],
                                           bm_sub[:, hi:hi + 1], RB, causal, chunk=2048,
                                           compute_dtype=torch.float32)
        outs.append(o)
    out = torch.cat(outs, dim=1)
    out.backward(do)
    t1 = time.perf_counter()
    return t1 - t0, len(heads)


def kept_flops_c2(t_heads, causal, sink, fwd=True, bwd=True, heads=None):
    bm = c2_masks(t_heads, causal, sink)
    if heads is not None:
        bm = bm[:, list(heads)]
    kept = int(bm.sum())
    RB, D = C2["RB"], C2["D"]
    per = (4 if fwd else 0) + (10 if bwd else 0)
    return kept, kept * per * RB * RB * D


def run_reference_arm(args):
    """The reference's CPU path of the headline step, timed on this box's host cores.  A step
    is a bounded sample of C2 -- 2 of the 32 heads, full N=8192, masked dense fp32 forward +
    autograd backward -- so every timed step is real work; value is the kept-block TFLOP/s
    of that sample (the same rate the whole problem would run at, since the masked dense
    path's cost is the same for every head)."""
    world, rank, _ = dist_setup(args.gpus)
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    t_heads = c2_thresholds(0)
    kept, flops = kept_flops_c2(t_heads, True, True)
    heads = (0, 1)
    kept_h, flops_h = kept_flops_c2(t_heads, True, True, heads=heads)
    for _ in range(args.warmup):
        cpu_reference_sample(heads, t_heads=t_heads)
    times = []
    for _ in range(args.steps):
        s, nh = cpu_reference_sample(heads, t_heads=t_heads)
        times.append(s)
    step = statistics.mean(times)
    value = flops_h / step / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_c2(args.gpus, t_heads, kept),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": "port", "measured_s": round(step, 4), "scale": 1,
                         "sample_heads": list(heads), "sample_kept_blocks": kept_h,
                         "sample_flops": flops_h,
                         "whole_step_s_extrapolated": round(step * flops / flops_h, 3),
                         "sample": f"one step = masked dense fp32 attention fwd+bwd (autograd) on "
                                   f"heads {list(heads)} of C2, full N=8192; value = the sample's "
                                   f"kept-block FLOPs / its measured time"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


METRIC = "sparse prefill fwd+bwd kept-block TFLOP/s (C2 bf16 N=8192 H=32/8 D=128)"


def config_c2(n_gpus, t_heads, kept):
    NB = C2["N"] // C2["RB"]
    return {"workload": "C2 block-sparse prefill fwd+bwd, tree routes depth 6, per-head LCA "
                        "threshold ~U{1..6}, causal + sink",
            "batch_per_gpu": 1, "heads": C2["H"], "kv_heads": C2["Hkv"], "seq_len": C2["N"],
            "head_dim": C2["D"], "route_block": C2["RB"], "thresholds": t_heads,
            "kept_blocks": kept,
            "sparsity_full_grid": 1 - kept / (C2["H"] * NB * NB),
            "sparsity_causal": 1 - kept / (C2["H"] * NB * (NB + 1) / 2),
            "parallelism": f"heads sharded, {n_gpus} x (32 q / 8 kv heads), no collective",
            "l2": "flushed between steps (256 MiB write)",
            "flops_per_kept_pair": "fwd 4*RB^2*D + bwd 10*RB^2*D"}


# ---------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------

class C2Problem:
    """Device-resident C2 inputs and the direct C-ABI step (build, fwd, bwd phases).

    ``kv_groups`` (default: all 8) selects the KV heads this problem holds, with their 4
    query heads each -- the strong-scaling split of C2's heads over GPUs.  The inputs are
    always drawn for the whole C2 problem from the seed, then sliced, so every split sees
    the same numbers."""

    def __init__(self, dev, seed, t_heads, causal=True, sink=True, kv_groups=None, fused=True):
        from ultrametric import _native as nat
        self.nat = nat
        self.dev = dev
        Z, H, Hkv, N, D, RB, TD = (C2[k] for k in ("Z", "H", "Hkv", "N", "D", "RB", "TD"))
        G = H // Hkv
        kv_groups = list(range(Hkv)) if kv_groups is None else list(kv_groups)
        heads = [g * G + j for g in kv_groups for j in range(G)]
        self.H, self.Hkv = len(heads), len(kv_groups)
        self.NB = N // RB
        gen = torch.Generator().manual_seed(seed)
        h_q = torch.randn(Z, H, N, D, generator=gen).bfloat16()
        h_k = torch.randn(Z, Hkv, N, D, generator=gen).bfloat16()
        h_v = torch.randn(Z, Hkv, N, D, generator=gen).bfloat16()
        h_do = torch.randn(Z, H, N, D, generator=gen).bfloat16()
        if self.H != H:
            h_q, h_do = h_q[:, heads].contiguous(), h_do[:, heads].contiguous()
            h_k, h_v = h_k[:, kv_groups].contiguous(), h_v[:, kv_groups].contiguous()
        self.h_q, self.h_k, self.h_v, self.h_do = (t.pin_memory() for t in (h_q, h_k, h_v, h_do))
        self.q, self.k, self.v, self.do = (t.to(dev) for t in (self.h_q, self.h_k, self.h_v, self.h_do))
        self.router = tree_router(Z, self.H, self.NB, TD).to(dev)
        self.t_heads = [t_heads[h] for h in heads]
        self.depth = torch.tensor(self.t_heads, dtype=torch.int32, device=dev)
        self.causal, self.sink = causal, sink
        self.scale = 1.0 / math.sqrt(D)
        NB = self.NB
        self.lists = torch.empty(Z, self.H, NB, NB, dtype=torch.int32, device=dev)
        self.counts = torch.empty(Z, self.H, NB, dtype=torch.int32, device=dev)
        self.out = torch.empty_like(self.q)
        self.lse = torch.empty(Z, self.H, N, dtype=torch.float32, device=dev)
        self.dq = torch.empty_like(self.q)
        self.dk = torch.empty_like(self.k)
        self.dv = torch.empty_like(self.v)
        wsb = int(nat.lib().sa_block_list_attention_bwd_workspace_bytes(Z, self.H, self.Hkv, N, D, RB))
        self.ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        fwb = int(nat.lib().sa_block_list_attention_fwd_workspace_bytes(Z, self.H, N, D, RB))
        self.fws = torch.empty(max(fwb, 256), dtype=torch.uint8, device=dev)
        self.build()
        torch.cuda.synchronize()
        self.kept = int(self.counts.sum())
        RB2D = RB * RB * D
        # per-kernel tensor work: the fused backward does S^T, dP^T, dV, dK, dQ (10 RB^2 D per
        # kept pair); the two-kernel path recomputes S and dP in both kernels (6 + 8)
        self.fused = fused
        self.flops = {"fwd": self.kept * 4 * RB2D, "bwd": self.kept * 10 * RB2D,
                      "dq": self.kept * 6 * RB2D, "dkdv": self.kept * 8 * RB2D}
        self.parts = ("build", "fwd", "prep", "bwd") if fused else ("build", "fwd", "prep", "dq", "dkdv")
        self.flops_alg = self.kept * 14 * RB2D
        # compulsory bytes of the forward: Q, O, LSE and each referenced K/V block once per KV head
        ref_kv = torch.zeros(Z, self.Hkv, NB, dtype=torch.bool, device=dev)
        for h in range(self.H):
            c = self.counts[0, h]
            m = torch.arange(NB, device=dev).view(1, -1) < c.view(-1, 1)
            ref_kv[0, h // G].index_put_((self.lists[0, h][m].long(),), torch.tensor(True, device=dev))
        self.fwd_bytes = (2 * self.q.numel() * 2 + self.lse.numel() * 4 +
                          int(ref_kv.sum()) * RB * D * 2 * 2)

    def build(self):
        nat, s = self.nat, torch.cuda.current_stream().cuda_stream
        nat.check(nat.lib().sa_build_block_lists(
            self.router.data_ptr(), nat.SA_I32, nat.strides(self.router), 1, self.H, self.NB, C2["TD"],
            self.depth.data_ptr(), 2, 1, int(self.causal), int(self.sink), 0,
            self.lists.data_ptr(), self.NB, self.counts.data_ptr(), s), "build")

    def fwd(self):
        nat, s = self.nat, torch.cuda.current_stream().cuda_stream
        N, D, RB = C2["N"], C2["D"], C2["RB"]
        nat.check(nat.lib().sa_block_list_attention_fwd(
            nat.SA_BF16, 1, self.H, self.Hkv, N, D, RB, self.q.data_ptr(), nat.strides(self.q),
            self.k.data_ptr(), nat.strides(self.k), self.v.data_ptr(), nat.strides(self.v),
            self.out.data_ptr(), nat.strides(self.out), self.lse.data_ptr(),
            self.lists.data_ptr(), self.NB, self.counts.data_ptr(), None, 0, None,
            int(self.causal), self.scale, self.fws.data_ptr(), self.fws.numel(), s), "fwd")

    def bwd(self, phase):
        nat, s = self.nat, torch.cuda.current_stream().cuda_stream
        N, D, RB = C2["N"], C2["D"], C2["RB"]
        nat.check(nat.lib().sa_block_list_attention_bwd_phase(
            phase, nat.SA_BF16, 1, self.H, self.Hkv, N, D, RB, self.q.data_ptr(), nat.strides(self.q),
            self.k.data_ptr(), nat.strides(self.k), self.v.data_ptr(), nat.strides(self.v),
            self.out.data_ptr(), nat.strides(self.out), self.do.data_ptr(), nat.strides(self.do),
            self.lse.data_ptr(), self.lists.data_ptr(), self.NB, self.counts.data_ptr(),
            None, 0, None, int(self.causal), self.scale,
            self.dq.data_ptr(), nat.strides(self.dq), self.dk.data_ptr(), nat.strides(self.dk),
            self.dv.data_ptr(), nat.strides(self.dv), None, self.ws.data_ptr(), self.ws.numel(), s),
            f"bwd phase {phase}")

    # our kernels per part.  fwd: planner + kernel.  Fused path -- prep: Delta (+ zeroing of
    # the dQ accumulator), transposed lists, dK/dV planner; bwd: fused kernel + split reduce +
    # dQ conversion.  Two-kernel path -- prep: Delta, transposed lists, planner; dq: planner +
    # kernel; dkdv: kernel + split reduce.
    LAUNCHES = {"build": 1, "fwd": 2, "prep": 3, "bwd": 3, "dq": 2, "dkdv": 2}

    def launches(self):
        return sum(self.LAUNCHES[p] for p in self.parts)

    def step(self, evs):
        evs[0].record()
        self.build()
        evs[1].record()
        self.fwd()
        evs[2].record()
        if self.fused:
            self.bwd(4)
            evs[3].record()
            self.bwd(5)
            evs[4].record()
        else:
            self.bwd(1)
            evs[3].record()
            self.bwd(2)
            evs[4].record()
            self.bwd(3)
            evs[5].record()

    def free_device(self):
        """Drop the device tensors (the counts and host copies stay) to make room for
        another process on this GPU."""
        for name in ("q", "k", "v", "do", "router", "depth", "lists", "out", "lse", "dq", "dk",
                     "dv", "ws", "fws"):
            setattr(self, name, None)

    def step_plain(self):
        self.build()
        self.fwd()
        for ph in ((4, 5) if self.fused else (1, 2, 3)):
            self.bwd(ph)


def flush_l2(buf):
    buf.zero_()


def time_c2(prob, steps, warmup, flush, barrier=None):
    ne = len(prob.parts) + 1
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(ne)] for _ in range(steps)]
    for _ in range(warmup):
        flush_l2(flush)
        prob.step([torch.cuda.Event(enable_timing=True) for _ in range(ne)])
    torch.cuda.synchronize()
    if barrier:
        barrier()
    torch.cuda.synchronize()
    for i in range(steps):
        flush_l2(flush)
        prob.step(evs[i])
    torch.cuda.synchronize()
    if barrier:
        barrier()
    torch.cuda.synchronize()
    parts = {p: [] for p in prob.parts}
    totals = []
    for e in evs:
        for j, p in enumerate(prob.parts):
            parts[p].append(e[j].elapsed_time(e[j + 1]))
        totals.append(e[0].elapsed_time(e[ne - 1]))
    return sum(totals), {p: statistics.mean(v) for p, v in parts.items()}


def time_c2_graph(prob, steps, warmup, flush):
    """The same step captured once in a CUDA graph and replayed (L2 flushed between
    replays, outside the events): what is left when host launch work is taken away.  The
    difference from the eager step is the launch and host overhead of the C-ABI calls."""
    try:
        for _ in range(2):
            prob.step_plain()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            prob.step_plain()
        torch.cuda.synchronize()
        for _ in range(warmup):
            flush_l2(flush)
            g.replay()
        torch.cuda.synchronize()
        times = []
        for _ in range(steps):
            flush_l2(flush)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        del g
        return {"ms_per_step": round(statistics.mean(times), 4),
                "ms_median": round(statistics.median(times), 4)}
    except Exception as ex:  # capture is a diagnostic; report why it did not run
        torch.cuda.synchronize()
        return {"error": f"{type(ex).__name__}: {str(ex)[:160]}"}


def time_e2e(prob, steps, warmup):
    """Public API end to end: pinned host -> device, block_list_attention autograd fwd+bwd,
    out/dq/dk/dv -> pinned host, per step."""
    from ultrametric import block_list_attention, build_block_lists
    dev = prob.dev
    h_out = torch.empty_like(prob.h_q).pin_memory()
    h_dq = torch.empty_like(prob.h_q).pin_memory()
    h_dk = torch.empty_like(prob.h_k).pin_memory()
    h_dv = torch.empty_like(prob.h_v).pin_memory()
    h_router = prob.router.cpu().pin_memory()

    def one():
        q = prob.h_q.to(dev, non_blocking=True).requires_grad_(True)
        k = prob.h_k.to(dev, non_blocking=True).requires_grad_(True)
        v = prob.h_v.to(dev, non_blocking=True).requires_grad_(True)
        do = prob.h_do.to(dev, non_blocking=True)
        r = h_router.to(dev, non_blocking=True)
        bl = build_block_lists(r, prob.t_heads, is_causal=prob.causal, sink_block=prob.sink, arity=2)
        out = block_list_attention(q, k, v, bl, route_block=C2["RB"], is_causal=prob.causal)
        out.backward(do)
        h_out.copy_(out.detach(), non_blocking=True)
        h_dq.copy_(q.grad, non_blocking=True)
        h_dk.copy_(k.grad, non_blocking=True)
        h_dv.copy_(v.grad, non_blocking=True)

    for _ in range(warmup):
        one()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        one()
        e1.record()
        e1.synchronize()
        total += e0.elapsed_time(e1)
    h2d = sum(t.numel() * t.element_size() for t in (prob.h_q, prob.h_k, prob.h_v, prob.h_do, h_router))
    d2h = sum(t.numel() * t.element_size() for t in (h_out, h_dq, h_dk, h_dv))
    return total / steps, h2d, d2h


def time_e2e_pipelined(prob, steps, warmup):
    """Public API end to end, as a serving or training loop runs it: every step still copies its
    own inputs pinned host -> device and its out/dq/dk/dv device -> pinned host, but on two copy
    streams, so the upload of step i+1 and the download of step i-1 overlap the compute of step i
    (inputs double-buffered on the device, outputs double-buffered on the host).  The timed region
    spans the first upload to the last download; ms per step = that span / steps."""
    from ultrametric import block_list_attention, build_block_lists
    dev = prob.dev
    h_in = (prob.h_q, prob.h_k, prob.h_v, prob.h_do, prob.router.cpu().pin_memory())
    d_in = [[torch.empty_like(t, device=dev) for t in h_in] for _ in range(2)]
    h_out = [[torch.empty_like(t).pin_memory() for t in (prob.h_q, prob.h_q, prob.h_k, prob.h_v)]
             for _ in range(2)]
    s_up, s_cmp, s_down = (torch.cuda.Stream(dev) for _ in range(3))
    cmp_done = [None, None]
    down_done = [None, None]

    def run(n):
        for i in range(n):
            slot = i & 1
            with torch.cuda.stream(s_up):
                if cmp_done[slot] is not None:
                    s_up.wait_event(cmp_done[slot])     # step i-2 has finished reading this slot
                for d, h in zip(d_in[slot], h_in):
                    d.copy_(h, non_blocking=True)
                up = torch.cuda.Event()
                up.record(s_up)
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(up)
                dq_, dk_, dv_, ddo, dr = d_in[slot]
                q = dq_.detach().requires_grad_(True)
                k = dk_.detach().requires_grad_(True)
                v = dv_.detach().requires_grad_(True)
                bl = build_block_lists(dr, prob.t_heads, is_causal=prob.causal,
                                       sink_block=prob.sink, arity=2)
                out = block_list_attention(q, k, v, bl, route_block=C2["RB"], is_causal=prob.causal)
                out.backward(ddo)
                res = (out.detach(), q.grad, k.grad, v.grad)
                ev = torch.cuda.Event()
                ev.record(s_cmp)
                cmp_done[slot] = ev
            with torch.cuda.stream(s_down):
                s_down.wait_event(ev)
                if down_done[slot] is not None:
                    s_down.wait_event(down_done[slot])
                for h, d in zip(h_out[slot], res):
                    d.record_stream(s_down)
                    h.copy_(d, non_blocking=True)
                dd = torch.cuda.Event()
                dd.record(s_down)
                down_done[slot] = dd

    run(warmup)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_up)
    run(steps)
    s_down.wait_stream(s_up)
    s_down.wait_stream(s_cmp)
    e1.record(s_down)
    e1.synchronize()
    h2d = sum(t.numel() * t.element_size() for t in h_in)
    d2h = sum(t.numel() * t.element_size() for t in h_out[0])
    return e0.elapsed_time(e1) / steps, h2d, d2h


def time_sdpa(prob, causal, steps=5):
    """Dense FlashAttention-equivalent: torch SDPA on the same inputs (K/V expanded to the
    query heads, as the reference's surgery path does with repeat_kv)."""
    import torch.nn.functional as F
    g = C2["H"] // C2["Hkv"]
    q = prob.q.detach()
    k = prob.k.detach().repeat_interleave(g, dim=1)
    v = prob.v.detach().repeat_interleave(g, dim=1)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    res = {}
    try:
        with torch.no_grad():
            for _ in range(3):
                F.scaled_dot_product_attention(q, k, v, is_causal=causal)
            torch.cuda.synchronize()
            e0.record()
            for _ in range(steps):
                F.scaled_dot_product_attention(q, k, v, is_causal=causal)
            e1.record()
            e1.synchronize()
        res["fwd_ms"] = e0.elapsed_time(e1) / steps
        qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
        for _ in range(3):
            F.scaled_dot_product_attention(qg, kg, vg, is_causal=causal).backward(prob.do)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(steps):
            F.scaled_dot_product_attention(qg, kg, vg, is_causal=causal).backward(prob.do)
        e1.record()
        e1.synchronize()
        res["fwd_bwd_ms"] = e0.elapsed_time(e1) / steps
    except Exception as ex:  # pragma: no cover - depends on the torch build
        res["error"] = f"{type(ex).__name__}: {str(ex)[:120]}"
    return res


def run_sweep(dev, flush, steps):
    NB = C2["N"] // C2["RB"]
    rows = []
    for name, t, causal, sink in (("50%", 1, True, True), ("90%", 4, True, True),
                                  ("98.4%", 6, False, False)):
        prob = C2Problem(dev, 0, [t] * C2["H"], causal=causal, sink=sink)
        total, parts = time_c2(prob, steps, 2, flush)
        ms = total / steps
        kept = prob.kept
        fwd_tf = prob.flops["fwd"] / (parts["fwd"] * 1e-3) / 1e12
        bwd_ms = sum(v for k, v in parts.items() if k not in ("build", "fwd"))
        sd = time_sdpa(prob, causal)
        rows.append({
            "target": name, "threshold": t, "causal": causal, "sink": sink, "kept_blocks": kept,
            "sparsity_full_grid": round(1 - kept / (C2["H"] * NB * NB), 4),
            "sparsity_causal": round(1 - kept / (C2["H"] * NB * (NB + 1) / 2), 4),
            "step_ms": round(ms, 4), "fwd_ms": round(parts["fwd"], 4), "bwd_ms": round(bwd_ms, 4),
            "build_ms": round(parts["build"], 4),
            "parts_ms": {k: round(v, 4) for k, v in parts.items()},
            "fwd_kept_tflops": round(fwd_tf, 2),
            "fwd_bwd_kept_tflops": round(prob.flops_alg / (ms * 1e-3) / 1e12, 2),
            "dense_sdpa": sd,
            "speedup_fwd_vs_sdpa": round(sd["fwd_ms"] / parts["fwd"], 2) if "fwd_ms" in sd else None,
            "speedup_fwd_bwd_vs_sdpa": round(sd["fwd_bwd_ms"] / ms, 2) if "fwd_bwd_ms" in sd else None,
        })
        del prob
        torch.cuda.empty_cache()
    return rows


C3 = dict(B=64, H=32, Hkv=8, D=128, page=64, TD=9, req_depth=4, local_blocks=1, sink_block=True,
          ctx_lo=2048, ctx_hi=32768)


def make_c3(dev, seed=0):
    """The C3 decode batch: 64 requests, H=32/8, D=128, page 64, ctx ~U[2048, 32768] (seeded),
    a shuffled physical page pool with random block tables, tree routes of the LOGICAL page
    index (depth 9) stored at the physical page id, a random query leaf per request (routes
    shared by all heads), req_depth 4, sink + most recent page.  Host-side metadata is kept
    for byte counts and the CPU oracle; the caches are drawn on the device."""
    B, H, Hkv, D, page, TD = (C3[k] for k in ("B", "H", "Hkv", "D", "page", "TD"))
    gen = torch.Generator().manual_seed(10 + seed)
    ctx = torch.randint(C3["ctx_lo"], C3["ctx_hi"] + 1, (B,), generator=gen, dtype=torch.int32)
    n_log = (ctx + page - 1) // page
    maxL = int(n_log.max())
    total = int(n_log.sum()) + 16
    perm = torch.randperm(total, generator=gen).to(torch.int32)
    bt = torch.zeros(B, maxL, dtype=torch.int32)
    logical_of = torch.zeros(total, dtype=torch.int64)
    off = 0
    for b in range(B):
        n = int(n_log[b])
        bt[b, :n] = perm[off:off + n]
        logical_of[perm[off:off + n].long()] = torch.arange(n)
        off += n
    bits = ((logical_of.view(-1, 1) >> torch.arange(TD - 1, -1, -1).view(1, -1)) & 1).to(torch.int32)
    ri = bits.view(total, 1, TD).expand(total, H, TD).contiguous()
    leaf = torch.randint(0, 1 << TD, (B,), generator=gen)
    qbits = ((leaf.view(-1, 1) >> torch.arange(TD - 1, -1, -1).view(1, -1)) & 1).to(torch.int32)
    qri = qbits.view(B, 1, TD).expand(B, H, TD).contiguous()
    g = torch.Generator(device=dev).manual_seed(20 + seed)
    kc = torch.randn(total, Hkv, page, D, generator=g, device=dev, dtype=torch.bfloat16)
    vc = torch.randn(total, Hkv, page, D, generator=g, device=dev, dtype=torch.bfloat16)
    q = torch.randn(B, H, D, generator=g, device=dev, dtype=torch.bfloat16)
    return {"q": q, "kc": kc, "vc": vc, "bt": bt.to(dev), "ctx": ctx.to(dev), "ri": ri.to(dev),
            "qri": qri.to(dev), "h_bt": bt, "h_ctx": ctx, "h_ri": ri, "h_qri": qri,
            "bits": bits, "qbits": qbits, "n_log": n_log, "total_pages": total}


def c3_routed_bytes(c3, requests):
    """Algorithmic bytes of a decode over ``requests``: the selected pages' valid tokens x
    Hkv x D x 2 B for K and V (each KV byte once per KV head; the routes are shared by the
    heads of a group) + Q and O.  Returns (bytes, selected pages)."""
    Hkv, D, page, H = C3["Hkv"], C3["D"], C3["page"], C3["H"]
    rd, local = C3["req_depth"], C3["local_blocks"]
    tokens = pages = 0
    for b in requests:
        n = int(c3["n_log"][b])
        lp = torch.arange(n)
        match = (c3["bits"][lp][:, :rd] == c3["qbits"][b, :rd]).all(-1)
        match[0] = True
        match[max(0, n - local):] = True
        valid = torch.clamp(int(c3["h_ctx"][b]) - lp * page, max=page)
        tokens += int(valid[match].sum())
        pages += int(match.sum())
    return tokens * Hkv * D * 2 * 2 + 2 * len(requests) * H * D * 2, pages


def c3_host_subset(c3, requests):
    """CPU copies of what the decode of ``requests`` reads: their pages in a compacted pool,
    with block tables and page routes re-indexed to it (for the CPU oracle)."""
    n_log = c3["n_log"]
    phys = torch.cat([c3["h_bt"][b, :int(n_log[b])].long() for b in requests])
    remap = {int(p): i for i, p in enumerate(phys.tolist())}
    maxL = max(int(n_log[b]) for b in requests)
    bt = torch.zeros(len(requests), maxL, dtype=torch.int32)
    for i, b in enumerate(requests):
        n = int(n_log[b])
        bt[i, :n] = torch.tensor([remap[int(p)] for p in c3["h_bt"][b, :n].tolist()], dtype=torch.int32)
    idx = phys.to(c3["kc"].device)
    return {"q": c3["q"][list(requests)].cpu(), "kc": c3["kc"][idx].cpu(), "vc": c3["vc"][idx].cpu(),
            "bt": bt, "ctx": c3["h_ctx"][list(requests)].clone(), "ri": c3["h_ri"][phys].clone(),
            "qri": c3["h_qri"][list(requests)].clone()}


def c3_decode(c3, requests=None):
    """One C3 decode through the public API (``requests``: a contiguous slice, for strong
    scaling; default all 64)."""
    from ultrametric import ultrametric_decode
    sl = slice(None) if requests is None else slice(requests[0], requests[-1] + 1)
    return ultrametric_decode(c3["q"][sl], c3["kc"], c3["vc"], c3["bt"][sl], c3["ctx"][sl],
                              c3["ri"], c3["qri"][sl], C3["req_depth"],
                              local_blocks=C3["local_blocks"], sink_block=C3["sink_block"])


def cpu_decode_baseline(c3, requests=(0, 21, 42, 63)):
    """The reference's CPU decode (_ultrametric_decode_reference, kernel_decode.py:129-185,
    restated in oracle/) on a request sample, scaled to the 64-request batch by routed bytes.
    The port reads the GQA cache head of each query head, which is what the reference's
    expanded cache gives it.  Returns (seconds for 64 requests, sample seconds, sample)."""
    from oracle import decode_oracle as dor
    sub = c3_host_subset(c3, list(requests))
    t0 = time.perf_counter()
    dor.ultrametric_decode_reference(sub["q"].float(), sub["kc"].float(), sub["vc"].float(), sub["bt"],
                                     sub["ctx"], sub["ri"], sub["qri"], C3["req_depth"],
                                     local_blocks=C3["local_blocks"], sink_block=C3["sink_block"],
                                     compute_dtype=torch.float32)
    s = time.perf_counter() - t0
    b_all, _ = c3_routed_bytes(c3, range(C3["B"]))
    b_sub, _ = c3_routed_bytes(c3, list(requests))
    return s * b_all / b_sub, s, list(requests)


def run_decode(dev, seed, steps, warmup, flush, peaks, world=1, rank=0, barrier=None, cpu=False):
    """C3 routed paged decode.  Weak scaling: every rank decodes its own 64-request batch.
    Strong scaling (world > 1): the one 64-request batch is split into contiguous request
    slices, one per rank, as the C3 config defines it.  Times are the max over ranks."""
    B = C3["B"]
    c3 = make_c3(dev, seed)
    routed_bytes, sel_pages = c3_routed_bytes(c3, range(B))

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        if barrier:
            barrier()
        tot = 0.0
        for _ in range(steps):
            flush_l2(flush)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            tot += e0.elapsed_time(e1)
        return max_over_ranks([tot / steps], world, dev)[0]

    ms = timed(lambda: c3_decode(c3))
    gbs = world * routed_bytes / (ms * 1e-3) / 1e9
    dense_bytes = int(c3["n_log"].sum()) * C3["page"] * C3["Hkv"] * C3["D"] * 2 * 2
    res = {
        "config": "C3: 64 req x 1 token, H=32/8, D=128, page 64, ctx~U[2048,32768], req_depth 4, sink+last page",
        "ms_per_step": round(ms, 4), "tok_per_s": round(world * B / (ms * 1e-3), 1),
        "requests_per_gpu": B, "scaling": "weak",
        "routed_gbs": round(gbs, 1), "routed_bytes": routed_bytes, "routed_pages": sel_pages,
        "dense_equivalent_bytes": dense_bytes,
        # per GPU (the slowest rank), against one GPU's measured copy bandwidth
        "roofline": {"bound": "hbm", "achieved": round(gbs / world, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(gbs / world / peaks["hbm_gbs"], 4), "per": "GPU"},
        "gpu_launches_per_step": 4,
    }
    if world > 1:
        per = B // world
        mine = list(range(rank * per, (rank + 1) * per))
        if seed != 0:  # every rank takes its slice of the same (seed 0) batch
            del c3
            torch.cuda.empty_cache()
            c3 = make_c3(dev, 0)
        ms_s = timed(lambda: c3_decode(c3, mine))
        res["strong"] = {"requests_per_gpu": per, "ms_per_step": round(ms_s, 4),
                         "tok_per_s": round(B / (ms_s * 1e-3), 1),
                         "routed_gbs": round(routed_bytes / (ms_s * 1e-3) / 1e9, 1),
                         "scaling": "strong: the one 64-request batch split over the ranks"}
    if cpu and rank == 0 and world == 1:
        torch.set_num_threads(os.cpu_count() or 1)
        cpu_s, sample_s, reqs = cpu_decode_baseline(c3)
        res["cpu_baseline"] = {"value": round(B / cpu_s, 3), "unit": "tok/s",
                               "ms_per_step": round(cpu_s * 1e3, 1),
                               "cores": torch.get_num_threads(), "kind": "port",
                               "measured_s": round(sample_s, 3), "scale": round(cpu_s / sample_s, 2),
                               "sample": f"_ultrametric_decode_reference (fp32, per query head) on "
                                         f"requests {reqs}, scaled to the 64-request batch by routed bytes"}
    del c3
    torch.cuda.empty_cache()
    return res


C5 = dict(Z=1, H=16, Hkv=8, N=131072, D=128, RB=128, TD=10, t=7)


def make_c5(dev, rank=0, world=1):
    """C5 inputs: N=131072, H=16/8, D=128, RB=128 (NB=1024), tree routes TD=10, threshold 7,
    causal + sink (5624 kept blocks per head), lists built on the device.  q/k/v hold this
    rank's contiguous chunk of N / world rows, drawn on the device (seed 40 + rank)."""
    from ultrametric import build_block_lists
    Z, H, Hkv, N, D, RB = (C5[k] for k in ("Z", "H", "Hkv", "N", "D", "RB"))
    router = tree_router(Z, H, N // RB, C5["TD"])
    bl = build_block_lists(router.to(dev), C5["t"], is_causal=True, sink_block=True, arity=2)
    Nl = N // world  # this rank's rows: with several ranks, the zigzag pair of chunks
    g = torch.Generator(device=dev).manual_seed(40 + rank)
    q = torch.randn(Z, H, Nl, D, generator=g, device=dev, dtype=torch.bfloat16)
    k = torch.randn(Z, Hkv, Nl, D, generator=g, device=dev, dtype=torch.bfloat16)
    v = torch.randn(Z, Hkv, Nl, D, generator=g, device=dev, dtype=torch.bfloat16)
    return {"q": q, "k": k, "v": v, "bl": bl, "router": router, "rows_per_rank": Nl}


def cpu_c5_baseline(c5, rows=1024):
    """The reference's CPU path for C5 cannot run whole (70 TFLOP of masked dense attention):
    time a slice of it -- head 0, the last ``rows`` query rows against all 131072 keys,
    masked dense fp32 in the query-chunked form of benchmarks/benchmark_block_list.py:106-123
    -- and scale by the rows and heads it stands for (every query chunk of that form scores
    all N keys).  Returns (seconds for the whole forward, sample seconds, scale)."""
    from oracle import attention_oracle as ao
    from oracle import block_list_oracle as blo
    N, H, RB = C5["N"], C5["H"], C5["RB"]
    bm = torch.from_numpy(blo.block_mask(c5["router"][:, :1].numpy(), C5["t"], is_causal=True,
                                         sink_block=True))
    q = c5["q"][:, :1].float().cpu()
    k = c5["k"][:, :1].float().cpu()
    v = c5["v"][:, :1].float().cpu()
    t0 = time.perf_counter()
    ao.masked_attention_chunked(q, k, v, bm, RB, True, chunk=rows, compute_dtype=torch.float32,
                                row_ranges=[(N - rows, N)])
    s = time.perf_counter() - t0
    scale = H * N / rows
    return s * scale, s, scale


def run_c5(dev, rank, world, steps, warmup, flush, barrier=None, cpu=False):
    """C5 very long prefill forward: N=131072, H=16/8, D=128, RB=128 (NB=1024), tree routes
    TD=10, threshold 7, causal + sink (5624 kept blocks per head).  One GPU: the whole
    sequence.  N GPUs: the sequence sharded contiguously, K/V chunks rotating over NCCL
    (ultrametric.ring), time = max over ranks."""
    from ultrametric.block_list import _fwd
    from ultrametric.ring import RingPlan, ring_block_list_attention
    Z, H, Hkv, N, D, RB = (C5[k] for k in ("Z", "H", "Hkv", "N", "D", "RB"))
    c5 = make_c5(dev, rank, world)
    q, k, v, bl, Nl = c5["q"], c5["k"], c5["v"], c5["bl"], c5["rows_per_rank"]
    kept = int(bl.counts.sum())
    scale = 1.0 / math.sqrt(D)
    # the ring's schedule depends only on the lists: planned once, like the lists themselves.
    # Zigzag layout: rank r holds chunks r and 2P - 1 - r, so the causal work is balanced.
    plan = RingPlan(bl, world, rank, Nl, RB, True, layout="zigzag") if world > 1 else None

    def one():
        if world == 1:
            _fwd(q, k, v, bl.lists, bl.counts, RB, True, scale, True, None)
        else:
            ring_block_list_attention(q, k, v, bl, route_block=RB, is_causal=True, plan=plan,
                                      layout="zigzag")

    for _ in range(warmup):
        one()
    torch.cuda.synchronize()
    if barrier:
        barrier()
    tot = 0.0
    for _ in range(steps):
        flush_l2(flush)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        one()
        e1.record()
        e1.synchronize()
        tot += e0.elapsed_time(e1)
    ms = max_over_ranks([tot / steps], world, dev)[0]
    flops = kept * 4 * RB * RB * D
    res = {"config": "C5: N=131072, H=16/8, D=128, RB=128, tree routes TD=10, t=7, causal + sink",
           "kept_blocks": kept, "kept_per_head": kept / H, "ms": round(ms, 4),
           "kept_tflops": round(flops / (ms * 1e-3) / 1e12, 2)}
    if world > 1:
        sent = sum(int(g.numel()) for _, g, _, _ in plan.exchange if g is not None)
        res["ring"] = {"ranks": world, "rows_per_rank": Nl, "layout": "zigzag (chunks r, 2P-1-r)",
                       "hops_computed": len(plan.hops),
                       "kv_rows_sent_by_rank0": sent,
                       "kv_bytes_sent_by_rank0": 2 * Z * Hkv * sent * D * 2,
                       "dense_ring_bytes_per_hop": 2 * Z * Hkv * Nl * D * 2,
                       "transport": "NCCL send/recv (torch.distributed) of the referenced K/V blocks only"}
    if cpu and rank == 0 and world == 1:
        torch.set_num_threads(os.cpu_count() or 1)
        cpu_s, sample_s, sc = cpu_c5_baseline(c5)
        res["cpu_baseline"] = {"value": round(flops / cpu_s / 1e12, 6), "unit": "TFLOP/s",
                               "ms": round(cpu_s * 1e3, 1), "cores": torch.get_num_threads(),
                               "kind": "port", "measured_s": round(sample_s, 3), "scale": sc,
                               "sample": "masked dense fp32 forward, head 0, the last 1024 query rows "
                                         "against all 131072 keys (query-chunked form), scaled by "
                                         "16 heads x 131072 rows / 1024 rows; rate on kept-block FLOPs"}
    del c5
    torch.cuda.empty_cache()
    return res


C4 = dict(Z=4, H=4, Hkv=1, N=32768, D=128, RB=128, levels=8, p=2, r=4, depth=(3, 4, 4, 4),
          local_blocks=1, layers=32)


def _torch_vote_glue(assign, r, rb):
    """The reference's torch glue for the block vote (surgery.py:543-547), restated for a
    same-GPU comparison: token argmax, one-hot, sum over each route block, argmax."""
    B, H, S, _, p = assign.shape
    nb = -(-S // rb)
    idx = assign[:, :, :S, :r, :].argmax(dim=-1)
    votes = torch.nn.functional.one_hot(idx, p).to(torch.float32)
    if nb * rb != S:
        votes = torch.nn.functional.pad(votes, (0, 0, 0, 0, 0, nb * rb - S))
    return votes.view(B, H, nb, rb, r, p).sum(3).argmax(-1).to(torch.int32)


def cpu_c4_baseline(q, k, v, bl, rows=1024):
    """The reference's CPU path for one C4 layer slice: query head 0 of sequence 0, the last
    ``rows`` query rows against all 32768 keys, masked dense fp32 (query-chunked form),
    scaled by rows x heads x sequences x layers.  Returns (seconds per layer, sample s, scale)."""
    from oracle import attention_oracle as ao
    N, RB = C4["N"], C4["RB"]
    lists, counts = bl.lists[:1, :1].cpu(), bl.counts[:1, :1].cpu()
    bm = torch.zeros(1, 1, N // RB, N // RB, dtype=torch.bool)
    for i in range(N // RB):
        c = int(counts[0, 0, i])
        bm[0, 0, i, lists[0, 0, i, :c].long()] = True
    qs, ks, vs = (t[:1, :1].float().cpu() for t in (q, k, v))
    t0 = time.perf_counter()
    ao.masked_attention_chunked(qs, ks, vs, bm, RB, True, chunk=rows, compute_dtype=torch.float32,
                                row_ranges=[(N - rows, N)])
    s = time.perf_counter() - t0
    scale = C4["Z"] * C4["H"] * N / rows
    return s * scale, s, scale


def run_c4(dev, rank, world, warmup, flush, barrier=None, cpu=False):
    """C4 Llama-3.1-8B-shaped surgery prefill, the attention sublayer on one GPU's KV group
    (the 8-GPU job splits the 32 heads by KV group): batch 4, N=32768, 4 query heads / 1 KV
    head, D=128, route_block 128 (NB=256), 32 layers, bf16, random init.  Per layer: that
    layer's Q/K/V and its router's per-token outputs (levels 8, p=2), then
    build_block_lists_from_assignments -- per-block majority vote of the first r=4 levels,
    per-head match depth 3/4/4/4, causal + sink + one local block -- and the block-list
    forward.  Depth d keeps ~2^-d of the causal triangle (plus sink, diagonal and local
    band), ~10 % on average over the four heads.  One step = all 32 layers; time = max over
    ranks.  The router's projection is not part of this library: a random-init router's
    argmax branches are uniformly random, so its outputs are drawn at random."""
    from ultrametric import build_block_lists
    from ultrametric.block_list import _fwd
    from ultrametric.surgery_routing import build_block_lists_from_assignments
    Z, H, Hkv, N, D, RB, L = (C4[k] for k in ("Z", "H", "Hkv", "N", "D", "RB", "layers"))
    NB = N // RB
    g = torch.Generator(device=dev).manual_seed(400 + rank)
    layers = []
    for _ in range(L):
        layers.append((torch.randn(Z, H, N, D, generator=g, device=dev, dtype=torch.bfloat16),
                       torch.randn(Z, Hkv, N, D, generator=g, device=dev, dtype=torch.bfloat16),
                       torch.randn(Z, Hkv, N, D, generator=g, device=dev, dtype=torch.bfloat16),
                       torch.randn(Z, H, N, C4["levels"], C4["p"], generator=g, device=dev,
                                   dtype=torch.bfloat16)))
    scale = 1.0 / math.sqrt(D)
    depth = torch.tensor(C4["depth"], dtype=torch.int32, device=dev)
    kw = dict(route_block=RB, req_depth=depth, is_causal=True, sink_block=True,
              local_blocks=C4["local_blocks"], arity=C4["p"])

    def lists_of(assign):
        return build_block_lists_from_assignments(assign, C4["r"], **kw)

    def step(collect=None):
        for q, k, v, assign in layers:
            bl = lists_of(assign)
            _fwd(q, k, v, bl.lists, bl.counts, RB, True, scale, True, None)
            if collect is not None:
                collect.append(bl.counts.sum())

    def timed(fn):
        torch.cuda.synchronize()
        if barrier:
            barrier()
        flush_l2(flush)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        return max_over_ranks([e0.elapsed_time(e1)], world, dev)[0]

    def graph_ms(fn):
        """Replay time of ``fn`` captured in a CUDA graph: the GPU time without the host's
        per-call overhead (these small launches are host-bound when called eagerly)."""
        try:
            fn()
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                fn()
            gr.replay()
            ms_g = timed(gr.replay)
            del gr
            return round(ms_g / L, 4)
        except Exception as ex:
            torch.cuda.synchronize()
            return f"capture failed: {type(ex).__name__}: {str(ex)[:100]}"

    counts = []
    for _ in range(max(1, warmup)):
        step(counts if not counts else None)
    kept = int(torch.stack(counts).sum())
    ms = timed(step)
    # the routing part alone, fused vs the reference's torch glue + builder on this GPU
    ms_lists = timed(lambda: [lists_of(a) for *_, a in layers])

    def glue():
        for *_, a in layers:
            route = _torch_vote_glue(a, C4["r"], RB)
            build_block_lists(route, depth, is_causal=True, sink_block=True,
                              local_blocks=C4["local_blocks"], arity=C4["p"])
    glue()
    ms_glue = timed(glue)
    causal_pairs = Z * H * NB * (NB + 1) // 2 * L
    flops = kept * 4 * RB * RB * D
    res = {"config": "C4: Llama-3.1-8B-shaped attention sublayer per GPU (1 of 8 KV groups), "
                     "batch 4, N=32768, H=4/1 per GPU, D=128, RB=128, 32 layers, router outputs "
                     "levels 8 p 2 -> majority vote r=4, per-head depth 3/4/4/4, causal + sink + local",
           "layers": L, "ms_all_layers": round(ms, 3), "ms_per_layer": round(ms / L, 4),
           "kept_blocks_all_layers": kept,
           "density_causal": round(kept / causal_pairs, 4),
           "kept_tflops": round(flops / (ms * 1e-3) / 1e12, 2),
           "whole_job_kept_tflops": round(world * flops / (ms * 1e-3) / 1e12, 2),
           "routing_ms_per_layer": {
               "fused_vote_and_lists": round(ms_lists / L, 4),
               "torch_vote_glue_plus_builder": round(ms_glue / L, 4),
               "fused_vote_and_lists_graph": graph_ms(lambda: [lists_of(a) for *_, a in layers]),
               "note": "eager calls are host-bound at this size; the graph replay gives the fused "
                       "path's GPU time (the torch glue copies host data and cannot be captured)"},
           "timed": "per layer: router outputs -> vote + lists (one C-ABI call) -> forward; "
                    "router projection not included"}
    if cpu and rank == 0 and world == 1:
        torch.set_num_threads(os.cpu_count() or 1)
        q, k, v, a = layers[0]
        cpu_layer_s, sample_s, sc = cpu_c4_baseline(q, k, v, lists_of(a))
        res["cpu_baseline"] = {"value": round(flops / L / cpu_layer_s / 1e12, 6), "unit": "TFLOP/s",
                               "ms_per_layer": round(cpu_layer_s * 1e3, 1),
                               "cores": torch.get_num_threads(), "kind": "port",
                               "measured_s": round(sample_s, 3), "scale": sc,
                               "sample": "masked dense fp32 forward of layer 0, sequence 0, head 0: "
                                         "the last 1024 query rows against all 32768 keys, scaled "
                                         "by 4 sequences x 4 heads x 32768 rows / 1024 rows per "
                                         "layer; rate on kept-block FLOPs"}
    del layers
    torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------------------------------------
# the reference's own Triton kernels on this GPU (the bar this build has to beat)
# ---------------------------------------------------------------------------------------

REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def run_reference_triton_subprocess(timeout_s=900):
    """Time the reference's Triton kernels in a child process (its ``ultrametric`` package
    would shadow ours in this one).  The reference is installed, unmodified, into
    baseline/_ref (``pip install --no-index --no-deps --target baseline/_ref`` of its
    source); without it the entry says unavailable."""
    if not os.path.isdir(os.path.join(REF_DIR, "ultrametric")):
        return {"unavailable": "reference not installed in baseline/_ref"}
    cmd = [sys.executable, os.path.abspath(__file__), "--reference-triton-worker"]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout_s)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"reference Triton timing exceeded {timeout_s} s"}
    for line in reversed(r.stdout.strip().splitlines()):
        if line.startswith("{"):
            try:
                return json.loads(line)
            except json.JSONDecodeError:
                break
    return {"unavailable": f"reference Triton worker rc={r.returncode}: "
                           f"{(r.stderr or r.stdout).strip().splitlines()[-1:] }"}


def _bench_ms(fn, flush, reps=20, warmup=3):
    """do_bench-style median over ``reps`` CUDA-event-timed calls, L2 flushed before each."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        flush_l2(flush)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    return statistics.median(times)


def reference_triton_worker(args):
    """Child process: import the reference's ``ultrametric`` from baseline/_ref (never this
    repository's) and time, on the same inputs as our arm:
      * build_block_lists(arity=2) (its fused Triton compaction, block_list.py:127-167);
      * block_list_attention forward and forward+backward (block_list.py:387-681) at C2 for
        the seeded threshold mix and the 50 / 90 / 98.4 % sweep points -- with K/V
        repeat-interleaved to the 32 query heads, since the reference has no GQA;
    Its decode kernel is not run (see the c3_decode entry).  Prints one JSON line."""
    ours = os.path.join(ROOT, "sparse-ai_b200")
    sys.path[:] = [p for p in sys.path if os.path.abspath(p) != ours]
    sys.path.insert(0, REF_DIR)
    import importlib
    rbl = importlib.import_module("ultrametric.block_list")
    assert os.path.abspath(rbl.__file__).startswith(REF_DIR), rbl.__file__
    import triton
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    res = {"source": "sparse-ai installed unmodified in baseline/_ref", "triton": triton.__version__,
           "timing": "median of 20 CUDA-event-timed calls, L2 flushed (256 MiB write) before each"}
    Z, H, Hkv, N, D, RB, TD = (C2[k] for k in ("Z", "H", "Hkv", "N", "D", "RB", "TD"))
    G = H // Hkv
    gen = torch.Generator().manual_seed(0)
    q = torch.randn(Z, H, N, D, generator=gen).bfloat16().to(dev)
    k = torch.randn(Z, Hkv, N, D, generator=gen).bfloat16().to(dev)
    v = torch.randn(Z, Hkv, N, D, generator=gen).bfloat16().to(dev)
    do = torch.randn(Z, H, N, D, generator=gen).bfloat16().to(dev)
    k = k.repeat_interleave(G, dim=1).contiguous()
    v = v.repeat_interleave(G, dim=1).contiguous()
    router = tree_router(Z, H, N // RB, TD).to(dev)
    cases = [("headline", c2_thresholds(0), True, True), ("50%", [1] * H, True, True),
             ("90%", [4] * H, True, True), ("98.4%", [6] * H, False, False)]
    rows = []
    for name, t_heads, causal, sink in cases:
        row = {"case": name}
        try:
            depth = torch.tensor(t_heads, dtype=torch.int64, device=dev)
            build = lambda: rbl.build_block_lists(router, depth, is_causal=causal, sink_block=sink, arity=2)
            row["build_ms"] = round(_bench_ms(build, flush), 4)
            bl = build()
            kept = int(bl.counts.sum())
            row["kept_blocks"] = kept
            with torch.no_grad():
                fwd = lambda: rbl.block_list_attention(q, k, v, bl, route_block=RB, is_causal=causal)
                row["fwd_ms"] = round(_bench_ms(fwd, flush), 4)
            qg, kg, vg = (t.detach().clone().requires_grad_(True) for t in (q, k, v))

            def fwd_bwd():
                out = rbl.block_list_attention(qg, kg, vg, bl, route_block=RB, is_causal=causal)
                out.backward(do)
            row["fwd_bwd_ms"] = round(_bench_ms(fwd_bwd, flush, reps=10), 4)
            f = RB * RB * D
            row["fwd_kept_tflops"] = round(kept * 4 * f / (row["fwd_ms"] * 1e-3) / 1e12, 2)
            row["fwd_bwd_kept_tflops"] = round(kept * 14 * f / (row["fwd_bwd_ms"] * 1e-3) / 1e12, 2)
            row["step_ms_with_build"] = round(row["fwd_bwd_ms"] + row["build_ms"], 4)
            del qg, kg, vg
        except Exception as ex:
            row["error"] = f"{type(ex).__name__}: {str(ex)[:200]}"
        rows.append(row)
        torch.cuda.empty_cache()
    res["c2"] = rows
    del q, k, v, do
    torch.cuda.empty_cache()
    # Not run: at C3 size the reference's decode kernel makes an illegal memory access on
    # B200.  Its offsets are int32 (kernel_decode.py:90-91: physical_block_idx * stride_k_b),
    # and the 32-head cache it needs (no GQA) holds 17.4k pages x 262144 elements, so every
    # page id >= 8192 overflows.  It faulted once in this benchmark and is not launched again.
    res["c3_decode"] = {
        "unavailable": "the reference's Triton decode kernel faulted (illegal memory access) on "
                       "the C3 batch: int32 page offsets (kernel_decode.py:90-91) overflow for the "
                       "32-head expanded cache of 17.4k pages; not run again"}
    print(json.dumps(res), flush=True)


def _merge_reference_triton(line, ref, ms_step):
    """Put the reference's Triton times beside ours: headline step, sweep rows, decode."""
    rows = {r.get("case"): r for r in ref.get("c2", [])}
    h = rows.get("headline", {})
    if "step_ms_with_build" in h:
        line["vs_reference_triton"] = {
            "reference_step_ms": h["step_ms_with_build"], "ours_step_ms": round(ms_step, 4),
            "speedup": round(h["step_ms_with_build"] / ms_step, 2),
            "note": "same inputs; the reference step = its build_block_lists(arity=2) + "
                    "block_list_attention fwd+bwd (K/V expanded to 32 heads)"}
    for r in line.get("sweep", []):
        t = rows.get(r["target"], {})
        if "fwd_ms" in t:
            r["reference_triton_ms"] = {"fwd": t["fwd_ms"], "fwd_bwd": t["fwd_bwd_ms"], "build": t["build_ms"]}
            r["speedup_fwd_vs_reference_triton"] = round(t["fwd_ms"] / r["fwd_ms"], 2)
            r["speedup_step_vs_reference_triton"] = round(t["step_ms_with_build"] / r["step_ms"], 2)
    d = line.get("decode")
    t = ref.get("c3_decode", {})
    if d is not None and "ms" in t:
        d["reference_triton_ms"] = t["ms"]
        d["speedup_vs_reference_triton"] = round(t["ms"] / d["ms_per_step"], 2)


def run_ours(args):
    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    barrier = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

        def barrier():
            dist.barrier()
    peaks, peak_kind = load_peaks()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    if args.decode_only:  # profiling aid: the C3 decode alone, one JSON line
        d = run_decode(dev, rank, args.steps, args.warmup, flush, peaks, world, rank, barrier)
        if rank == 0:
            print(json.dumps({"decode": d}), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    t_heads = c2_thresholds(0) if args.threshold is None else [args.threshold] * C2["H"]
    prob = C2Problem(dev, seed=rank, t_heads=t_heads)
    prob_launches = prob.launches()
    with ClockSampler(local) as clk:
        total_ms, parts = time_c2(prob, args.steps, args.warmup, flush, barrier)
    keys = list(parts)
    red = max_over_ranks([total_ms] + [parts[k] for k in keys], world, dev)
    total_ms = red[0]
    parts = dict(zip(keys, red[1:]))
    ms_step = total_ms / args.steps
    value = prob.flops_alg * world / (ms_step * 1e-3) / 1e12

    # dominant kernel roofline (tensor-bound kernels of the step)
    kern = max((p for p in prob.parts if p in prob.flops), key=lambda p: parts[p])
    achieved = prob.flops[kern] / (parts[kern] * 1e-3) / 1e12
    traffic = None
    tf = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tf):
        with open(tf) as f:
            traffic = json.load(f).get(kern)

    # the reproducible two-kernel backward (deterministic=True) on the same problem, for scale
    det = C2Problem(dev, seed=rank, t_heads=t_heads, fused=False)
    tot_d, parts_d = time_c2(det, args.steps, args.warmup, flush, barrier)
    keys_d = list(parts_d)
    red_d = max_over_ranks([tot_d] + [parts_d[k] for k in keys_d], world, dev)
    two_kernel = {"ms_per_step": round(red_d[0] / args.steps, 4),
                  "breakdown_ms": {k: round(v, 4) for k, v in zip(keys_d, red_d[1:])},
                  "note": "deterministic=True: separate dQ and dK/dV kernels (14 RB^2 D of MMA "
                          "work per kept pair against the fused kernel's 10)"}
    del det
    torch.cuda.empty_cache()

    graph = time_c2_graph(prob, args.steps, args.warmup, flush)
    if "ms_per_step" in graph:
        graph["ms_per_step"] = round(max_over_ranks([graph["ms_per_step"]], world, dev)[0], 4)
        graph["kept_tflops_whole_job"] = round(prob.flops_alg * world / (graph["ms_per_step"] * 1e-3) / 1e12, 2)
    graph["eager_ms_per_step"] = round(ms_step, 4)

    strong = None
    if world > 1 and C2["Hkv"] % world == 0:
        # strong scaling: C2's 8 KV groups (and their 32 query heads) split over the ranks
        per = C2["Hkv"] // world
        sub = C2Problem(dev, seed=0, t_heads=t_heads, kv_groups=range(rank * per, (rank + 1) * per))
        tot_s, parts_s = time_c2(sub, args.steps, args.warmup, flush, barrier)
        ms_s = max_over_ranks([tot_s / args.steps], world, dev)[0]
        kept_all = torch.tensor([sub.kept], dtype=torch.float64, device=dev)
        import torch.distributed as dist
        dist.all_reduce(kept_all)
        flops_all = float(kept_all.item()) * 14 * C2["RB"] ** 2 * C2["D"]
        strong = {"kv_groups_per_gpu": per, "q_heads_per_gpu": sub.H, "ms_per_step": round(ms_s, 4),
                  "kept_tflops_whole_job": round(flops_all / (ms_s * 1e-3) / 1e12, 2),
                  "scaling": "strong: C2's heads split over the ranks by KV group, no collective"}
        del sub
        torch.cuda.empty_cache()

    if barrier:
        barrier()
    e2e_serial_ms, h2d, d2h = time_e2e(prob, max(3, args.steps // 2), 2)
    if barrier:
        barrier()
    e2e_ms, h2d_p, d2h_p = time_e2e_pipelined(prob, max(4, args.steps), 3)
    assert (h2d_p, d2h_p) == (h2d, d2h)
    e2e_ms, e2e_serial_ms = max_over_ranks([e2e_ms, e2e_serial_ms], world, dev)
    e2e_value = prob.flops_alg * world / (e2e_ms * 1e-3) / 1e12

    extras = {}
    if not args.quick:
        extras["sweep"] = run_sweep(dev, flush, steps=5)  # per GPU (rank 0's numbers)
        extras["c5"] = run_c5(dev, rank, world, max(3, args.steps // 2), args.warmup, flush, barrier,
                              cpu=not args.no_cpu)
        extras["c4"] = run_c4(dev, rank, world, 1, flush, barrier, cpu=not args.no_cpu)
        extras["decode"] = run_decode(dev, rank, args.steps, args.warmup, flush, peaks, world, rank,
                                      barrier, cpu=not args.no_cpu)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        torch.set_num_threads(os.cpu_count() or 1)
        heads = (0, 1)
        s, nh = cpu_reference_sample(heads, t_heads=t_heads)
        _, flops_h = kept_flops_c2(t_heads, True, True, heads=heads)
        cpu = {"value": flops_h / s / 1e12, "unit": "TFLOP/s",
               "cores": torch.get_num_threads(), "kind": "port", "measured_s": round(s, 3),
               "scale": round(prob.flops_alg / flops_h, 3),
               "whole_step_s_extrapolated": round(s * prob.flops_alg / flops_h, 2),
               "sample": f"masked dense fp32 attention fwd+bwd (autograd) on heads {list(heads)} of "
                         f"C2 at N=8192; value = the sample's kept-block FLOPs / its time"}

    ref_triton = None
    if rank == 0 and world == 1 and not args.quick and not args.no_reference_triton:
        prob.free_device()
        torch.cuda.empty_cache()
        ref_triton = run_reference_triton_subprocess()

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": config_c2(world, t_heads, prob.kept),
            "breakdown_ms": {p: round(v, 4) for p, v in parts.items()},
            "roofline": {"bound": "tensor", "kernel": kern, "achieved": round(achieved, 2),
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(achieved / peaks["bf16_tflops"], 4), "traffic": traffic,
                         "peak_source": f"{peak_kind} bf16 burst",
                         "flops_per_launch": prob.flops[kern],
                         "fwd": {"ms": round(parts["fwd"], 4),
                                 "tflops": round(prob.flops["fwd"] / (parts["fwd"] * 1e-3) / 1e12, 2),
                                 "hbm_gbs": round(prob.fwd_bytes / (parts["fwd"] * 1e-3) / 1e9, 1),
                                 "compulsory_bytes": prob.fwd_bytes}},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 3), "unit": "TFLOP/s", "ms_per_step": round(e2e_ms, 3),
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "ultrametric.block_list_attention autograd (ctypes -> C ABI)",
                    "pipelined": "upload of step i+1 and download of step i-1 overlap step i's "
                                 "compute on two copy streams; every step's copies inside the "
                                 "timed region",
                    "serial_ms_per_step": round(e2e_serial_ms, 3),
                    "serial_value": round(prob.flops_alg * world / (e2e_serial_ms * 1e-3) / 1e12, 3)},
            "clocks": clk.summary(),
            "gpu_launches": prob_launches * args.steps,
            "cuda_graph": graph,
            "two_kernel_backward": two_kernel,
            **extras,
        }
        if strong is not None:
            line["c2_strong"] = strong
        if ref_triton is not None:
            line["reference_triton"] = ref_triton
            _merge_reference_triton(line, ref_triton, ms_step)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--quick", action="store_true", help="headline only (no sweep / decode)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--decode-only", action="store_true",
                    help="profiling aid: time only the C3 routed decode")
    ap.add_argument("--no-reference-triton", action="store_true",
                    help="skip timing the reference's own Triton kernels on this GPU")
    ap.add_argument("--reference-triton-worker", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--threshold", type=int, default=None,
                    help="profiling aid: every head uses this LCA threshold instead of the seeded mix")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.reference_triton_worker:
        reference_triton_worker(args)
    elif args.impl == "reference":
        run_reference_arm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

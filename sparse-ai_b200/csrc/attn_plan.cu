// Planner and split-reduce kernels for the persistent tcgen05 attention kernels.
#include <string>

#include "attn_plan.cuh"

namespace sa {
namespace {

constexpr int kPlanThreads = 512;
constexpr int kBins = 128;
constexpr int kMinSplit = 16;  // never split a dK/dV item into chunks smaller than this

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Sizes as int32: the planner runs on one SM, where 64-bit divisions per item cost more
// than its memory traffic (launch_plan rejects item counts above INT32_MAX).
struct PlanArgs {
  int kind;
  int Z, H, Hkv, RB, NB, QT, items;
  const int32_t* counts;    // forward lists' counts (Z, H, NB)
  const int32_t* q_counts;  // transposed lists' counts (Z, H, NB)
  int ctas;
  int skip;  // items [0, skip) are not queued (the forward's first wave takes them directly)
  PlanPtrs plan;
  int* weights;
};

__device__ __forceinline__ int item_weight(const PlanArgs& a, int item) {
  if (a.kind == kPlanDkdv) {
    const int zg_total = a.Z * a.Hkv;
    const int kt = item / zg_total, zg = item - kt * zg_total;
    const int z = zg / a.Hkv, hk = zg - z * a.Hkv;
    const int kb = kt * 128 / a.RB;
    const int group = a.H / a.Hkv;
    int n = 0;
    for (int h = hk * group; h < (hk + 1) * group; ++h) n += a.q_counts[((int64_t)z * a.H + h) * a.NB + kb];
    return n * (a.RB / 64);
  }
  const int zh_total = a.Z * a.H;
  const int qi = item / zh_total, zh = item - qi * zh_total;
  const int qb = (a.QT - 1 - qi) * 128 / a.RB;
  const int c = a.counts[(int64_t)zh * a.NB + qb];
  return c * (a.RB / (a.kind == kPlanFwd ? 128 : 64));
}

// Heavier work -> smaller bin (4 bins per octave).
__device__ __forceinline__ int weight_bin(int w) {
  const unsigned x = (unsigned)w + 1u;
  const int e = 31 - __clz(x);
  const int frac = e >= 2 ? (int)((x >> (e - 2)) & 3u) : (int)((x << (2 - e)) & 3u);
  const int key = min(e * 4 + frac, kBins - 1);
  return kBins - 1 - key;
}

constexpr int kPlanWarps = kPlanThreads / 32;

// Counting sort of the items by weight bin: per-warp histograms in shared memory (no
// cross-warp contention), one exclusive scan over [bin][warp] in bin order, then each item
// takes its queue slots with an atomic on its warp's cursor.  The order inside a bin does
// not matter: items write disjoint outputs and split items are reduced in chunk order.
__global__ void __launch_bounds__(kPlanThreads) plan_kernel(PlanArgs a) {
  // a kernel launched as this grid's programmatic dependent may start now; it waits for this
  // grid (griddepcontrol.wait) before it reads the queue
  pdl_trigger();
  // Items skip + tid + k * blockDim for k < kRegItems keep their weight in registers; larger
  // item counts spill the rest to a.weights.  Every pass over the items is one coalesced sweep.
  constexpr int kRegItems = 8;
  __shared__ int s_cnt[kBins][kPlanWarps];  // counts, then cursors
  __shared__ int s_wsum[kPlanWarps];
  __shared__ unsigned long long s_total;
  __shared__ int s_wmin, s_wmax;
  __shared__ int s_slots, s_nsplit, s_entries;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthr = blockDim.x;
  for (int b = tid; b < kBins * kPlanWarps; b += nthr) (&s_cnt[0][0])[b] = 0;
  if (tid == 0) {
    s_total = 0;
    s_wmin = 0x7fffffff;
    s_wmax = 0;
    s_slots = 0;
    s_nsplit = 0;
    s_entries = 0;
  }
  __syncthreads();
  int wreg[kRegItems];
  unsigned long long tot = 0;
#pragma unroll
  for (int k = 0; k < kRegItems; ++k) {  // independent loads, all in flight together
    const int i = a.skip + tid + k * nthr;
    wreg[k] = i < a.items ? item_weight(a, i) : 0;
    tot += (unsigned long long)wreg[k];
  }
  for (int i = a.skip + tid + kRegItems * nthr; i < a.items; i += nthr) {
    const int w = item_weight(a, i);
    a.weights[i] = w;
    tot += (unsigned long long)w;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
  if (lane == 0) atomicAdd(&s_total, tot);
  {  // weight range: with every weight equal the sort is the identity
    int wmin = 0x7fffffff, wmax = 0;
#pragma unroll
    for (int k = 0; k < kRegItems; ++k)
      if (a.skip + tid + k * nthr < a.items) {
        wmin = min(wmin, wreg[k]);
        wmax = max(wmax, wreg[k]);
      }
    for (int i = a.skip + tid + kRegItems * nthr; i < a.items; i += nthr) {
      wmin = min(wmin, a.weights[i]);
      wmax = max(wmax, a.weights[i]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      wmin = min(wmin, __shfl_xor_sync(0xffffffffu, wmin, o));
      wmax = max(wmax, __shfl_xor_sync(0xffffffffu, wmax, o));
    }
    if (lane == 0) {
      atomicMin(&s_wmin, wmin);
      atomicMax(&s_wmax, wmax);
    }
  }
  __syncthreads();
  int T = 0x7fffffff;
  if (a.kind == kPlanDkdv) {
    const unsigned long long t = (s_total + a.ctas - 1) / (unsigned long long)a.ctas;
    T = (int)max((unsigned long long)kMinSplit, t);
  }
  // All weights equal and none to split (very sparse lists: every item one key tile): the
  // heaviest-first order is the index order, so the queue is left unwritten and the kernels
  // hand out items skip + k directly; the sort's latency would otherwise sit in front of the
  // consumers' second fetch.
  if (s_wmin == s_wmax && s_wmax <= T) {
    if (tid == 0) {
      a.plan.header->counter = 0;
      a.plan.header->n_entries = a.items > a.skip ? a.items - a.skip : 0;
      a.plan.header->n_split = 0;
      a.plan.header->natural = 1 + s_wmax;  // nonzero; the forward reads the weight back
    }
    return;
  }
  auto chunks_of = [&](int w) { return w > T ? (w + T - 1) / T : 1; };
  auto bin_of = [&](int w, int chunks) { return weight_bin((w + chunks - 1) / chunks); };
  // ---- per-warp histograms
#pragma unroll
  for (int k = 0; k < kRegItems; ++k) {
    const int i = a.skip + tid + k * nthr;
    if (i < a.items) {
      const int c = chunks_of(wreg[k]);
      atomicAdd(&s_cnt[bin_of(wreg[k], c)][warp], c);
    }
  }
  for (int i = a.skip + tid + kRegItems * nthr; i < a.items; i += nthr) {
    const int w = a.weights[i], c = chunks_of(w);
    atomicAdd(&s_cnt[bin_of(w, c)][warp], c);
  }
  __syncthreads();
  // ---- exclusive scan over the flat [bin][warp] array (heavy bins first)
  {
    constexpr int kPer = kBins * kPlanWarps / kPlanThreads;
    int* flat = &s_cnt[0][0];
    int v[kPer], sum = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      v[j] = flat[tid * kPer + j];
      sum += v[j];
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) s_wsum[warp] = incl;
    __syncthreads();
    int base = 0;
    for (int q = 0; q < warp; ++q) base += s_wsum[q];
    int run = base + incl - sum;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      flat[tid * kPer + j] = run;
      run += v[j];
    }
    if (tid == nthr - 1) s_entries = run;
  }
  __syncthreads();
  // ---- scatter
  auto scatter_one = [&](int i, int w) {
    const int chunks = chunks_of(w);
    int slot_base = -1;
    if (chunks > 1) {  // rare: at most one split item per CTA of the kernel
      slot_base = atomicAdd(&s_slots, chunks);
      const int k = atomicAdd(&s_nsplit, 1);
      a.plan.splits[k] = SplitItem{i, slot_base, chunks, 0};
    }
    const int pos0 = atomicAdd(&s_cnt[bin_of(w, chunks)][warp], chunks);
    for (int c = 0; c < chunks; ++c) {
      const int b0 = (int)((int64_t)w * c / chunks), b1 = (int)((int64_t)w * (c + 1) / chunks);
      a.plan.queue[pos0 + c] = WorkEntry{i, b0, b1, slot_base < 0 ? -1 : slot_base + c};
    }
  };
#pragma unroll
  for (int k = 0; k < kRegItems; ++k) {
    const int i = a.skip + tid + k * nthr;
    if (i < a.items) scatter_one(i, wreg[k]);
  }
  for (int i = a.skip + tid + kRegItems * nthr; i < a.items; i += nthr) scatter_one(i, a.weights[i]);
  __syncthreads();
  if (tid == 0) {
    a.plan.header->counter = 0;
    a.plan.header->n_entries = s_entries;
    a.plan.header->n_split = s_nsplit;
    a.plan.header->natural = 0;
  }
}

// grid (ctas, kReduceSlices): block (k, s) sums, in chunk order, rows [s * R, (s + 1) * R) of
// split item k's chunk partials (if item k exists), four chunks' loads in flight at a time.
constexpr int kReduceSlices = 16;

template <int D>
__global__ void __launch_bounds__(256) dkdv_reduce_kernel(AttnParams p, PlanPtrs plan) {
  const int k = blockIdx.x;
  if (k >= plan.header->n_split) return;
  const SplitItem si = plan.splits[k];
  const int64_t zg_total = p.Z * p.Hkv;
  const int64_t kt = si.item / zg_total, zg = si.item % zg_total;
  const int64_t z = zg / p.Hkv, hk = zg % p.Hkv;
  const int64_t k0 = kt * 128;
  constexpr int RS = 2 * D;                 // a partial row: dV[D] then dK[D]
  constexpr int R = 128 / kReduceSlices;    // rows of this block
  const bool bf = p.dtype == SA_BF16;
  const int64_t cstride = (int64_t)128 * RS;  // floats between consecutive chunks
  for (int e = threadIdx.x * 4; e < R * RS; e += blockDim.x * 4) {
    const int r = blockIdx.y * R + e / RS, c = e % RS;
    const float* src = plan.partials + ((int64_t)si.slot_base * 128 + r) * RS + c;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int ch0 = 0; ch0 < si.chunks; ch0 += 4) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        v[u] = ch0 + u < si.chunks ? *reinterpret_cast<const float4*>(src + (ch0 + u) * cstride)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 4; ++u) {  // chunk order kept: deterministic sums
        acc.x += v[u].x;
        acc.y += v[u].y;
        acc.z += v[u].z;
        acc.w += v[u].w;
      }
    }
    const int64_t key = k0 + r;
    if (key >= p.N) continue;
    const bool is_k = c >= D;
    const int col = is_k ? c - D : c;
    uint16_t* dst = static_cast<uint16_t*>(is_k ? p.dk : p.dv) +
                    z * (is_k ? p.dks[0] : p.dvs[0]) + hk * (is_k ? p.dks[1] : p.dvs[1]) +
                    key * (is_k ? p.dks[2] : p.dvs[2]) + col;
    const float f[4] = {acc.x, acc.y, acc.z, acc.w};
    uint16_t h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (bf) {
        const __nv_bfloat16 b = __float2bfloat16_rn(f[i]);
        h[i] = *reinterpret_cast<const uint16_t*>(&b);
      } else {
        const __half b = __float2half_rn(f[i]);
        h[i] = *reinterpret_cast<const uint16_t*>(&b);
      }
    }
    *reinterpret_cast<uint2*>(dst) = make_uint2(h[0] | ((uint32_t)h[1] << 16), h[2] | ((uint32_t)h[3] << 16));
  }
}

}  // namespace

int64_t plan_workspace_bytes(int kind, int64_t items, int ctas, int64_t D) {
  size_t b = 256;                                                 // header
  b += align256((size_t)(items + 2 * ctas) * sizeof(WorkEntry));  // queue
  b += align256((size_t)(ctas + 1) * sizeof(SplitItem));          // split items
  b += align256((size_t)items * sizeof(int));                     // weights
  if (kind == kPlanDkdv) b += align256((size_t)2 * ctas * 128 * 2 * D * sizeof(float));
  return (int64_t)b;
}

PlanPtrs plan_carve(void* ws, int kind, int64_t items, int ctas, int64_t D) {
  char* w = static_cast<char*>(ws);
  PlanPtrs p{};
  p.header = reinterpret_cast<PlanHeader*>(w);
  w += 256;
  p.queue = reinterpret_cast<WorkEntry*>(w);
  w += align256((size_t)(items + 2 * ctas) * sizeof(WorkEntry));
  p.splits = reinterpret_cast<SplitItem*>(w);
  w += align256((size_t)(ctas + 1) * sizeof(SplitItem));
  w += align256((size_t)items * sizeof(int));  // weights (the planner finds them below)
  p.partials = kind == kPlanDkdv ? reinterpret_cast<float*>(w) : nullptr;
  return p;
}

int launch_plan(int kind, const AttnParams& p, int64_t items, int ctas, const PlanPtrs& plan,
                cudaStream_t stream, int skip) {
  if (items > INT32_MAX || p.Z * p.H * p.NB > INT32_MAX)
    return fail(SA_EUNSUPPORTED, "too many work items");
  PlanArgs a{};
  a.kind = kind;
  a.Z = (int)p.Z;
  a.H = (int)p.H;
  a.Hkv = (int)p.Hkv;
  a.RB = (int)p.RB;
  a.NB = (int)p.NB;
  a.QT = (int)((p.N + 127) / 128);
  a.items = (int)items;
  a.counts = p.counts;
  a.q_counts = p.q_counts;
  a.ctas = ctas;
  a.skip = skip;
  a.plan = plan;
  a.weights = reinterpret_cast<int*>(reinterpret_cast<char*>(plan.splits) +
                                     align256((size_t)(ctas + 1) * sizeof(SplitItem)));
  plan_kernel<<<1, kPlanThreads, 0, stream>>>(a);
  return check_launch("plan_kernel");
}

int launch_dkdv_reduce(const AttnParams& p, const PlanPtrs& plan, int ctas, cudaStream_t stream) {
  const dim3 grid((unsigned)ctas, kReduceSlices);
  if (p.D == 64)
    dkdv_reduce_kernel<64><<<grid, 256, 0, stream>>>(p, plan);
  else if (p.D == 128)
    dkdv_reduce_kernel<128><<<grid, 256, 0, stream>>>(p, plan);
  else
    return fail(SA_EUNSUPPORTED, "dkdv reduce: head_dim");
  return check_launch("dkdv_reduce_kernel");
}

}  // namespace sa

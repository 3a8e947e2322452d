// Planner and split-reduce kernels for the persistent tcgen05 attention kernels.
#include <string>

#include "attn_plan.cuh"

namespace sa {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kBins = 128;
constexpr int kMinSplit = 16;  // never split a dK/dV item into chunks smaller than this

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct PlanArgs {
  int kind;
  int64_t Z, H, Hkv, RB, NB, QT, items;
  const int32_t* counts;    // forward lists' counts (Z, H, NB)
  const int32_t* q_counts;  // transposed lists' counts (Z, H, NB)
  int ctas;
  PlanPtrs plan;
  int* weights;
};

__device__ __forceinline__ int item_weight(const PlanArgs& a, int64_t item) {
  if (a.kind == kPlanDkdv) {
    const int64_t zg_total = a.Z * a.Hkv;
    const int64_t kt = item / zg_total, zg = item % zg_total;
    const int64_t z = zg / a.Hkv, hk = zg % a.Hkv;
    const int64_t kb = kt * 128 / a.RB;
    const int64_t group = a.H / a.Hkv;
    int n = 0;
    for (int64_t h = hk * group; h < (hk + 1) * group; ++h) n += a.q_counts[(z * a.H + h) * a.NB + kb];
    return n * (int)(a.RB / 64);
  }
  const int64_t zh_total = a.Z * a.H;
  const int64_t qt = a.QT - 1 - item / zh_total, zh = item % zh_total;
  const int64_t qb = qt * 128 / a.RB;
  const int c = a.counts[zh * a.NB + qb];
  return c * (int)(a.RB / (a.kind == kPlanFwd ? 128 : 64));
}

// Heavier work -> smaller bin (4 bins per octave).
__device__ __forceinline__ int weight_bin(int w) {
  const unsigned x = (unsigned)w + 1u;
  const int e = 31 - __clz(x);
  const int frac = e >= 2 ? (int)((x >> (e - 2)) & 3u) : (int)((x << (2 - e)) & 3u);
  const int key = min(e * 4 + frac, kBins - 1);
  return kBins - 1 - key;
}

// atomicAdd(&ctr[bin], n) aggregated over the lanes of a warp that share `bin`; returns this
// lane's base (lanes of a group get consecutive ranges in lane order).  Avoids serialising
// hundreds of shared-memory atomics on one address when most items share a bin.
__device__ __forceinline__ int warp_bin_add(int* ctr, int bin, int n) {
  const unsigned peers = __match_any_sync(__activemask(), bin);
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(peers) - 1;
  int incl = n;  // inclusive prefix of n over the lower lanes of the group
  int total = 0;
  for (unsigned m = peers; m; m &= m - 1) {
    const int l = __ffs(m) - 1;
    const int v = __shfl_sync(peers, n, l);
    total += v;
    if (l < lane) incl += v;
  }
  int base = 0;
  if (lane == leader) base = atomicAdd(&ctr[bin], total);
  base = __shfl_sync(peers, base, leader);
  return base + incl - n;
}

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(PlanArgs a) {
  __shared__ int s_hist[kBins];
  __shared__ int s_cursor[kBins];
  __shared__ unsigned long long s_total;
  __shared__ int s_slots, s_nsplit, s_entries;
  const int tid = threadIdx.x;
  for (int b = tid; b < kBins; b += blockDim.x) s_hist[b] = 0;
  if (tid == 0) {
    s_total = 0;
    s_slots = 0;
    s_nsplit = 0;
    s_entries = 0;
  }
  __syncthreads();
  unsigned long long tot = 0;
  for (int64_t i = tid; i < a.items; i += blockDim.x) {
    const int w = item_weight(a, i);
    a.weights[i] = w;
    tot += (unsigned long long)w;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
  if ((tid & 31) == 0) atomicAdd(&s_total, tot);
  __syncthreads();
  int T = 0x7fffffff;
  if (a.kind == kPlanDkdv) {
    const unsigned long long t = (s_total + a.ctas - 1) / (unsigned long long)a.ctas;
    T = (int)max((unsigned long long)kMinSplit, t);
  }
  // histogram of entries by chunk weight (warp-uniform trip count for the warp atomics)
  for (int64_t i0 = 0; i0 < a.items; i0 += blockDim.x) {
    const int64_t i = i0 + tid;
    if (i < a.items) {
      const int w = a.weights[i];
      const int chunks = w > T ? (w + T - 1) / T : 1;
      const int wc = (w + chunks - 1) / chunks;
      warp_bin_add(s_hist, weight_bin(wc), chunks);
    }
  }
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int b = 0; b < kBins; ++b) {
      s_cursor[b] = run;
      run += s_hist[b];
    }
    s_entries = run;
  }
  __syncthreads();
  for (int64_t i0 = 0; i0 < a.items; i0 += blockDim.x) {
    const int64_t i = i0 + tid;
    if (i >= a.items) continue;
    const int w = a.weights[i];
    const int chunks = w > T ? (w + T - 1) / T : 1;
    const int wc = (w + chunks - 1) / chunks;
    const int bin = weight_bin(wc);
    int slot_base = -1;
    if (chunks > 1) {  // rare: at most one split item per CTA of the kernel
      slot_base = atomicAdd(&s_slots, chunks);
      const int k = atomicAdd(&s_nsplit, 1);
      a.plan.splits[k] = SplitItem{(int)i, slot_base, chunks, 0};
    }
    const int pos0 = warp_bin_add(s_cursor, bin, chunks);
    for (int c = 0; c < chunks; ++c) {
      const int b0 = (int)((int64_t)w * c / chunks), b1 = (int)((int64_t)w * (c + 1) / chunks);
      a.plan.queue[pos0 + c] = WorkEntry{(int)i, b0, b1, slot_base < 0 ? -1 : slot_base + c};
    }
  }
  __syncthreads();
  if (tid == 0) {
    a.plan.header->counter = 0;
    a.plan.header->n_entries = s_entries;
    a.plan.header->n_split = s_nsplit;
  }
}

// grid = ctas blocks; block k sums the chunks of split item k (if any) in chunk order.
template <int D>
__global__ void __launch_bounds__(256) dkdv_reduce_kernel(AttnParams p, PlanPtrs plan) {
  const int k = blockIdx.x;
  if (k >= plan.header->n_split) return;
  const SplitItem si = plan.splits[k];
  const int64_t zg_total = p.Z * p.Hkv;
  const int64_t kt = si.item / zg_total, zg = si.item % zg_total;
  const int64_t z = zg / p.Hkv, hk = zg % p.Hkv;
  const int64_t k0 = kt * 128;
  constexpr int RS = 2 * D;  // a partial row: dV[D] then dK[D]
  const bool bf = p.dtype == SA_BF16;
  for (int e = threadIdx.x * 4; e < 128 * RS; e += blockDim.x * 4) {
    const int r = e / RS, c = e % RS;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int ch = 0; ch < si.chunks; ++ch) {
      const float4 v = *reinterpret_cast<const float4*>(
          plan.partials + ((int64_t)(si.slot_base + ch) * 128 + r) * RS + c);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    const int64_t key = k0 + r;
    if (key >= p.N) continue;
    const bool is_k = c >= D;
    const int col = is_k ? c - D : c;
    uint16_t* dst = static_cast<uint16_t*>(is_k ? p.dk : p.dv) +
                    z * (is_k ? p.dks[0] : p.dvs[0]) + hk * (is_k ? p.dks[1] : p.dvs[1]) +
                    key * (is_k ? p.dks[2] : p.dvs[2]) + col;
    const float f[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (bf) {
        const __nv_bfloat16 h = __float2bfloat16_rn(f[i]);
        dst[i] = *reinterpret_cast<const uint16_t*>(&h);
      } else {
        const __half h = __float2half_rn(f[i]);
        dst[i] = *reinterpret_cast<const uint16_t*>(&h);
      }
    }
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
                cudaStream_t stream) {
  PlanArgs a{};
  a.kind = kind;
  a.Z = p.Z;
  a.H = p.H;
  a.Hkv = p.Hkv;
  a.RB = p.RB;
  a.NB = p.NB;
  a.QT = (p.N + 127) / 128;
  a.items = items;
  a.counts = p.counts;
  a.q_counts = p.q_counts;
  a.ctas = ctas;
  a.plan = plan;
  a.weights = reinterpret_cast<int*>(reinterpret_cast<char*>(plan.splits) +
                                     align256((size_t)(ctas + 1) * sizeof(SplitItem)));
  if (items > INT32_MAX) return fail(SA_EUNSUPPORTED, "too many work items");
  plan_kernel<<<1, kPlanThreads, 0, stream>>>(a);
  return check_launch("plan_kernel");
}

int launch_dkdv_reduce(const AttnParams& p, const PlanPtrs& plan, int ctas, cudaStream_t stream) {
  if (p.D == 64)
    dkdv_reduce_kernel<64><<<ctas, 256, 0, stream>>>(p, plan);
  else if (p.D == 128)
    dkdv_reduce_kernel<128><<<ctas, 256, 0, stream>>>(p, plan);
  else
    return fail(SA_EUNSUPPORTED, "dkdv reduce: head_dim");
  return check_launch("dkdv_reduce_kernel");
}

}  // namespace sa

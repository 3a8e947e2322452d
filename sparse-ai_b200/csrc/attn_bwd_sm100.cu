// Block-list attention backward on sm_100a: TMA + tcgen05 (TMEM accumulators).
//
// Same semantics as src/ultrametric/block_list.py:494-584 (dQ) and :586-681 (dK/dV) of
// sparse-ai: P = exp2(s*scale*log2e + bias*log2e - lse*log2e) on the visible (row, key)
// pairs, dS = P * (dP - Delta), dQ = scale * dS K, dK = scale * dS^T Q, dV = P^T dO,
// d_soft_bias[z,h,qb,t] = sum of the unscaled dS of the block pair.
//
// Both kernels are persistent (one CTA per SM, work from the planner's queue), 10 warps (the
// fused kernel below adds an eleventh, its second MMA issuer):
//   warp 0      TMA producer (and the queue fetch)
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer
//   warps 2-9   two elementwise groups of 4 warps (a thread owns one TMEM lane = row); the
//               groups ping-pong over the streamed sub-tiles (group = sub-tile index % 2), so
//               one group's TMEM loads and exp2 overlap the other's
//
// dQ kernel:   work item = (128-row query tile, z, h); Q and dO tiles resident; the listed
//              key blocks stream as 64-key sub-tiles (K and V) through a 4-stage ring.
//                S[b]  = Q  K_j^T  (M=128, N=64, K=D)     b = j % 2 (TMEM double buffer)
//                dP[b] = dO V_j^T  (M=128, N=64, K=D)
//                dQ   += dS_j K_j  (M=128, N=D, K=64)     dS_j (bf16 pairs) written back
//                                                         into TMEM over S[b]: A from TMEM
// dK/dV kernel: work item = (128-key tile, z, KV head) or a chunk of a heavy one (fp32
//              partials, summed by dkdv_reduce_kernel); K and V tiles resident; for every
//              query head of the GQA group and every query block of its transposed list,
//              64-row sub-tiles of Q, dO and their row stats stream through a 4-stage ring.
//                S^T[b]  = K Q_i^T  (M=128, N=64, K=D)
//                dP^T[b] = V dO_i^T (M=128, N=64, K=D)
//                dV     += P^T_i dO_i (M=128, N=D, K=64)  P^T (bf16) in TMEM over S^T[b]
//                dK     += dS^T_i Q_i (M=128, N=D, K=64)  dS^T (bf16) in TMEM over dP^T[b]
// The elementwise warps never rescale: the forward's LSE is final.
#include <string>
#include <type_traits>

#include "sched.cuh"

namespace sa {
namespace {

constexpr int kRows = 128;  // resident tile rows (TMEM lanes)
constexpr int kSub = 64;    // streamed sub-tile rows
constexpr int kStages = 4;    // streamed ring depth (dQ kernel)
constexpr int kKvStages = 4;  // streamed ring depth (dK/dV kernel)
constexpr int kEw = 8;                      // elementwise warps: 2 per TMEM lane quarter
constexpr int kEwThreads = kEw * 32;
constexpr int kBwdThreads = 64 + kEwThreads;
// fused backward: producer (warp 0), A-block MMA issuer (warp 1), the two elementwise groups
// (warps 2-9) and the B-block MMA issuer (warp 10)
constexpr int kFuThreads = 96 + kEwThreads;
constexpr int kFuBWarp = 2 + kEw;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColP = 128, kColAcc = 256;  // S[2]: 0/64, dP[2]: 128/192

struct BwdArgs {
  CUtensorMap tm_q, tm_do, tm_k, tm_v, tm_dq;
  int64_t Z, H, Hkv, N, RB, NB, tiles;
  const int32_t* lists;
  int64_t list_stride;
  const int32_t* counts;
  const int32_t* k_lists;  // (Z, H, NB, NB) transposed lists
  const int32_t* k_slots;
  const int32_t* q_counts;
  const float* lse;
  const float* delta;
  const void* bias;
  int bias_dtype;
  int64_t bs[4];
  float* dbias;
  const float* stats;  // (Z*H, ceil(N/64), {lse*log2e[64], delta[64]})
  void* dq;
  int64_t dqs[4];
  void* dk;
  int64_t dks[4];
  void* dv;
  int64_t dvs[4];
  int causal;
  float scale;
  unsigned* status;
  SchedArgs sched;
  float* partials;  // dK/dV: fp32 [slot][128][dV D | dK D] for split chunks
  float* dq_acc;  // fused kernel: fp32 dQ accumulator (Z*H, N, D) contiguous, zeroed
};

__device__ __forceinline__ uint32_t pack2(float lo, float hi, bool bf16) {
  uint32_t r;
  if (bf16)
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float bias_log2(const BwdArgs& a, int64_t z, int64_t h, int64_t qb,
                                           int64_t slot) {
  if (!a.bias) return 0.f;
  return load_any_f32(a.bias, a.bias_dtype, z * a.bs[0] + h * a.bs[1] + qb * a.bs[2] + slot * a.bs[3]) *
         kLog2e;
}

// Store NC consecutive TMEM columns (starting at taddr) of one row, as bf16/fp16, to
// base[z, h, row, c0 : c0 + NC].
template <int NC>
__device__ __forceinline__ void store_cols(void* base, const int64_t* st, int64_t z, int64_t h,
                                           int64_t row, int c0, uint32_t taddr, bool bf16,
                                           bool valid, bool zero) {
  using T = __nv_bfloat16;  // both half types are 2 bytes; pack2 picks the format
  T* dst = static_cast<T*>(base) + z * st[0] + h * st[1] + row * st[2] + c0;
#pragma unroll
  for (int c = 0; c < NC / 32; ++c) {
    float o[32];
    if (!zero) {
      tmem_ld32(taddr + c * 32, o);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = 0.f;
    }
    if (valid) {
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        uint4 w;
        w.x = pack2(o[v * 8 + 0], o[v * 8 + 1], bf16);
        w.y = pack2(o[v * 8 + 2], o[v * 8 + 3], bf16);
        w.z = pack2(o[v * 8 + 4], o[v * 8 + 5], bf16);
        w.w = pack2(o[v * 8 + 6], o[v * 8 + 7], bf16);
        *reinterpret_cast<uint4*>(dst + c * 32 + v * 8) = w;
      }
    }
  }
}

// Per streamed stage: what the producer read from the lists, handed to the elementwise
// warps through shared memory (released by the stage's full mbarrier), so that no consumer
// reads the lists from global memory on its critical path.
struct StageMeta {
  int64_t start;  // first key (dQ kernel) or first query (dK/dV kernel) of the sub-tile
  float b2;       // soft-bias * log2(e) of the block pair
  int pad;
};

__device__ __forceinline__ void init_bars(uint64_t* bars, const uint32_t* counts, int n) {
  for (int i = 0; i < n; ++i) mbar_init(&bars[i], counts[i]);
  fence_mbar_init();
}

// =======================================================================================
// dQ kernel
// =======================================================================================
template <int D>
struct DqLayout {
  static constexpr uint32_t kQ = 0;                          // [128][D]
  static constexpr uint32_t kDO = kRows * D * 2;             // [128][D]
  static constexpr uint32_t kKV = 2 * kRows * D * 2;         // stages x (K [64][D], V [64][D])
  static constexpr uint32_t kStage = 2 * kSub * D * 2;
  static constexpr uint32_t kOut = kKV + kStages * kStage;  // dQ staging: D/64 boxes [128][64]
  static constexpr uint32_t kBars = kOut + kRows * D * 2;
  static constexpr uint32_t kMeta = kBars + 256;  // StageMeta[kStages]
  static constexpr uint32_t kRingOff = kMeta + 128;  // WorkEntry[kRing]
  static constexpr uint32_t kAlloc = kRingOff + 128 + 1024;
  static_assert(kAlloc <= 232448, "dQ shared-memory layout too large");
};

enum { DQ_QFULL = 0, DQ_QEMPTY, DQ_KVFULL0, DQ_KVEMPTY0 = DQ_KVFULL0 + kStages,
       DQ_SFULL0 = DQ_KVEMPTY0 + kStages, DQ_DSFULL0 = DQ_SFULL0 + 2, DQ_DONE = DQ_DSFULL0 + 2,
       DQ_OFULL, DQ_ODRAIN, DQ_WFULL0,
       DQ_WEMPTY0 = DQ_WFULL0 + kRing, DQ_NUM = DQ_WEMPTY0 + kRing };

struct DqItem {
  int64_t z, h, hk, q_start, qb, row_id;
};

__device__ __forceinline__ DqItem dq_item(const BwdArgs& a, int64_t item) {
  DqItem it;
  const int64_t zh_total = a.Z * a.H;
  const int64_t qt = a.tiles - 1 - item / zh_total;
  const int64_t zh = item % zh_total;
  it.z = zh / a.H;
  it.h = zh % a.H;
  it.hk = it.h / (a.H / a.Hkv);
  it.q_start = qt * kRows;
  it.qb = it.q_start / a.RB;
  it.row_id = zh * a.NB + it.qb;
  return it;
}

// 64-key sub-tiles of a dQ item: the static-schedule weight.
__device__ __forceinline__ int dq_item_tiles(const BwdArgs& a, int64_t item) {
  return a.counts[dq_item(a, item).row_id] * (int)(a.RB / kSub);
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kBwdThreads, 1) bwd_dq_sm100_kernel(const __grid_constant__ BwdArgs a) {
  using L = DqLayout<D>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::kBars);
  StageMeta* meta = reinterpret_cast<StageMeta*>(sm + L::kMeta);
  WorkEntry* ring = reinterpret_cast<WorkEntry*>(sm + L::kRingOff);
  __shared__ uint32_t s_tmem;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int spb = (int)(a.RB / kSub);

  if (threadIdx.x == 0) {
    uint32_t cnt[DQ_NUM];
    for (int i = 0; i < DQ_NUM; ++i) cnt[i] = 1;
    cnt[DQ_DSFULL0] = cnt[DQ_DSFULL0 + 1] = kEwThreads / 2;  // one group per buffer
    cnt[DQ_OFULL] = kEwThreads;  // the dQ tile is staged for its TMA store
    for (int i = 0; i < kRing; ++i) cnt[DQ_WEMPTY0 + i] = 1 + kEwThreads;
    init_bars(bars, cnt, DQ_NUM);
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&a.tm_q);
      prefetch_tmap(&a.tm_do);
      prefetch_tmap(&a.tm_k);
      prefetch_tmap(&a.tm_v);
      uint32_t kv = 0, jq = 0;
      bool ok = true;
      auto weight = [&](int64_t i) { return dq_item_tiles(a, i); };
      WorkFetcher fetch;
      fetch.init(&a.sched, weight);
      for (uint32_t w = 0; ok; ++w) {
        const WorkEntry e = fetch.next(weight);
        if (!(ok = ring_put(ring, &bars[DQ_WFULL0], &bars[DQ_WEMPTY0], w, e, a.status))) break;
        if (e.item < 0) break;
        const DqItem it = dq_item(a, e.item);
        if (e.end == e.begin) {
          fetch.reserve(weight);
          continue;
        }
        if (!(ok = mbar_wait(&bars[DQ_QEMPTY], (jq & 1) ^ 1, a.status))) break;
        ++jq;
        mbar_arrive_expect_tx(&bars[DQ_QFULL], 2 * kRows * D * 2);
        for (int c = 0; c < D / 64; ++c) {
          tma_load_4d(sm + L::kQ + c * kRows * 128, &a.tm_q, &bars[DQ_QFULL], c * 64,
                      (int)it.q_start, (int)it.h, (int)it.z);
          tma_load_4d(sm + L::kDO + c * kRows * 128, &a.tm_do, &bars[DQ_QFULL], c * 64,
                      (int)it.q_start, (int)it.h, (int)it.z);
        }
        const int32_t* lst = a.lists + it.row_id * a.list_stride;
        for (int j = e.begin; j < e.end && ok; ++j, ++kv) {
          const int64_t k0 = (int64_t)lst[j / spb] * a.RB + (j % spb) * kSub;
          const uint32_t st = kv % kStages, ph = (kv / kStages) & 1;
          if (!(ok = mbar_wait(&bars[DQ_KVEMPTY0 + st], ph ^ 1, a.status))) break;
          unsigned char* stage = sm + L::kKV + st * L::kStage;
          meta[st].start = k0;
          meta[st].b2 = bias_log2(a, it.z, it.h, it.qb, j / spb);
          mbar_arrive_expect_tx(&bars[DQ_KVFULL0 + st], L::kStage);
          for (int c = 0; c < D / 64; ++c) {
            tma_load_4d(stage + c * kSub * 128, &a.tm_k, &bars[DQ_KVFULL0 + st], c * 64, (int)k0,
                        (int)it.hk, (int)it.z);
            tma_load_4d(stage + kSub * D * 2 + c * kSub * 128, &a.tm_v, &bars[DQ_KVFULL0 + st],
                        c * 64, (int)k0, (int)it.hk, (int)it.z);
          }
          if (j == e.end - 1) fetch.reserve(weight);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16(kRows, kSub, BF16, false, false);
      constexpr uint32_t id_dq = idesc_f16(kRows, D, BF16, false, true);
      const uint32_t q_addr = smem_u32(sm + L::kQ), do_addr = smem_u32(sm + L::kDO);
      uint32_t kv = 0, s_it = 0, ds_it = 0, jq = 0;
      bool ok = true;
      auto issue_dq = [&](uint32_t kv_u, bool first) -> bool {
        const uint32_t db = ds_it & 1, dph = (ds_it >> 1) & 1;
        if (!mbar_wait(&bars[DQ_DSFULL0 + db], dph, a.status)) return false;
        tc_fence_after();
        const uint32_t st = kv_u % kStages;
        const uint32_t k_addr = smem_u32(sm + L::kKV + st * L::kStage);
        // dS (bf16 pairs) sits in TMEM over the S columns of buffer db
#pragma unroll
        for (int kk = 0; kk < kSub / 16; ++kk)
          tc_mma_f16_ts(tmem + kColAcc, tmem + kColS + db * kSub + kk * 8,
                        smem_desc(k_addr + kk * 16 * 128, kSub * 128, 1024), id_dq,
                        (!first || kk > 0) ? 1u : 0u);
        tc_commit(&bars[DQ_KVEMPTY0 + st]);
        ++ds_it;
        return true;
      };
      for (uint32_t w = 0; ok; ++w) {
        WorkEntry e;
        if (!(ok = ring_get(ring, &bars[DQ_WFULL0], &bars[DQ_WEMPTY0], w, e, a.status))) break;
        if (e.item < 0) break;
        const int n_sub = e.end - e.begin;
        if (n_sub == 0) continue;
        if (!(ok = mbar_wait(&bars[DQ_QFULL], jq & 1, a.status))) break;
        ++jq;
        const uint32_t kv0 = kv;
        for (int j = 0; j < n_sub && ok; ++j, ++kv) {
          const uint32_t st = kv % kStages, ph = (kv / kStages) & 1;
          const uint32_t sb = s_it & 1;
          // TMEM buffer sb is reusable: the dQ MMA of sub-tile s_it - 2 (which reads its dS)
          // was issued after its DSFULL wait, before this point, in MMA issue order
          if (!(ok = mbar_wait(&bars[DQ_KVFULL0 + st], ph, a.status))) break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sm + L::kKV + st * L::kStage);
          const uint32_t v_addr = k_addr + kSub * D * 2;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t oa = (kk >> 2) * (kRows * 128) + (kk & 3) * 32;
            const uint32_t ob = (kk >> 2) * (kSub * 128) + (kk & 3) * 32;
            tc_mma_f16(tmem + kColS + sb * kSub, smem_desc(q_addr + oa, 16, 1024),
                       smem_desc(k_addr + ob, 16, 1024), id_s, kk > 0 ? 1u : 0u);
            tc_mma_f16(tmem + kColP + sb * kSub, smem_desc(do_addr + oa, 16, 1024),
                       smem_desc(v_addr + ob, 16, 1024), id_s, kk > 0 ? 1u : 0u);
          }
          tc_commit(&bars[DQ_SFULL0 + sb]);
          if (j == n_sub - 1) tc_commit(&bars[DQ_QEMPTY]);
          ++s_it;
          if (j > 0) ok = issue_dq(kv0 + j - 1, j - 1 == 0);
        }
        if (ok) ok = issue_dq(kv0 + n_sub - 1, n_sub == 1);
        if (ok) tc_commit(&bars[DQ_DONE]);
      }
    }
  } else {
    const int quarter = warp & 3;
    // Two groups of 4 warps ping-pong over the sub-tiles: group g takes the sub-tiles with
    // s_it % 2 == g, i.e. TMEM S/dP buffer g and dS buffer g, so two sub-tiles are in
    // flight and one group's latency overlaps the other's work.  Each thread owns a full
    // 64-column row of its group's sub-tiles.
    const int grp = (warp - 2) >> 2;
    const int rl = quarter * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    const float scale2 = a.scale * kLog2e;
    const bool issuer = warp == 2 && lane == 0;  // issues the dQ tile stores
    uint32_t s_it = 0, done_it = 0, kv = 0, n_store = 0, n_drain = 0;
    bool ok = true;
    for (uint32_t w = 0; ok; ++w) {
      WorkEntry e;
      if (!(ok = ring_get_warp(ring, &bars[DQ_WFULL0], &bars[DQ_WEMPTY0], w, e, a.status))) break;
      if (e.item < 0) break;
      const DqItem it = dq_item(a, e.item);
      const int n_sub = e.end - e.begin;
      const int64_t row = it.q_start + rl;
      const int64_t zh = it.z * a.H + it.h;
      float lse2 = 0.f, dl = 0.f;
      if (row < a.N) {
        const float lv = a.lse[zh * a.N + row];
        lse2 = lv == -INFINITY ? 0.f : lv * kLog2e;  // block_list.py:553 (lse_safe)
        dl = a.delta[zh * a.N + row];
      }
      for (int j = e.begin; j < e.end && ok; ++j, ++kv, ++s_it) {
        const uint32_t sb = s_it & 1;
        if ((int)sb != grp) continue;  // the other group's sub-tile
        const int slot = j / spb;
        // this stage's K/V stay resident until the dQ MMA of sub-tile j, which waits for us
        const uint32_t st = kv % kStages;
        if (!(ok = mbar_wait_warp(&bars[DQ_KVFULL0 + st], (kv / kStages) & 1, a.status))) break;
        const int64_t k0 = meta[st].start;
        const float b2 = meta[st].b2;
        const uint32_t sph = (s_it >> 1) & 1;
        if (!(ok = mbar_wait_warp(&bars[DQ_SFULL0 + sb], sph, a.status))) break;
        tc_fence_after();
        float s[kSub], dp[kSub];
        tmem_ld32(lane_addr + kColS + sb * kSub, *reinterpret_cast<float(*)[32]>(s));
        tmem_ld32(lane_addr + kColS + sb * kSub + 32, *reinterpret_cast<float(*)[32]>(s + 32));
        tmem_ld32(lane_addr + kColP + sb * kSub, *reinterpret_cast<float(*)[32]>(dp));
        tmem_ld32(lane_addr + kColP + sb * kSub + 32, *reinterpret_cast<float(*)[32]>(dp + 32));
        tmem_wait_ld();
        int64_t lim64 = a.N - 1 - k0;  // keys k0 + c with c <= lim are visible to this row
        if (a.causal) lim64 = min(lim64, row - k0);
        if (row >= a.N) lim64 = -1;
        const int lim = (int)max((int64_t)-1, min((int64_t)kSub, lim64));
        const bool full = lim >= kSub - 1;
        uint32_t pk[kSub / 2];
        float rs = 0.f;
#pragma unroll
        for (int c = 0; c < kSub; c += 2) {
          float d0 = fast_exp2(fmaf(s[c], scale2, b2) - lse2) * (dp[c] - dl);
          float d1 = fast_exp2(fmaf(s[c + 1], scale2, b2) - lse2) * (dp[c + 1] - dl);
          if (!full) {
            d0 = c <= lim ? d0 : 0.f;
            d1 = c + 1 <= lim ? d1 : 0.f;
          }
          rs += d0 + d1;
          pk[c / 2] = pack2(d0 * a.scale, d1 * a.scale, BF16);
        }
        // packed dS overwrites columns [0, 32) of this lane's S (already in registers)
        tmem_st16(lane_addr + kColS + sb * kSub, pk);
        tmem_st16(lane_addr + kColS + sb * kSub + 16, pk + 16);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars[DQ_DSFULL0 + sb]);
        if (a.dbias) {
#pragma unroll
          for (int o = 16; o; o >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, o);
          if (lane == 0) atomicAdd(&a.dbias[it.row_id * a.list_stride + slot], rs);
        }
      }
      if (!ok) break;
      if (n_sub > 0) {
        if (!(ok = mbar_wait_warp(&bars[DQ_DONE], done_it & 1, a.status))) break;
        ++done_it;
        tc_fence_after();
      }
      // dQ tile -> shared memory (128-byte swizzled 128 x 64 boxes; each group its D/2
      // columns) -> one TMA tile store per box.  The staging buffer is rewritten only after
      // the previous item's store has read it.
      if (n_store > n_drain) {
        if (issuer) {
          tma_store_wait_read();
          mbar_arrive(&bars[DQ_ODRAIN]);
        }
        if (!(ok = mbar_wait_warp(&bars[DQ_ODRAIN], n_drain & 1, a.status))) break;
        ++n_drain;
      }
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        const int col = grp * (D / 2) + c * 32;
        float o[32];
        if (n_sub > 0) {
          tmem_ld32(lane_addr + kColAcc + col, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        unsigned char* box = sm + L::kOut + (col >> 6) * (kRows * 128);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const int unit = ((col & 63) >> 3) + v;
          const uint32_t off = rl * 128 + ((unit ^ (rl & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(box + off)),
                       "r"(pack2(o[v * 8 + 0], o[v * 8 + 1], BF16)),
                       "r"(pack2(o[v * 8 + 2], o[v * 8 + 3], BF16)),
                       "r"(pack2(o[v * 8 + 4], o[v * 8 + 5], BF16)),
                       "r"(pack2(o[v * 8 + 6], o[v * 8 + 7], BF16))
                       : "memory");
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars[DQ_OFULL]);
      if (issuer) {
        if (mbar_wait(&bars[DQ_OFULL], n_store & 1, a.status)) {
          for (int b = 0; b < D / 64; ++b)
            tma_store_4d(&a.tm_dq, sm + L::kOut + b * (kRows * 128), b * 64, (int)it.q_start,
                         (int)it.h, (int)it.z);
        } else {
          ok = false;
        }
      }
      __syncwarp();
      ok = __all_sync(0xffffffffu, ok);
      ++n_store;
    }
  }
  // dQ stores still in flight must have read the staging buffer before shared memory goes away
  if (warp == 2 && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// =======================================================================================
// dK / dV kernel
// =======================================================================================
template <int D>
struct DkvLayout {
  static constexpr uint32_t kK = 0;                         // [128][D]
  static constexpr uint32_t kV = kRows * D * 2;             // [128][D]
  static constexpr uint32_t kQD = 2 * kRows * D * 2;        // stages x (Q, dO, stats)
  static constexpr uint32_t kStats = 2 * kSub * D * 2;      // stage offset: lse2[64], delta[64]
  static constexpr uint32_t kStage = kStats + 1024;         // keeps the tiles 1024-aligned
  static constexpr uint32_t kBars = kQD + kKvStages * kStage;
  static constexpr uint32_t kMeta = kBars + 256;  // StageMeta[kStages]
  static constexpr uint32_t kRingOff = kMeta + 128;  // WorkEntry[kRing]
  static constexpr uint32_t kAlloc = kRingOff + 128 + 1024;
};

enum { KV_KVFULL = 0, KV_KVEMPTY, KV_QFULL0, KV_QEMPTY0 = KV_QFULL0 + kKvStages,
       KV_SFULL0 = KV_QEMPTY0 + kKvStages, KV_PFULL0 = KV_SFULL0 + 2, KV_DONE = KV_PFULL0 + 2,
       KV_WFULL0, KV_WEMPTY0 = KV_WFULL0 + kRing, KV_NUM = KV_WEMPTY0 + kRing };

struct KvItem {
  int64_t z, hk, k0, kb;
};

__device__ __forceinline__ KvItem kv_item(const BwdArgs& a, int64_t item) {
  KvItem it;
  const int64_t zg_total = a.Z * a.Hkv;
  const int64_t kt = item / zg_total;
  const int64_t zg = item % zg_total;
  it.z = zg / a.Hkv;
  it.hk = zg % a.Hkv;
  it.k0 = kt * kRows;
  it.kb = it.k0 / a.RB;
  return it;
}

// Visit the streamed query sub-tiles [begin, end) of a dK/dV work item, in the item's fixed
// order: query heads of the group, then the head's transposed list, then 64-row sub-tiles.
template <typename F>
__device__ __forceinline__ bool for_each_qtile(const BwdArgs& a, const KvItem& it, int begin,
                                               int end, F&& f) {
  const int64_t group = a.H / a.Hkv;
  const int spb = (int)(a.RB / kSub);
  int pos = 0;
  for (int64_t h = it.hk * group; h < (it.hk + 1) * group && pos < end; ++h) {
    const int64_t krow = (it.z * a.H + h) * a.NB + it.kb;
    const int n_h = a.q_counts[krow] * spb;
    if (pos + n_h <= begin) {
      pos += n_h;
      continue;
    }
    for (int t = max(0, begin - pos); t < n_h && pos + t < end; ++t) {
      const int j = t / spb, sub = t % spb;
      const int64_t qb = a.k_lists[krow * a.NB + j];
      const int64_t slot = a.k_slots[krow * a.NB + j];
      if (!f(h, qb, slot, qb * a.RB + sub * kSub)) return false;
    }
    pos += n_h;
  }
  return true;
}

__device__ __forceinline__ int kv_item_tiles(const BwdArgs& a, const KvItem& it) {
  const int64_t group = a.H / a.Hkv;
  int n = 0;
  for (int64_t h = it.hk * group; h < (it.hk + 1) * group; ++h)
    n += a.q_counts[(it.z * a.H + h) * a.NB + it.kb];
  return n * (int)(a.RB / kSub);
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kBwdThreads, 1) bwd_dkdv_sm100_kernel(const __grid_constant__ BwdArgs a) {
  using L = DkvLayout<D>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::kBars);
  StageMeta* meta = reinterpret_cast<StageMeta*>(sm + L::kMeta);
  WorkEntry* ring = reinterpret_cast<WorkEntry*>(sm + L::kRingOff);
  __shared__ uint32_t s_tmem;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    uint32_t cnt[KV_NUM];
    for (int i = 0; i < KV_NUM; ++i) cnt[i] = 1;
    cnt[KV_PFULL0] = cnt[KV_PFULL0 + 1] = kEwThreads / 2;  // one group per buffer
    for (int i = 0; i < kRing; ++i) cnt[KV_WEMPTY0 + i] = 1 + kEwThreads;
    init_bars(bars, cnt, KV_NUM);
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&a.tm_q);
      prefetch_tmap(&a.tm_do);
      prefetch_tmap(&a.tm_k);
      prefetch_tmap(&a.tm_v);
      uint32_t qd = 0, jk = 0;
      bool ok = true;
      auto weight = [&](int64_t i) { return kv_item_tiles(a, kv_item(a, i)); };
      WorkFetcher fetch;
      fetch.init(&a.sched, weight);
      for (uint32_t w = 0; ok; ++w) {
        const WorkEntry e = fetch.next(weight);
        if (!(ok = ring_put(ring, &bars[KV_WFULL0], &bars[KV_WEMPTY0], w, e, a.status))) break;
        if (e.item < 0) break;
        const KvItem it = kv_item(a, e.item);
        if (e.end == e.begin) {
          fetch.reserve(weight);
          continue;
        }
        if (!(ok = mbar_wait(&bars[KV_KVEMPTY], (jk & 1) ^ 1, a.status))) break;
        ++jk;
        mbar_arrive_expect_tx(&bars[KV_KVFULL], 2 * kRows * D * 2);
        for (int c = 0; c < D / 64; ++c) {
          tma_load_4d(sm + L::kK + c * kRows * 128, &a.tm_k, &bars[KV_KVFULL], c * 64, (int)it.k0,
                      (int)it.hk, (int)it.z);
          tma_load_4d(sm + L::kV + c * kRows * 128, &a.tm_v, &bars[KV_KVFULL], c * 64, (int)it.k0,
                      (int)it.hk, (int)it.z);
        }
        uint32_t done = 0;
        ok = for_each_qtile(a, it, e.begin, e.end,
                            [&](int64_t h, int64_t qb, int64_t slot, int64_t q0) -> bool {
          const uint32_t st = qd % kKvStages, ph = (qd / kKvStages) & 1;
          if (!mbar_wait(&bars[KV_QEMPTY0 + st], ph ^ 1, a.status)) return false;
          unsigned char* stage = sm + L::kQD + st * L::kStage;
          meta[st].start = q0;
          meta[st].b2 = bias_log2(a, it.z, h, qb, slot);
          mbar_arrive_expect_tx(&bars[KV_QFULL0 + st], L::kStats + 2 * kSub * 4);
          for (int c = 0; c < D / 64; ++c) {
            tma_load_4d(stage + c * kSub * 128, &a.tm_q, &bars[KV_QFULL0 + st], c * 64, (int)q0,
                        (int)h, (int)it.z);
            tma_load_4d(stage + kSub * D * 2 + c * kSub * 128, &a.tm_do, &bars[KV_QFULL0 + st],
                        c * 64, (int)q0, (int)h, (int)it.z);
          }
          const int64_t zh = it.z * a.H + h;
          bulk_load(stage + L::kStats, a.stats + (zh * ((a.N + kSub - 1) / kSub) + q0 / kSub) * 2 * kSub,
                    2 * kSub * 4, &bars[KV_QFULL0 + st]);
          ++qd;
          if ((int)++done == e.end - e.begin) fetch.reserve(weight);
          return true;
        });
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16(kRows, kSub, BF16, false, false);
      constexpr uint32_t id_acc = idesc_f16(kRows, D, BF16, false, true);
      const uint32_t k_addr = smem_u32(sm + L::kK), v_addr = smem_u32(sm + L::kV);
      uint32_t qd = 0, s_it = 0, p_it = 0, jk = 0;
      bool ok = true;
      auto issue_acc = [&](uint32_t qd_u, bool first) -> bool {
        const uint32_t pb = p_it & 1;
        if (!mbar_wait(&bars[KV_PFULL0 + pb], (p_it >> 1) & 1, a.status)) return false;
        tc_fence_after();
        const uint32_t st = qd_u % kKvStages;
        const uint32_t q_addr = smem_u32(sm + L::kQD + st * L::kStage);
        const uint32_t do_addr = q_addr + kSub * D * 2;
        // P^T / dS^T sit in TMEM over the S^T / dP^T columns of buffer pb (bf16 pairs)
#pragma unroll
        for (int kk = 0; kk < kSub / 16; ++kk) {
          const uint32_t acc = (!first || kk > 0) ? 1u : 0u;
          tc_mma_f16_ts(tmem + kColAcc, tmem + kColS + pb * kSub + kk * 8,
                        smem_desc(do_addr + kk * 16 * 128, kSub * 128, 1024), id_acc, acc);
          tc_mma_f16_ts(tmem + kColAcc + D, tmem + kColP + pb * kSub + kk * 8,
                        smem_desc(q_addr + kk * 16 * 128, kSub * 128, 1024), id_acc, acc);
        }
        tc_commit(&bars[KV_QEMPTY0 + st]);
        ++p_it;
        return true;
      };
      for (uint32_t w = 0; ok; ++w) {
        WorkEntry e;
        if (!(ok = ring_get(ring, &bars[KV_WFULL0], &bars[KV_WEMPTY0], w, e, a.status))) break;
        if (e.item < 0) break;
        const int n = e.end - e.begin;
        if (n == 0) continue;
        if (!(ok = mbar_wait(&bars[KV_KVFULL], jk & 1, a.status))) break;
        ++jk;
        const uint32_t qd0 = qd;
        for (int i = 0; i < n && ok; ++i) {
          const uint32_t st = qd % kKvStages, ph = (qd / kKvStages) & 1;
          const uint32_t sb = s_it & 1;
          if (!(ok = mbar_wait(&bars[KV_QFULL0 + st], ph, a.status))) break;
          // TMEM buffer sb is reusable: the dV/dK MMAs of sub-tile s_it - 2, which read its
          // P^T / dS^T, were issued (after their PFULL wait) before this point, and MMAs of one
          // thread execute in issue order.
          tc_fence_after();
          const uint32_t q_addr = smem_u32(sm + L::kQD + st * L::kStage);
          const uint32_t do_addr = q_addr + kSub * D * 2;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t oa = (kk >> 2) * (kRows * 128) + (kk & 3) * 32;
            const uint32_t ob = (kk >> 2) * (kSub * 128) + (kk & 3) * 32;
            tc_mma_f16(tmem + kColS + sb * kSub, smem_desc(k_addr + oa, 16, 1024),
                       smem_desc(q_addr + ob, 16, 1024), id_s, kk > 0 ? 1u : 0u);
            tc_mma_f16(tmem + kColP + sb * kSub, smem_desc(v_addr + oa, 16, 1024),
                       smem_desc(do_addr + ob, 16, 1024), id_s, kk > 0 ? 1u : 0u);
          }
          tc_commit(&bars[KV_SFULL0 + sb]);
          if (i == n - 1) tc_commit(&bars[KV_KVEMPTY]);
          ++s_it;
          if (i > 0) ok = issue_acc(qd0 + i - 1, i - 1 == 0);
          ++qd;
        }
        if (ok) ok = issue_acc(qd0 + n - 1, n == 1);
        if (ok) tc_commit(&bars[KV_DONE]);
      }
    }
  } else {
    const int quarter = warp & 3;
    // Two groups of 4 warps ping-pong over the sub-tiles: group g takes the sub-tiles with
    // s_it % 2 == g (TMEM S^T/dP^T buffer g, P^T/dS^T buffer g); each thread owns one key
    // row and all 64 query columns of its group's sub-tiles.
    const int grp = (warp - 2) >> 2;
    const int half = grp;                // epilogue: which half of the D columns
    const int rl = quarter * 32 + lane;  // key row within the tile
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    const float scale2 = a.scale * kLog2e;
    uint32_t s_it = 0, done_it = 0, qd = 0;
    bool ok = true;
    for (uint32_t w = 0; ok; ++w) {
      WorkEntry e;
      if (!(ok = ring_get_warp(ring, &bars[KV_WFULL0], &bars[KV_WEMPTY0], w, e, a.status))) break;
      if (e.item < 0) break;
      const KvItem it = kv_item(a, e.item);
      const int n = e.end - e.begin;
      const int64_t key = it.k0 + rl;
      for (int i = 0; i < n && ok; ++i, ++qd, ++s_it) {
        const uint32_t sb = s_it & 1, sph = (s_it >> 1) & 1;
        if ((int)sb != grp) continue;  // the other group's sub-tile
        // the stage's TMA writes (Q, dO, row stats) and its meta are visible once its phase
        // completed; the stage stays resident until the dV/dK MMAs of this sub-tile
        const uint32_t st = qd % kKvStages, ph = (qd / kKvStages) & 1;
        if (!(ok = mbar_wait_warp(&bars[KV_QFULL0 + st], ph, a.status))) break;
        const float* stats = reinterpret_cast<const float*>(sm + L::kQD + st * L::kStage + L::kStats);
        const int64_t q0 = meta[st].start;
        const float b2 = meta[st].b2;
        if (!(ok = mbar_wait_warp(&bars[KV_SFULL0 + sb], sph, a.status))) break;
        tc_fence_after();
        // query q0 + c sees this key iff key < N, q0 + c < N and, when causal, key <= q0 + c:
        // visible columns are [lo, hi) (int32, clamped once per sub-tile)
        const int64_t cmin = a.causal ? key - q0 : 0;
        const int lo = (int)max((int64_t)0, min((int64_t)kSub, cmin));
        const int hi = key < a.N ? (int)max((int64_t)0, min((int64_t)kSub, a.N - q0)) : 0;
        const bool full = lo == 0 && hi == kSub;
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {  // two 32-column halves keep the live registers low
          float s[32], dp[32];
          tmem_ld32(lane_addr + kColS + sb * kSub + hc * 32, s);
          tmem_ld32(lane_addr + kColP + sb * kSub + hc * 32, dp);
          tmem_wait_ld();
          const float4* l2v = reinterpret_cast<const float4*>(stats + hc * 32);
          const float4* dlv = reinterpret_cast<const float4*>(stats + kSub + hc * 32);
          uint32_t pk[16], dk[16];
#pragma unroll
          for (int c4 = 0; c4 < 8; ++c4) {
            const float4 l4 = l2v[c4], d4 = dlv[c4];
            const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dv[4] = {d4.x, d4.y, d4.z, d4.w};
            float p[4], d[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int c = c4 * 4 + u;
              p[u] = fast_exp2(fmaf(s[c], scale2, b2) - lv[u]);
              d[u] = p[u] * (dp[c] - dv[u]) * a.scale;
              if (!full) {
                const int cc = hc * 32 + c;
                const bool vis = cc >= lo && cc < hi;
                p[u] = vis ? p[u] : 0.f;
                d[u] = vis ? d[u] : 0.f;
              }
            }
            pk[c4 * 2] = pack2(p[0], p[1], BF16);
            pk[c4 * 2 + 1] = pack2(p[2], p[3], BF16);
            dk[c4 * 2] = pack2(d[0], d[1], BF16);
            dk[c4 * 2 + 1] = pack2(d[2], d[3], BF16);
          }
          // packed P^T / dS^T overwrite columns [hc*16, hc*16+16) of this lane's S^T / dP^T,
          // which this thread has already read (half hc = 1 reads columns 32-63 only)
          tmem_st16(lane_addr + kColS + sb * kSub + hc * 16, pk);
          tmem_st16(lane_addr + kColP + sb * kSub + hc * 16, dk);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars[KV_PFULL0 + sb]);
      }
      if (!ok) break;
      if (n > 0) {
        if (!(ok = mbar_wait_warp(&bars[KV_DONE], done_it & 1, a.status))) break;
        ++done_it;
        tc_fence_after();
      }
      const int c0 = half * (D / 2);
      if (e.slot < 0) {
        store_cols<D / 2>(a.dv, a.dvs, it.z, it.hk, key, c0, lane_addr + kColAcc + c0, BF16,
                          key < a.N, n == 0);
        store_cols<D / 2>(a.dk, a.dks, it.z, it.hk, key, c0, lane_addr + kColAcc + D + c0, BF16,
                          key < a.N, n == 0);
      } else {
        // a chunk of a split item: fp32 partial row [dV | dK] into its slot
        float* prow = a.partials + ((int64_t)e.slot * kRows + rl) * (2 * D);
#pragma unroll
        for (int part = 0; part < 2; ++part) {
#pragma unroll
          for (int c = 0; c < D / 2; c += 32) {
            float o[32];
            if (n > 0) {
              tmem_ld32(lane_addr + kColAcc + part * D + c0 + c, o);
              tmem_wait_ld();
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = 0.f;
            }
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(prow + part * D + c0 + c + i) =
                  make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
          }
        }
      }
      tc_fence_before();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// =======================================================================================
// fused dK / dV / dQ kernel (head_dim 128): one pass over the transposed lists
// =======================================================================================
//
// The dK/dV kernel's pipeline plus, per streamed 64-row query sub-tile,
//    dQ^T = K^T dS^T   (M=128 head-dim rows, N=64 query rows, K=128 keys)
// with K^T read MN-major from the resident K tile and dS^T (bf16) written by the elementwise
// warps into shared memory as well as into TMEM.  Tensor work per kept pair is 10 RB^2 D
// (S^T, dP^T, dV, dK, dQ) against 14 for the separate dQ and dK/dV kernels, and there is one
// elementwise pass instead of two.
//
// TMEM (512 columns): S^T[2] at 0 / 64 (double-buffered: P^T and dS^T bf16 pairs overwrite
// them, half hc of the 64 query columns holding P^T at [32 hc, 32 hc + 16) and dS^T at
// [32 hc + 16, 32 hc + 32)), one dP^T buffer at 128, one dQ^T buffer at 192, dV at 256 and dK
// at 384.  The tensor pipe runs A(j+1) B(j) A(j+2) B(j+1) ..., where A(j) = S^T, dP^T of
// sub-tile j and B(j) = dV += P^T dO, dK += dS^T Q, dQ^T = K^T dS^T.  A(j)'s S^T MMAs need
// B(j-2)'s dV / dK MMAs to have read the S^T buffer (SFREE), its dP^T MMAs the dP^T buffer
// read out by sub-tile j-1's group (DPFREE); B(j) needs dQ^T(j-1) read out (DQEMPTY).
//
// The owning group reads dQ^T out of TMEM and stages it as fp32 rows [q][d] in the
// sub-tile's own Q/dO stage, whose tiles B(j) no longer needs once DQFULL(j) fired; one
// bulk reduction (cp.reduce.async.bulk .add.f32, performed at L2) adds the rows into an
// fp32 dQ accumulator, and the group's leader hands the stage back to the loader once the
// reduction has read it.  dQ's summation order depends on timing, so it is not bitwise
// reproducible from run to run; the two-kernel path is.
//
// Two threads issue the MMAs: warp 1 the A blocks, warp kFuBWarp the B blocks, each in
// sub-tile order (a thread issuing tcgen05.mma is held at each issue while the tensor pipe is
// busy, so one thread for both left the pipe idle through its waits and commits).  The
// accumulating MMAs all come from one thread in sub-tile order, so dV and dK sums are
// reproducible.

constexpr int kFuStages = 4;


struct FuLayout {
  static constexpr int D = 128;
  static constexpr uint32_t kK = 0;                      // [128][128] (2 boxes of 64 columns)
  static constexpr uint32_t kV = kRows * D * 2;
  static constexpr uint32_t kQD = 2 * kRows * D * 2;     // stages x (Q [64][D], dO [64][D])
  static constexpr uint32_t kStage = 2 * kSub * D * 2;   // later: dQ rows [64][D] fp32
  static constexpr uint32_t kDsT = kQD + kFuStages * kStage;  // 2 x dS^T [128 keys][64 q] bf16
  static constexpr uint32_t kDsTBytes = kRows * kSub * 2;
  static constexpr uint32_t kStats = kDsT + 2 * kDsTBytes;  // stages x {lse*log2e[64], delta[64]}
  static constexpr uint32_t kBars = kStats + kFuStages * 512;
  static constexpr uint32_t kMeta = kBars + 256;  // FuMeta[kFuStages]
  static constexpr uint32_t kRingOff = kMeta + 32 * kFuStages;
  static constexpr uint32_t kTmemSlot = kRingOff + 16 * kRing;
  static constexpr uint32_t kBytes = kTmemSlot + 16;
  // alignment slack for the 1024-byte aligned tiles, as far as the opt-in limit allows; the
  // kernel checks the padding it needs against %dynamic_smem_size
  static constexpr uint32_t kAlloc = kBytes + 1024 <= 232448 ? kBytes + 1024 : 232448;
  static_assert(kDsT % 1024 == 0 && kStage % 1024 == 0, "swizzled tiles need 1024-byte alignment");
  static_assert(kStage == kSub * D * 4, "a Q/dO stage holds the sub-tile's fp32 dQ rows");
  static_assert(kBytes <= 232448, "fused backward shared-memory layout too large");
};

struct FuMeta {
  int64_t start;     // first query row of the sub-tile
  int64_t zh;        // z * H + h of its query head
  int64_t bias_idx;  // d_soft_bias element of the block pair, or -1
  float b2;          // soft bias * log2(e)
  int qb;            // query block
};
static_assert(sizeof(FuMeta) == 32, "FuMeta layout");

constexpr uint32_t kFuColDp = 128, kFuColDq = 192;  // TMEM: single dP^T and dQ^T buffers

enum { FU_KVFULL = 0, FU_KVEMPTY, FU_QFULL0, FU_QEMPTY0 = FU_QFULL0 + kFuStages,
       FU_SFULL0 = FU_QEMPTY0 + kFuStages, FU_PFULL0 = FU_SFULL0 + 2, FU_DPFREE = FU_PFULL0 + 2,
       FU_DQFULL0, FU_DQEMPTY = FU_DQFULL0 + 2, FU_DONE, FU_EPI, FU_GSYNC0,
       FU_SFREE0 = FU_GSYNC0 + 2, FU_WFULL0 = FU_SFREE0 + 2, FU_WEMPTY0 = FU_WFULL0 + kRing,
       FU_NUM = FU_WEMPTY0 + kRing };
static_assert(FU_NUM * 8 <= 256, "fused backward barriers");

// BIAS_GRAD: the launch wants the soft-bias gradient (a.dbias).  A separate instantiation, so
// that the kernel without it gets a register allocation free of the running dS sum.
template <bool BF16, bool BIAS_GRAD>
__global__ void __launch_bounds__(kFuThreads, 1) bwd_fused_sm100_kernel(const __grid_constant__ BwdArgs a) {
  using L = FuLayout;
  constexpr int D = L::D;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  {
    const uint32_t base = smem_u32(smem_raw);
    uint32_t dyn;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
    if ((((base + 1023u) & ~1023u) - base) + L::kBytes > dyn) {  // uniform over the CTA
      if (threadIdx.x == 0) raise_status(a.status, kStatusSmemLayout);
      return;
    }
  }
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::kBars);
  FuMeta* meta = reinterpret_cast<FuMeta*>(sm + L::kMeta);
  WorkEntry* ring = reinterpret_cast<WorkEntry*>(sm + L::kRingOff);
  uint32_t& s_tmem = *reinterpret_cast<uint32_t*>(sm + L::kTmemSlot);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    uint32_t cnt[FU_NUM];
    for (int i = 0; i < FU_NUM; ++i) cnt[i] = 1;
    for (int b = 0; b < 2; ++b) {
      cnt[FU_PFULL0 + b] = kEwThreads / 2;   // the owning group
      cnt[FU_GSYNC0 + b] = kEwThreads / 2;   // group-wide sync of group b
    }
    cnt[FU_DPFREE] = kEwThreads / 2;   // the sub-tile's group has read dP^T
    cnt[FU_DQEMPTY] = kEwThreads / 2;  // the sub-tile's group has read dQ^T
    cnt[FU_EPI] = kEwThreads;          // both groups have read the dV / dK accumulators
    cnt[FU_KVEMPTY] = 2;               // both MMA issuers' last MMAs of the item completed
    // QEMPTY: one arrival, the owning group's leader once its dQ reduction read the stage
    for (int i = 0; i < kRing; ++i) cnt[FU_WEMPTY0 + i] = 2 + kEwThreads;  // both issuers, the groups
    init_bars(bars, cnt, FU_NUM);
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&a.tm_q);
      prefetch_tmap(&a.tm_do);
      prefetch_tmap(&a.tm_k);
      prefetch_tmap(&a.tm_v);
      uint32_t qd = 0, jk = 0;
      bool ok = true;
      auto weight = [&](int64_t i) { return kv_item_tiles(a, kv_item(a, i)); };
      WorkFetcher fetch;
      fetch.init(&a.sched, weight);
      for (uint32_t w = 0; ok; ++w) {
        const WorkEntry e = fetch.next(weight);
        if (!(ok = ring_put(ring, &bars[FU_WFULL0], &bars[FU_WEMPTY0], w, e, a.status))) break;
        if (e.item < 0) break;
        const KvItem it = kv_item(a, e.item);
        if (e.end == e.begin) {
          fetch.reserve(weight);
          continue;
        }
        if (!(ok = mbar_wait(&bars[FU_KVEMPTY], (jk & 1) ^ 1, a.status))) break;
        ++jk;
        mbar_arrive_expect_tx(&bars[FU_KVFULL], 2 * kRows * D * 2);
        for (int c = 0; c < D / 64; ++c) {
          tma_load_4d(sm + L::kK + c * kRows * 128, &a.tm_k, &bars[FU_KVFULL], c * 64, (int)it.k0,
                      (int)it.hk, (int)it.z);
          tma_load_4d(sm + L::kV + c * kRows * 128, &a.tm_v, &bars[FU_KVFULL], c * 64, (int)it.k0,
                      (int)it.hk, (int)it.z);
        }
        uint32_t done = 0;
        ok = for_each_qtile(a, it, e.begin, e.end,
                            [&](int64_t h, int64_t qb, int64_t slot, int64_t q0) -> bool {
          const uint32_t st = qd % kFuStages, ph = (qd / kFuStages) & 1;
          if (!mbar_wait(&bars[FU_QEMPTY0 + st], ph ^ 1, a.status)) return false;
          unsigned char* stage = sm + L::kQD + st * L::kStage;
          const int64_t zh = it.z * a.H + h;
          meta[st].start = q0;
          meta[st].zh = zh;
          meta[st].bias_idx = a.dbias ? (zh * a.NB + qb) * a.list_stride + slot : -1;
          meta[st].b2 = bias_log2(a, it.z, h, qb, slot);
          meta[st].qb = (int)qb;
          // the previous user of the stage wrote dQ rows into it with generic stores, and
          // its reduction read them, before the leader's QEMPTY arrival
          mbar_arrive_expect_tx(&bars[FU_QFULL0 + st], L::kStage + 2 * kSub * 4);
          for (int c = 0; c < D / 64; ++c) {
            tma_load_4d(stage + c * kSub * 128, &a.tm_q, &bars[FU_QFULL0 + st], c * 64, (int)q0,
                        (int)h, (int)it.z);
            tma_load_4d(stage + kSub * D * 2 + c * kSub * 128, &a.tm_do, &bars[FU_QFULL0 + st],
                        c * 64, (int)q0, (int)h, (int)it.z);
          }
          bulk_load(sm + L::kStats + st * 512,
                    a.stats + (zh * ((a.N + kSub - 1) / kSub) + q0 / kSub) * 2 * kSub, 2 * kSub * 4,
                    &bars[FU_QFULL0 + st]);
          ++qd;
          if ((int)++done == e.end - e.begin) fetch.reserve(weight);
          return true;
        });
      }
    }
  } else if (warp == 1) {
    // A blocks: S^T = K Q^T and dP^T = V dO^T of every sub-tile, in order.  The B blocks have
    // their own issuing thread (warp kFuBWarp): a thread that issues tcgen05.mma is held at
    // each issue while the tensor pipe is busy (~72-82 cycles per MMA here, traced), so one
    // thread issuing both kinds left the pipe idle through every wait, fence and commit
    // between its blocks (~54 % of each sub-tile).  The two threads meet only through
    // mbarriers: A(j) writes S^T buffer j & 1, which B(j - 2)'s dV / dK MMAs read (SFREE).
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16(kRows, kSub, BF16, false, false);
      // base descriptors (K-major for S^T / dP^T); per-MMA tiles by desc_add
      const uint64_t kd_k = smem_desc(smem_u32(sm + L::kK), 16, 1024);
      const uint64_t vd_k = smem_desc(smem_u32(sm + L::kV), 16, 1024);
      uint32_t ga = 0, jk = 0;  // sub-tiles with A issued (all items), K/V tiles
      bool ok = true;
      for (uint32_t w = 0; ok; ++w) {
        WorkEntry e;
        if (!(ok = ring_get(ring, &bars[FU_WFULL0], &bars[FU_WEMPTY0], w, e, a.status))) break;
        if (e.item < 0) break;
        const int n = e.end - e.begin;
        if (n == 0) continue;
        if (!(ok = mbar_wait(&bars[FU_KVFULL], jk & 1, a.status))) break;
        ++jk;
        for (int i = 0; i < n && ok; ++i, ++ga) {
          const uint32_t st = ga % kFuStages, ph = (ga / kFuStages) & 1, sb = ga & 1;
          // S^T once B(ga - 2) has released its buffer and the sub-tile's Q / dO stage is
          // loaded; dP^T once sub-tile ga - 1's group has read the single dP^T buffer.  That
          // group frees it halfway through its elementwise pass, so issuing the S^T MMAs first
          // leaves only the dP^T half of the block on the next sub-tile's critical path.
          ok = (ga < 2 || mbar_wait(&bars[FU_SFREE0 + sb], ((ga - 2) >> 1) & 1, a.status)) &&
               mbar_wait(&bars[FU_QFULL0 + st], ph, a.status);
          if (!ok) break;
          tc_fence_after();
          const uint64_t qd_k = smem_desc(smem_u32(sm + L::kQD + st * L::kStage), 16, 1024);
          const uint64_t dod_k = desc_add(qd_k, kSub * D * 2);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t oa = (kk >> 2) * (kRows * 128) + (kk & 3) * 32;
            const uint32_t ob = (kk >> 2) * (kSub * 128) + (kk & 3) * 32;
            tc_mma_f16(tmem + kColS + sb * kSub, desc_add(kd_k, oa), desc_add(qd_k, ob), id_s,
                       kk > 0 ? 1u : 0u);
          }
          if (!(ok = ga == 0 || mbar_wait(&bars[FU_DPFREE], (ga - 1) & 1, a.status))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t oa = (kk >> 2) * (kRows * 128) + (kk & 3) * 32;
            const uint32_t ob = (kk >> 2) * (kSub * 128) + (kk & 3) * 32;
            tc_mma_f16(tmem + kFuColDp, desc_add(vd_k, oa), desc_add(dod_k, ob), id_s,
                       kk > 0 ? 1u : 0u);
          }
          tc_commit(&bars[FU_SFULL0 + sb]);
        }
        if (!ok) break;
        tc_commit(&bars[FU_KVEMPTY]);  // this thread's last MMA of the item has read K / V
      }
    }
  } else if (warp == kFuBWarp) {
    // B blocks: dV += P^T dO, dK += dS^T Q, dQ^T = K^T dS^T of every sub-tile, in order, once
    // its P^T / dS^T are written (PFULL) and dQ^T(gb - 1) was read out (DQEMPTY).  The item's
    // first one overwrites the dV / dK accumulators: the previous item's epilogue must have
    // read them (EPI).
    if (lane == 0) {
      constexpr uint32_t id_acc = idesc_f16(kRows, D, BF16, false, true);
      // dQ^T = K^T dS^T: A (head dim x keys) and B (keys x query rows) both MN-major
      constexpr uint32_t id_dq = idesc_f16(kRows, kSub, BF16, true, true);
      const uint64_t kd_mn = smem_desc(smem_u32(sm + L::kK), kRows * 128, 1024);
      const uint64_t dsd0_mn = smem_desc(smem_u32(sm + L::kDsT), kSub * 128, 1024);
      uint32_t gb = 0, jk = 0, n_items = 0;
      bool ok = true;
      for (uint32_t w = 0; ok; ++w) {
        WorkEntry e;
        if (!(ok = ring_get(ring, &bars[FU_WFULL0], &bars[FU_WEMPTY0], w, e, a.status))) break;
        if (e.item < 0) break;
        const int n = e.end - e.begin;
        if (n == 0) continue;
        // K is an operand of the dQ^T MMAs: the item's K / V tiles are in place
        if (!(ok = mbar_wait(&bars[FU_KVFULL], jk & 1, a.status))) break;
        ++jk;
        for (int ib = 0; ib < n && ok; ++ib, ++gb) {
          const uint32_t pb = gb & 1;
          ok = (ib > 0 || n_items == 0 || mbar_wait(&bars[FU_EPI], (n_items - 1) & 1, a.status)) &&
               (gb == 0 || mbar_wait(&bars[FU_DQEMPTY], (gb - 1) & 1, a.status)) &&
               mbar_wait(&bars[FU_PFULL0 + pb], (gb >> 1) & 1, a.status);
          if (!ok) break;
          tc_fence_after();
          const uint32_t st = gb % kFuStages;
          const uint64_t qd_mn = smem_desc(smem_u32(sm + L::kQD + st * L::kStage), kSub * 128, 1024);
          const uint64_t dod_mn = desc_add(qd_mn, kSub * D * 2);
          const uint32_t colS = kColS + pb * kSub;
#pragma unroll
          for (int kk = 0; kk < kSub / 16; ++kk) {
            const uint32_t acc = (ib > 0 || kk > 0) ? 1u : 0u;
            const uint32_t pcol = colS + (kk >> 1) * 32 + (kk & 1) * 8;  // P^T, then dS^T + 16
            tc_mma_f16_ts(tmem + kColAcc, tmem + pcol, desc_add(dod_mn, kk * 16 * 128), id_acc, acc);
            tc_mma_f16_ts(tmem + kColAcc + D, tmem + pcol + 16, desc_add(qd_mn, kk * 16 * 128), id_acc,
                          acc);
          }
          // S^T buffer pb (P^T / dS^T) is read once these complete: the dQ^T MMAs below take
          // dS^T from shared memory, so A(gb + 2) need not wait for them
          tc_commit(&bars[FU_SFREE0 + pb]);
          const uint64_t dsd_mn = desc_add(dsd0_mn, pb * L::kDsTBytes);
#pragma unroll
          for (int kk = 0; kk < kRows / 16; ++kk)
            tc_mma_f16(tmem + kFuColDq, desc_add(kd_mn, kk * 16 * 128),
                       desc_add(dsd_mn, kk * 16 * 128), id_dq, kk > 0 ? 1u : 0u);
          tc_commit(&bars[FU_DQFULL0 + pb]);
        }
        if (!ok) break;
        tc_commit(&bars[FU_KVEMPTY]);  // the last dQ^T MMA has read K
        tc_commit(&bars[FU_DONE]);
        ++n_items;
      }
    }
  } else {
    const int quarter = warp & 3;
    const int grp = (warp - 2) >> 2;
    const int half = grp;
    const int rl = quarter * 32 + lane;  // key row (S^T, dP^T, dV, dK) / head-dim row (dQ^T)
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    const float scale2 = a.scale * kLog2e;
    const bool leader = (warp & 3) == 2 && lane == 0;  // one thread per group (warps 2 and 6)
    uint32_t s_it = 0, done_it = 0, qd = 0, gsync = 0;
    int pend_st = -1;  // the leader's stage awaiting its reduction's read before release
    bool ok = true;
    // Sync of this group's 4 warps on an mbarrier with a bounded wait (a named barrier would
    // wait forever on a warp that gave up); warp-uniform result.
    auto group_sync = [&]() -> bool {
      mbar_arrive(&bars[FU_GSYNC0 + grp]);
      return mbar_wait_warp(&bars[FU_GSYNC0 + grp], gsync++ & 1, a.status);
    };
    for (uint32_t w = 0; ok; ++w) {
      WorkEntry e;
      if (!(ok = ring_get_warp(ring, &bars[FU_WFULL0], &bars[FU_WEMPTY0], w, e, a.status))) break;
      if (e.item < 0) break;
      const KvItem it = kv_item(a, e.item);
      const int n = e.end - e.begin;
      const int64_t key = it.k0 + rl;
      for (int i = 0; i < n && ok; ++i, ++qd, ++s_it) {
        const uint32_t sb = s_it & 1, sph = (s_it >> 1) & 1;
        if ((int)sb != grp) continue;
        const uint32_t st = qd % kFuStages, ph = (qd / kFuStages) & 1;
        if (!(ok = mbar_wait_warp(&bars[FU_QFULL0 + st], ph, a.status))) break;
        float* stats = reinterpret_cast<float*>(sm + L::kStats + st * 512);
        // the sub-tile's meta stays put until this group's leader hands the stage back, so it
        // is read where it is needed instead of held in registers across the loop
        const FuMeta* m = &meta[st];
        const int64_t q0 = m->start;
        // per-column constants of the sub-tile, once for the group, over its stage's row
        // stats (only this group reads them): soft bias - lse (both in log2 units) and
        // -delta * scale, so that an element costs one f32x2 FMA per pair for the exponent
        // and one for dP - delta
        if (rl < kSub) {
          stats[rl] = m->b2 - stats[rl];
          stats[kSub + rl] = -stats[kSub + rl] * a.scale;
        }
        if (!(ok = mbar_wait_warp(&bars[FU_SFULL0 + sb], sph, a.status))) break;
        tc_fence_after();
        if (!(ok = group_sync())) break;  // the column constants are visible
        const int64_t cmin = a.causal ? key - q0 : 0;
        const int lo = (int)max((int64_t)0, min((int64_t)kSub, cmin));
        const int hi = key < a.N ? (int)max((int64_t)0, min((int64_t)kSub, a.N - q0)) : 0;
        const bool full = lo == 0 && hi == kSub;
        unsigned char* dsrow = sm + L::kDsT + sb * L::kDsTBytes + rl * 128;
        const uint64_t scale2x2 = f32x2(scale2, scale2), scalex2 = f32x2(a.scale, a.scale);
        uint64_t rs2 = 0;  // dS * scale summed in pairs (the soft bias gradient, rescaled below)
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          // S^T and dP^T by 32-column halves (registers: holding all of dP^T spills).  The
          // dP^T buffer is released once its second half is read, well before A(s_it + 1)
          // is due (it follows B(s_it - 1) on the tensor pipe)
          float s[32], dp[32];
          tmem_ld32(lane_addr + kColS + sb * kSub + hc * 32, s);
          tmem_ld32(lane_addr + kFuColDp + hc * 32, dp);
          tmem_wait_ld();
          if (hc == 1) {
            tc_fence_before();
            mbar_arrive(&bars[FU_DPFREE]);
          }
          const float4* cv = reinterpret_cast<const float4*>(stats + hc * 32);
          const float4* nv = reinterpret_cast<const float4*>(stats + kSub + hc * 32);
          // two quarters of 16 query columns: packed P^T / dS^T (8 columns each) go out as soon
          // as a quarter is done, which keeps the live registers below the spill line
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {
            uint32_t pk[8], dk[8];
#pragma unroll
            for (int c4i = 0; c4i < 4; ++c4i) {
              const int c4 = qq * 4 + c4i;
              const float4 c = cv[c4], nd = nv[c4];
              const int c0 = c4 * 4, cd = hc * 32 + c0;
              float p[4], d[4];
              f32x2_split(fma_f32x2(f32x2(s[c0], s[c0 + 1]), scale2x2, f32x2(c.x, c.y)), p[0], p[1]);
              f32x2_split(fma_f32x2(f32x2(s[c0 + 2], s[c0 + 3]), scale2x2, f32x2(c.z, c.w)), p[2], p[3]);
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                p[u] = fast_exp2(p[u]);
                if (!full) p[u] = (cd + u >= lo && cd + u < hi) ? p[u] : 0.f;
              }
              const uint64_t d01 = mul_f32x2(f32x2(p[0], p[1]),
                                             fma_f32x2(f32x2(dp[c0], dp[c0 + 1]), scalex2, f32x2(nd.x, nd.y)));
              const uint64_t d23 = mul_f32x2(f32x2(p[2], p[3]),
                                             fma_f32x2(f32x2(dp[c0 + 2], dp[c0 + 3]), scalex2, f32x2(nd.z, nd.w)));
              if constexpr (BIAS_GRAD) rs2 = add_f32x2(rs2, add_f32x2(d01, d23));
              f32x2_split(d01, d[0], d[1]);
              f32x2_split(d23, d[2], d[3]);
              pk[c4i * 2] = pack2(p[0], p[1], BF16);
              pk[c4i * 2 + 1] = pack2(p[2], p[3], BF16);
              dk[c4i * 2] = pack2(d[0], d[1], BF16);
              dk[c4i * 2 + 1] = pack2(d[2], d[3], BF16);
            }
            // P^T and dS^T (bf16 pairs) into this half's S^T columns, which this thread has
            // read: quarter qq's P^T at [32 hc + 8 qq, +8), its dS^T 16 columns further on
            tmem_st8(lane_addr + kColS + sb * kSub + hc * 32 + qq * 8, pk);
            tmem_st8(lane_addr + kColS + sb * kSub + hc * 32 + 16 + qq * 8, dk);
            // dS^T row `rl`, query columns [32 hc + 16 qq, +16), into the dQ MMA's B tile
            // (128-byte rows, 16-byte units swizzled by the row's low 3 bits).  The buffer's
            // previous dQ^T MMA (sub-tile s_it - 2, this group's) completed before this
            // group read its dQ^T out.
#pragma unroll
            for (int v = 0; v < 2; ++v) {
              const int unit = hc * 4 + qq * 2 + v;
              asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                               smem_u32(dsrow + ((unit ^ (rl & 7)) << 4))),
                           "r"(dk[v * 4 + 0]), "r"(dk[v * 4 + 1]), "r"(dk[v * 4 + 2]), "r"(dk[v * 4 + 3])
                           : "memory");
            }
          }
        }
        tmem_wait_st();
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&bars[FU_PFULL0 + sb]);
        if constexpr (BIAS_GRAD) {
          const int64_t bidx = m->bias_idx;
          float r0, r1;
          f32x2_split(rs2, r0, r1);
          float rs = (r0 + r1) / a.scale;
#pragma unroll
          for (int o = 16; o; o >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, o);
          if (lane == 0) atomicAdd(&a.dbias[bidx], rs);
        }
        // this group's previous stage goes back to the loader once its reduction has read it
        // (long done by now: off the elementwise path)
        if (leader && pend_st >= 0) {
          bulk_wait_read();
          mbar_arrive(&bars[FU_QEMPTY0 + pend_st]);
          pend_st = -1;
        }
        // dQ^T of this sub-tile: out of TMEM, release the buffer, stage the rows, reduce
        // one barrier per sub-tile parity: this group saw the phase before last of its own
        if (!(ok = mbar_wait_warp(&bars[FU_DQFULL0 + sb], sph, a.status))) break;
        tc_fence_after();
        const int rows = (int)min((int64_t)kSub, a.N - q0);
        float* stg = reinterpret_cast<float*>(sm + L::kQD + st * L::kStage);
#pragma unroll
        // both halves first, so that the buffer (which B of the next sub-tile overwrites) goes
        // back after two loads; then dQ^T -> fp32 rows [q][d] over the stage's Q/dO tiles (B of
        // this sub-tile, their last reader, has completed: DQFULL), added into the accumulator
        // by one bulk reduction performed at L2
        float dq0[32], dq1[32];
        tmem_ld32(lane_addr + kFuColDq, dq0);
        tmem_ld32(lane_addr + kFuColDq + 32, dq1);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&bars[FU_DQEMPTY]);
#pragma unroll
        for (int r = 0; r < 32; ++r) stg[r * D + rl] = dq0[r];
#pragma unroll
        for (int r = 0; r < 32; ++r) stg[(32 + r) * D + rl] = dq1[r];
        fence_proxy_async_smem();
        if (!(ok = group_sync())) break;
        if (leader) {
          bulk_reduce_add_f32(a.dq_acc + (m->zh * a.N + q0) * D, stg, (uint32_t)rows * D * 4);
          pend_st = (int)st;
        }
      }
      if (!ok) break;
      if (n > 0) {
        if (!(ok = mbar_wait_warp(&bars[FU_DONE], done_it & 1, a.status))) break;
        ++done_it;
        tc_fence_after();
      }
      const int c0 = half * (D / 2);
      if (e.slot < 0) {
        store_cols<D / 2>(a.dv, a.dvs, it.z, it.hk, key, c0, lane_addr + kColAcc + c0, BF16,
                          key < a.N, n == 0);
        store_cols<D / 2>(a.dk, a.dks, it.z, it.hk, key, c0, lane_addr + kColAcc + D + c0, BF16,
                          key < a.N, n == 0);
      } else {
        float* prow = a.partials + ((int64_t)e.slot * kRows + rl) * (2 * D);
#pragma unroll
        for (int part = 0; part < 2; ++part) {
#pragma unroll
          for (int c = 0; c < D / 2; c += 32) {
            float o[32];
            if (n > 0) {
              tmem_ld32(lane_addr + kColAcc + part * D + c0 + c, o);
              tmem_wait_ld();
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = 0.f;
            }
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(prow + part * D + c0 + c + i) =
                  make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
          }
        }
      }
      tc_fence_before();
      if (n > 0) mbar_arrive(&bars[FU_EPI]);
    }
    // a stage still held for its reduction: the loader has nothing left to load into it, but
    // release it all the same so that every QEMPTY phase completes
    if (leader && pend_st >= 0) {
      bulk_wait_read();
      mbar_arrive(&bars[FU_QEMPTY0 + pend_st]);
    }
  }
  // bulk reductions still in flight complete before the CTA (and its shared memory) ends
  if ((warp == 2 || warp == 6) && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, bool BF16>
int launch_t(const AttnParams& p, cudaStream_t stream, int parts) {
  BwdArgs a{};
  a.Z = p.Z;
  a.H = p.H;
  a.Hkv = p.Hkv;
  a.N = p.N;
  a.RB = p.RB;
  a.NB = p.NB;
  a.lists = p.lists;
  a.list_stride = p.list_stride;
  a.counts = p.counts;
  a.k_lists = p.k_lists;
  a.k_slots = p.k_slots;
  a.q_counts = p.q_counts;
  a.lse = p.lse;
  a.delta = p.delta;
  a.bias = p.bias;
  a.bias_dtype = p.bias_dtype;
  for (int i = 0; i < 4; ++i) {
    a.bs[i] = p.bs[i];
    a.dqs[i] = p.dqs[i];
    a.dks[i] = p.dks[i];
    a.dvs[i] = p.dvs[i];
  }
  a.dbias = p.dbias;
  a.stats = p.stats;
  a.dq = p.dq;
  a.dk = p.dk;
  a.dv = p.dv;
  a.causal = p.causal;
  a.scale = p.scale;
  a.status = p.status;
  const int sms = device_sm_count();
  if (parts & kBwdDq) {
    int rc = make_tmap_4d(&a.tm_q, p.q, p.dtype, p.Z, p.H, p.N, D, p.qs, 64, kRows);
    if (!rc) rc = make_tmap_4d(&a.tm_do, p.dout, p.dtype, p.Z, p.H, p.N, D, p.dos, 64, kRows);
    if (!rc) rc = make_tmap_4d(&a.tm_k, p.k, p.dtype, p.Z, p.Hkv, p.N, D, p.ks, 64, kSub);
    if (!rc) rc = make_tmap_4d(&a.tm_v, p.v, p.dtype, p.Z, p.Hkv, p.N, D, p.vs, 64, kSub);
    if (!rc) rc = make_tmap_4d(&a.tm_dq, p.dq, p.dtype, p.Z, p.H, p.N, D, p.dqs, 64, kRows);
    if (rc) return fail(SA_ELAUNCH, std::string("dQ tensor maps: ") + sa_last_error());
    a.tiles = (p.N + kRows - 1) / kRows;
    const int64_t items = a.Z * a.H * a.tiles;
    const int ctas = (int)std::min<int64_t>(items, sms);
    a.sched = SchedArgs{nullptr, nullptr, items, 0};
    auto kern = bwd_dq_sm100_kernel<D, BF16>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, DqLayout<D>::kAlloc);
    if (p.plan_dq) {
      // As in the forward: each CTA's first item is its own index (late query tiles first);
      // the planner, launched just before with this kernel as its programmatic dependent,
      // queues the rest heaviest-first while that first wave runs.
      const PlanPtrs pp = plan_carve(p.plan_dq, kPlanDq, items, ctas, D);
      int e = launch_plan(kPlanDq, p, items, ctas, pp, stream, ctas);
      if (e) return e;
      a.sched = SchedArgs{pp.header, pp.queue, items, 1};
      e = launch_dependent(kern, dim3((unsigned)ctas), dim3(kBwdThreads), DqLayout<D>::kAlloc,
                           stream, "bwd_dq_sm100_kernel", a);
      if (e) return e;
    } else {
      kern<<<(unsigned)ctas, kBwdThreads, DqLayout<D>::kAlloc, stream>>>(a);
      int e = check_launch("bwd_dq_sm100_kernel");
      if (e) return e;
    }
  }
  if (parts & kBwdDkDv) {
    int rc = make_tmap_4d(&a.tm_q, p.q, p.dtype, p.Z, p.H, p.N, D, p.qs, 64, kSub);
    if (!rc) rc = make_tmap_4d(&a.tm_do, p.dout, p.dtype, p.Z, p.H, p.N, D, p.dos, 64, kSub);
    if (!rc) rc = make_tmap_4d(&a.tm_k, p.k, p.dtype, p.Z, p.Hkv, p.N, D, p.ks, 64, kRows);
    if (!rc) rc = make_tmap_4d(&a.tm_v, p.v, p.dtype, p.Z, p.Hkv, p.N, D, p.vs, 64, kRows);
    if (rc) return fail(SA_ELAUNCH, std::string("dK/dV tensor maps: ") + sa_last_error());
    a.tiles = (p.N + kRows - 1) / kRows;
    const int64_t items = a.Z * a.Hkv * a.tiles;
    const int ctas = (int)std::min<int64_t>(items, sms);
    a.sched = SchedArgs{nullptr, nullptr, items, 0};
    PlanPtrs pp{};
    if (p.plan_dkdv) {
      pp = plan_carve(p.plan_dkdv, kPlanDkdv, items, ctas, D);
      a.sched = SchedArgs{pp.header, pp.queue, items, 0};
      a.partials = pp.partials;
    }
    auto kern = bwd_dkdv_sm100_kernel<D, BF16>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, DkvLayout<D>::kAlloc);
    kern<<<(unsigned)ctas, kBwdThreads, DkvLayout<D>::kAlloc, stream>>>(a);
    int e = check_launch("bwd_dkdv_sm100_kernel");
    if (e) return e;
    if (p.plan_dkdv) {
      e = launch_dkdv_reduce(p, pp, ctas, stream);
      if (e) return e;
    }
  }
  return SA_OK;
}

// dQ (Z, H, N, 128) with strides <- fp32 accumulator (Z*H, N, 128) contiguous; HBM-bound,
// 16-byte stores (rows 16-byte aligned, as the fused kernel's eligibility requires).
template <bool BF16>
__global__ void __launch_bounds__(256) dq_convert_kernel(const float* __restrict__ acc, void* dq,
                                                         int64_t s0, int64_t s1, int64_t s2,
                                                         int64_t H, int64_t N, int64_t n8) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const int64_t row = i / 16, c8 = i % 16;  // 16 groups of 8 columns per row
  const int64_t zh = row / N, q = row % N, z = zh / H, h = zh % H;
  const float4 a0 = __ldcs(reinterpret_cast<const float4*>(acc) + i * 2);
  const float4 a1 = __ldcs(reinterpret_cast<const float4*>(acc) + i * 2 + 1);
  uint4 o;
  o.x = pack2(a0.x, a0.y, BF16);
  o.y = pack2(a0.z, a0.w, BF16);
  o.z = pack2(a1.x, a1.y, BF16);
  o.w = pack2(a1.z, a1.w, BF16);
  *reinterpret_cast<uint4*>(static_cast<uint16_t*>(dq) + z * s0 + h * s1 + q * s2 + c8 * 8) = o;
}

template <bool BF16>
int launch_fused_t(const AttnParams& p, cudaStream_t stream) {
  constexpr int D = 128;
  BwdArgs a{};
  a.Z = p.Z;
  a.H = p.H;
  a.Hkv = p.Hkv;
  a.N = p.N;
  a.RB = p.RB;
  a.NB = p.NB;
  a.lists = p.lists;
  a.list_stride = p.list_stride;
  a.counts = p.counts;
  a.k_lists = p.k_lists;
  a.k_slots = p.k_slots;
  a.q_counts = p.q_counts;
  a.lse = p.lse;
  a.delta = p.delta;
  a.bias = p.bias;
  a.bias_dtype = p.bias_dtype;
  for (int i = 0; i < 4; ++i) {
    a.bs[i] = p.bs[i];
    a.dqs[i] = p.dqs[i];
    a.dks[i] = p.dks[i];
    a.dvs[i] = p.dvs[i];
  }
  a.dbias = p.dbias;
  a.stats = p.stats;
  a.dq = p.dq;
  a.dk = p.dk;
  a.dv = p.dv;
  a.causal = p.causal;
  a.scale = p.scale;
  a.status = p.status;
  a.dq_acc = p.dq_acc;
  if (!a.dq_acc || !p.plan_dkdv) return fail(SA_EINVAL, "fused backward: missing dQ accumulator / plan");
  int rc = make_tmap_4d(&a.tm_q, p.q, p.dtype, p.Z, p.H, p.N, D, p.qs, 64, kSub);
  if (!rc) rc = make_tmap_4d(&a.tm_do, p.dout, p.dtype, p.Z, p.H, p.N, D, p.dos, 64, kSub);
  if (!rc) rc = make_tmap_4d(&a.tm_k, p.k, p.dtype, p.Z, p.Hkv, p.N, D, p.ks, 64, kRows);
  if (!rc) rc = make_tmap_4d(&a.tm_v, p.v, p.dtype, p.Z, p.Hkv, p.N, D, p.vs, 64, kRows);
  if (rc) return fail(SA_ELAUNCH, std::string("fused backward tensor maps: ") + sa_last_error());
  a.tiles = (p.N + kRows - 1) / kRows;
  const int64_t items = a.Z * a.Hkv * a.tiles;
  const int ctas = (int)std::min<int64_t>(items, device_sm_count());
  const PlanPtrs pp = plan_carve(p.plan_dkdv, kPlanDkdv, items, ctas, D);
  a.sched = SchedArgs{pp.header, pp.queue, items, 0};
  a.partials = pp.partials;
  auto kern = a.dbias ? bwd_fused_sm100_kernel<BF16, true> : bwd_fused_sm100_kernel<BF16, false>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FuLayout::kAlloc);
  kern<<<(unsigned)ctas, kFuThreads, FuLayout::kAlloc, stream>>>(a);
  rc = check_launch("bwd_fused_sm100_kernel");
  if (rc) return rc;
  rc = launch_dkdv_reduce(p, pp, ctas, stream);
  if (rc) return rc;
  // dQ = the fp32 accumulator rounded to bf16 / fp16 (8 elements per thread)
  const int64_t n8 = p.Z * p.H * p.N * (D / 8);
  dq_convert_kernel<BF16><<<(unsigned)((n8 + 255) / 256), 256, 0, stream>>>(
      p.dq_acc, p.dq, p.dqs[0], p.dqs[1], p.dqs[2], p.H, p.N, n8);
  return check_launch("dq_convert_kernel");
}

}  // namespace

bool bwd_sm100_eligible(const AttnParams& p);

bool bwd_fused_eligible(const AttnParams& p) {
  // the prep's vectorised Delta kernel zeroes the dQ accumulator: O must suit it too
  if (reinterpret_cast<uintptr_t>(p.out) % 16) return false;
  for (int i = 0; i < 3; ++i)
    if (p.os[i] % 8) return false;
  return bwd_sm100_eligible(p) && p.D == 128 && p.RB % kRows == 0;
}

bool bwd_sm100_eligible(const AttnParams& p) {
  if (p.dtype != SA_BF16 && p.dtype != SA_F16) return false;
  if (p.D != 64 && p.D != 128) return false;
  if (p.RB % kRows) return false;
  const void* ptrs[7] = {p.q, p.k, p.v, p.dout, p.dq, p.dk, p.dv};
  for (auto ptr : ptrs)
    if (reinterpret_cast<uintptr_t>(ptr) % 16) return false;
  for (int i = 0; i < 3; ++i)
    if (p.qs[i] % 8 || p.ks[i] % 8 || p.vs[i] % 8 || p.dos[i] % 8 || p.dqs[i] % 8 ||
        p.dks[i] % 8 || p.dvs[i] % 8)
      return false;
  return p.N <= INT32_MAX;
}

int64_t bwd_plan_bytes(int which, int64_t Z, int64_t H, int64_t Hkv, int64_t N, int64_t D) {
  const int64_t tiles = (N + kRows - 1) / kRows;
  const int sms = device_sm_count();
  if (which == kPlanDq) {
    const int64_t items = Z * H * tiles;
    return plan_workspace_bytes(kPlanDq, items, (int)std::min<int64_t>(items, sms), D);
  }
  const int64_t items = Z * Hkv * tiles;
  return plan_workspace_bytes(kPlanDkdv, items, (int)std::min<int64_t>(items, sms), D);
}

int plan_bwd_sm100(const AttnParams& p, cudaStream_t stream, int which) {
  if (!bwd_sm100_eligible(p)) return SA_OK;
  const int64_t tiles = (p.N + kRows - 1) / kRows;
  const int sms = device_sm_count();
  if (p.plan_dq && (which & kBwdDq)) {
    const int64_t items = p.Z * p.H * tiles;
    const int ctas = (int)std::min<int64_t>(items, sms);
    const int rc = launch_plan(kPlanDq, p, items, ctas, plan_carve(p.plan_dq, kPlanDq, items, ctas, p.D),
                               stream);
    if (rc) return rc;
  }
  if (p.plan_dkdv && (which & kBwdDkDv)) {
    const int64_t items = p.Z * p.Hkv * tiles;
    const int ctas = (int)std::min<int64_t>(items, sms);
    const int rc = launch_plan(kPlanDkdv, p, items, ctas,
                               plan_carve(p.plan_dkdv, kPlanDkdv, items, ctas, p.D), stream);
    if (rc) return rc;
  }
  return SA_OK;
}

int launch_bwd_sm100(const AttnParams& p, cudaStream_t stream, int parts) {
  if (!bwd_sm100_eligible(p)) return SA_EUNSUPPORTED;
  if (p.dtype != SA_BF16 && p.dtype != SA_F16) return SA_EUNSUPPORTED;
  if (p.D != 64 && p.D != 128) return SA_EUNSUPPORTED;
  if (p.RB % kRows) return SA_EUNSUPPORTED;
  const void* ptrs[7] = {p.q, p.k, p.v, p.dout, p.dq, p.dk, p.dv};
  for (auto ptr : ptrs)
    if (reinterpret_cast<uintptr_t>(ptr) % 16) return SA_EUNSUPPORTED;
  for (int i = 0; i < 3; ++i)
    if (p.qs[i] % 8 || p.ks[i] % 8 || p.vs[i] % 8 || p.dos[i] % 8 || p.dqs[i] % 8 ||
        p.dks[i] % 8 || p.dvs[i] % 8)
      return SA_EUNSUPPORTED;
  if (p.N > INT32_MAX) return SA_EUNSUPPORTED;
  const bool bf = p.dtype == SA_BF16;
  if (parts & kBwdFused) {
    if (!bwd_fused_eligible(p)) return SA_EUNSUPPORTED;
    return bf ? launch_fused_t<true>(p, stream) : launch_fused_t<false>(p, stream);
  }
  if (p.D == 64) return bf ? launch_t<64, true>(p, stream, parts) : launch_t<64, false>(p, stream, parts);
  return bf ? launch_t<128, true>(p, stream, parts) : launch_t<128, false>(p, stream, parts);
}

}  // namespace sa

// Block-list attention forward on sm_100a: TMA + tcgen05 (TMEM accumulators).
//
// Same semantics as src/ultrametric/block_list.py:387-470 of sparse-ai (walk only the
// query block's own list, token-level causal and tail masks, exp2 online softmax, empty rows
// -> 0 / lse -inf, natural-log LSE, optional per-(row block, slot) logit bias).
//
// Persistent kernel, one CTA per SM, 6 warps:
//   warp 0      TMA producer: Q tile once per work item, K/V tiles of each listed key block
//               into a 2-stage ring (128 x D bf16/fp16 tiles, 128-byte swizzle).
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer:
//                 S[t%2] = Q K_t^T   (M=128, N=128, K=D; fp32 in TMEM)
//                 O     += P_{t} V_t (M=128, N=D,   K=128; fp32 in TMEM)
//               QK of tile t+1 is issued before PV of tile t so the tensor core works while
//               the softmax warps process S_t.
//   warps 2-5   softmax: thread = query row (TMEM lane); tcgen05.ld of S, masking, row max,
//               exp2, P (bf16/fp16) written to shared memory in the MMA's swizzled K-major
//               layout; O rescaled in TMEM only when the row max grows by more than 2^8
//               (lazy rescale); epilogue O / l -> global, LSE.
// Work item = (query tile of 128 rows, z, h).  With a planner workspace the items come
// heaviest-first from the device-built queue (one atomic per item); without one, round-robin
// with late (heavier, under causal masking) query tiles first.
#include <string>
#include <type_traits>

#include "sched.cuh"

namespace sa {
namespace {

constexpr int kT = 128;           // rows of a query tile and of a key tile
constexpr int kFwdThreads = 192;  // 6 warps
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColO = 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct FwdArgs {
  CUtensorMap tm_q, tm_k, tm_v;
  int64_t Z, H, Hkv, N, RB, NB, QT;
  const int32_t* lists;
  int64_t list_stride;
  const int32_t* counts;
  const void* bias;
  int bias_dtype;
  int64_t bs[4];
  void* out;
  int64_t os[4];
  float* lse;
  int causal;
  float scale;
  int accumulate;  // continue the online softmax from the O / LSE already in out / lse
  unsigned* status;
  SchedArgs sched;
};

template <int D>
struct FwdLayout {
  static constexpr uint32_t kTileBytes = kT * D * 2;  // one 128 x D half-precision tile
  static constexpr uint32_t kQ = 0;
  static constexpr uint32_t kK0 = kQ + kTileBytes;
  static constexpr uint32_t kV0 = kK0 + 2 * kTileBytes;
  static constexpr uint32_t kP = kV0 + 2 * kTileBytes;
  static constexpr uint32_t kBars = kP + kT * kT * 2;
  static constexpr uint32_t kMeta = kBars + 256;  // TileMeta[2]
  static constexpr uint32_t kRingOff = kMeta + 64;  // WorkEntry[kRing]
  static constexpr uint32_t kBytes = kRingOff + 128;
  static constexpr uint32_t kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
};

// barrier slots
enum { B_QFULL = 0, B_QEMPTY, B_KFULL0, B_KFULL1, B_KEMPTY0, B_KEMPTY1, B_VFULL0, B_VFULL1,
       B_VEMPTY0, B_VEMPTY1, B_SFULL0, B_SFULL1, B_SEMPTY0, B_SEMPTY1, B_PFULL, B_ODONE,
       B_WFULL0, B_WEMPTY0 = B_WFULL0 + kRing, B_NUM = B_WEMPTY0 + kRing };

// Per K/V stage: what the producer learned from the lists, handed to the softmax warps
// through shared memory (released by the stage's V mbarrier) so that no consumer reads
// the lists from global memory on its critical path.
struct TileMeta {
  int64_t key_start;
  float b2;  // soft-bias * log2(e) of the block pair
  int pad;
};

struct ItemInfo {
  int64_t z, h, hk, q_start, qb, row_id;
};

__device__ __forceinline__ ItemInfo item_info(const FwdArgs& a, int64_t item) {
  ItemInfo it;
  const int64_t zh_total = a.Z * a.H;
  const int64_t qt = a.QT - 1 - item / zh_total;
  const int64_t zh = item % zh_total;
  it.z = zh / a.H;
  it.h = zh % a.H;
  it.hk = it.h / (a.H / a.Hkv);
  it.q_start = qt * kT;
  it.qb = it.q_start / a.RB;
  it.row_id = zh * a.NB + it.qb;
  return it;
}

// 128-key tiles of an item (its whole list): the static-schedule weight.
__device__ __forceinline__ int item_tiles(const FwdArgs& a, int64_t item) {
  const ItemInfo it = item_info(a, item);
  return a.counts[it.row_id] * (int)(a.RB / kT);
}

__device__ __forceinline__ int64_t key_start_of(const FwdArgs& a, const ItemInfo& it, int t) {
  const int spb = (int)(a.RB / kT);
  const int64_t kb = a.lists[it.row_id * a.list_stride + t / spb];
  return kb * a.RB + (int64_t)(t % spb) * kT;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi, bool bf16) {
  uint32_t r;
  if (bf16)
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kFwdThreads, 1) fwd_sm100_kernel(const __grid_constant__ FwdArgs a) {
  using L = FwdLayout<D>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::kBars);
  TileMeta* meta = reinterpret_cast<TileMeta*>(sm + L::kMeta);  // [2], one per K/V stage
  WorkEntry* ring = reinterpret_cast<WorkEntry*>(sm + L::kRingOff);
  __shared__ uint32_t s_tmem_base;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bars[B_QFULL], 1);
    mbar_init(&bars[B_QEMPTY], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[B_KFULL0 + i], 1);
      mbar_init(&bars[B_KEMPTY0 + i], 1);
      mbar_init(&bars[B_VFULL0 + i], 1);
      mbar_init(&bars[B_VEMPTY0 + i], 1);
      mbar_init(&bars[B_SFULL0 + i], 1);
      mbar_init(&bars[B_SEMPTY0 + i], 128);
    }
    mbar_init(&bars[B_PFULL], 128);
    mbar_init(&bars[B_ODONE], 1);
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&bars[B_WFULL0 + i], 1);
      mbar_init(&bars[B_WEMPTY0 + i], 1 + 128);  // the MMA thread and the softmax threads
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&a.tm_q);
      prefetch_tmap(&a.tm_k);
      prefetch_tmap(&a.tm_v);
      uint32_t kv = 0, jq = 0;
      bool ok = true;
      auto weight = [&](int64_t i) { return item_tiles(a, i); };
      WorkFetcher fetch;
      fetch.init(&a.sched, weight);
      for (uint32_t w = 0; ok; ++w) {
        const WorkEntry e = fetch.next(weight);
        if (!(ok = ring_put(ring, &bars[B_WFULL0], &bars[B_WEMPTY0], w, e, a.status))) break;
        if (e.item < 0) break;
        const ItemInfo it = item_info(a, e.item);
        if (e.end == e.begin) {
          fetch.reserve(weight);
          continue;
        }
        ok = mbar_wait(&bars[B_QEMPTY], (jq & 1) ^ 1, a.status);
        if (!ok) break;
        mbar_arrive_expect_tx(&bars[B_QFULL], L::kTileBytes);
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sm + L::kQ + c * kT * 128, &a.tm_q, &bars[B_QFULL], c * 64,
                      (int)it.q_start, (int)it.h, (int)it.z);
        ++jq;
        for (int t = e.begin; t < e.end && ok; ++t, ++kv) {
          const int64_t ks = key_start_of(a, it, t);
          const uint32_t st = kv & 1, ph = (kv >> 1) & 1;
          ok = mbar_wait(&bars[B_KEMPTY0 + st], ph ^ 1, a.status);
          if (!ok) break;
          mbar_arrive_expect_tx(&bars[B_KFULL0 + st], L::kTileBytes);
          for (int c = 0; c < D / 64; ++c)
            tma_load_4d(sm + L::kK0 + st * L::kTileBytes + c * kT * 128, &a.tm_k,
                        &bars[B_KFULL0 + st], c * 64, (int)ks, (int)it.hk, (int)it.z);
          ok = mbar_wait(&bars[B_VEMPTY0 + st], ph ^ 1, a.status);
          if (!ok) break;
          meta[st].key_start = ks;
          meta[st].b2 = a.bias ? load_any_f32(a.bias, a.bias_dtype,
                                              it.z * a.bs[0] + it.h * a.bs[1] + it.qb * a.bs[2] +
                                                  (t / (int)(a.RB / kT)) * a.bs[3]) *
                                     kLog2e
                               : 0.f;
          mbar_arrive_expect_tx(&bars[B_VFULL0 + st], L::kTileBytes);
          for (int c = 0; c < D / 64; ++c)
            tma_load_4d(sm + L::kV0 + st * L::kTileBytes + c * kT * 128, &a.tm_v,
                        &bars[B_VFULL0 + st], c * 64, (int)ks, (int)it.hk, (int)it.z);
          if (t == e.end - 1) fetch.reserve(weight);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_f16(kT, kT, BF16, false, false);
      constexpr uint32_t idesc_pv = idesc_f16(kT, D, BF16, false, true);
      const uint32_t q_addr = smem_u32(sm + L::kQ);
      const uint32_t p_addr = smem_u32(sm + L::kP);
      uint32_t kv = 0, s_it = 0, pv = 0, jq = 0;
      bool ok = true;
      auto issue_pv = [&](uint32_t kv_u, bool first) -> bool {
        const uint32_t st = kv_u & 1, ph = (kv_u >> 1) & 1;
        if (!mbar_wait(&bars[B_PFULL], pv & 1, a.status)) return false;
        if (!mbar_wait(&bars[B_VFULL0 + st], ph, a.status)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sm + L::kV0 + st * L::kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kT / 16; ++kk) {
          const uint64_t ad = smem_desc(p_addr + (kk >> 2) * (kT * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = smem_desc(v_addr + kk * 16 * 128, kT * 128, 1024);
          tc_mma_f16(tmem + kColO, ad, bd, idesc_pv, (!first || kk > 0) ? 1u : 0u);
        }
        tc_commit(&bars[B_ODONE]);
        tc_commit(&bars[B_VEMPTY0 + st]);
        ++pv;
        return true;
      };
      for (uint32_t w = 0; ok; ++w) {
        WorkEntry e;
        if (!(ok = ring_get(ring, &bars[B_WFULL0], &bars[B_WEMPTY0], w, e, a.status))) break;
        if (e.item < 0) break;
        const int n_sub = e.end - e.begin;
        if (n_sub == 0) continue;
        ok = mbar_wait(&bars[B_QFULL], jq & 1, a.status);
        ++jq;
        if (!ok) break;
        const uint32_t kv0 = kv;
        for (int t = 0; t < n_sub && ok; ++t, ++kv) {
          const uint32_t st = kv & 1, ph = (kv >> 1) & 1;
          const uint32_t sb = s_it & 1, sph = (s_it >> 1) & 1;
          ok = mbar_wait(&bars[B_KFULL0 + st], ph, a.status) &&
               mbar_wait(&bars[B_SEMPTY0 + sb], sph ^ 1, a.status);
          if (!ok) break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sm + L::kK0 + st * L::kTileBytes);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * (kT * 128) + (kk & 3) * 32;
            tc_mma_f16(tmem + (sb ? kColS1 : kColS0), smem_desc(q_addr + off, 16, 1024),
                       smem_desc(k_addr + off, 16, 1024), idesc_qk, kk > 0 ? 1u : 0u);
          }
          tc_commit(&bars[B_SFULL0 + sb]);
          tc_commit(&bars[B_KEMPTY0 + st]);
          if (t == n_sub - 1) tc_commit(&bars[B_QEMPTY]);
          ++s_it;
          if (t > 0) ok = issue_pv(kv0 + t - 1, t - 1 == 0 && !a.accumulate);
        }
        if (ok) ok = issue_pv(kv0 + n_sub - 1, n_sub == 1 && !a.accumulate);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax warps
    const int quarter = warp & 3;
    const int rl = quarter * 32 + lane;  // row within the tile == TMEM lane
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    const float scale2 = a.scale * kLog2e;
    unsigned char* p_tile = sm + L::kP;
    uint32_t s_it = 0, od = 0, kv = 0;
    bool ok = true;
    for (uint32_t w = 0; ok; ++w) {
      WorkEntry e;
      if (!(ok = ring_get_warp(ring, &bars[B_WFULL0], &bars[B_WEMPTY0], w, e, a.status))) break;
      if (e.item < 0) break;
      const ItemInfo it = item_info(a, e.item);
      const int n_sub = e.end - e.begin;
      const int64_t row = it.q_start + rl;
      float m_used = -INFINITY, l_sum = 0.f;
      using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      T* orow = static_cast<T*>(a.out) + it.z * a.os[0] + it.h * a.os[1] + row * a.os[2];
      if (a.accumulate && n_sub > 0) {
        // Seed TMEM O and the softmax state with the previous (normalised) output and its
        // LSE: with the reference max at the LSE, that output has weight 1 (l = 1).  The
        // previous item's PV completed before its epilogue read O, so O is free here.
        const float lp = row < a.N ? a.lse[(it.z * a.H + it.h) * a.N + row] : -INFINITY;
        if (lp != -INFINITY) {
          m_used = lp * kLog2e;
          l_sum = 1.f;
        }
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w = make_uint4(0, 0, 0, 0);
            if (lp != -INFINITY) w = *reinterpret_cast<const uint4*>(orow + c * 32 + v * 8);
            const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
            for (int i = 0; i < 8; ++i) o[v * 8 + i] = to_f32<T>(e[i]);
          }
          tmem_st32(lane_addr + kColO + c * 32, o);
        }
        tmem_wait_st();
      }
      for (int t = 0; t < n_sub && ok; ++t, ++kv) {
        const uint32_t sb = s_it & 1, sph = (s_it >> 1) & 1;
        if (!mbar_wait_warp(&bars[B_SFULL0 + sb], sph, a.status)) { ok = false; break; }
        tc_fence_after();
        float s[kT];
#pragma unroll
        for (int c = 0; c < kT / 32; ++c) {
          float chunk[32];
          tmem_ld32(lane_addr + (sb ? kColS1 : kColS0) + c * 32, chunk);
#pragma unroll
          for (int i = 0; i < 32; ++i) s[c * 32 + i] = chunk[i];
        }
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&bars[B_SEMPTY0 + sb]);
        ++s_it;

        // the V stage of this tile stays resident until PV(t), which waits for this warp
        if (!mbar_wait_warp(&bars[B_VFULL0 + (kv & 1)], (kv >> 1) & 1, a.status)) { ok = false; break; }
        const int64_t ks = meta[kv & 1].key_start;
        const float b2 = meta[kv & 1].b2;
        // keys key_start + c are visible for c <= lim (int32, clamped once per tile)
        int64_t lim64 = a.N - 1 - ks;
        if (a.causal) lim64 = min(lim64, row - ks);
        const int lim = (int)max((int64_t)-1, min((int64_t)kT, lim64));
        float mt = -INFINITY;
        if (lim >= kT - 1) {
#pragma unroll
          for (int c = 0; c < kT; ++c) {
            s[c] = fmaf(s[c], scale2, b2);
            mt = fmaxf(mt, s[c]);
          }
        } else {
#pragma unroll
          for (int c = 0; c < kT; ++c) {
            s[c] = c <= lim ? fmaf(s[c], scale2, b2) : -INFINITY;
            mt = fmaxf(mt, s[c]);
          }
        }
        // lazy rescale: move the reference max only when it grows by > 2^8
        float m_new = m_used;
        if (mt > -INFINITY && (m_used == -INFINITY || mt > m_used + kRescaleThreshold)) m_new = mt;
        const float m_ref = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = (m_used == -INFINITY) ? 1.f : fast_exp2(m_used - m_ref);
        const bool rescale = (m_new != m_used) && (m_used != -INFINITY);
        float rs = 0.f;
        uint32_t pk[kT / 2];
#pragma unroll
        for (int c = 0; c < kT; c += 2) {
          const float p0 = fast_exp2(s[c] - m_ref);
          const float p1 = fast_exp2(s[c + 1] - m_ref);
          rs += p0 + p1;
          pk[c / 2] = pack2(p0, p1, BF16);
        }
        // P buffer and O are free once PV of the previous tile completed (a seeded O is
        // ours from the start)
        if (t > 0) {
          if (!mbar_wait_warp(&bars[B_ODONE], od & 1, a.status)) { ok = false; break; }
          ++od;
          tc_fence_after();
        }
        if (t > 0 || a.accumulate) {
          if (__any_sync(0xffffffffu, rescale)) {
            const float f = rescale ? alpha : 1.f;
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
              float o[32];
              tmem_ld32(lane_addr + kColO + c * 32, o);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] *= f;
              tmem_st32(lane_addr + kColO + c * 32, o);
            }
            tmem_wait_st();
          }
        }
        // P row -> shared memory, 128-byte swizzled K-major (two 64-key chunks)
#pragma unroll
        for (int u = 0; u < kT / 8; ++u) {
          const int kc = u >> 3, unit = u & 7;
          const uint32_t off = kc * (kT * 128) + rl * 128 + ((unit ^ (rl & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(p_tile + off)),
                       "r"(pk[u * 4 + 0]), "r"(pk[u * 4 + 1]), "r"(pk[u * 4 + 2]),
                       "r"(pk[u * 4 + 3])
                       : "memory");
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&bars[B_PFULL]);
        l_sum = (m_used == -INFINITY ? 0.f : l_sum * alpha) + rs;
        if (rescale || m_used == -INFINITY) m_used = m_new;
      }
      if (!ok) break;
      // ---------------------------------------------------------------- epilogue
      float inv = 0.f;
      if (n_sub > 0) {
        if (!mbar_wait_warp(&bars[B_ODONE], od & 1, a.status)) { ok = false; break; }
        ++od;
        tc_fence_after();
        inv = 1.f / (l_sum == 0.f ? 1.f : l_sum);
      }
      if (a.accumulate && n_sub == 0) continue;  // nothing new: out / lse stay as they are
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float o[32];
        if (n_sub > 0) {
          tmem_ld32(lane_addr + kColO + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (row < a.N) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack2(o[v * 8 + 0] * inv, o[v * 8 + 1] * inv, BF16);
            w.y = pack2(o[v * 8 + 2] * inv, o[v * 8 + 3] * inv, BF16);
            w.z = pack2(o[v * 8 + 4] * inv, o[v * 8 + 5] * inv, BF16);
            w.w = pack2(o[v * 8 + 6] * inv, o[v * 8 + 7] * inv, BF16);
            *reinterpret_cast<uint4*>(orow + c * 32 + v * 8) = w;
          }
        }
      }
      tc_fence_before();
      if (a.lse && row < a.N)
        a.lse[(it.z * a.H + it.h) * a.N + row] =
            n_sub > 0 ? (m_used + log2f(l_sum)) * kLn2 : -INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, bool BF16>
int launch_t(const AttnParams& p, cudaStream_t stream) {
  FwdArgs a{};
  int rc = make_tmap_4d(&a.tm_q, p.q, p.dtype, p.Z, p.H, p.N, D, p.qs, 64, kT);
  if (!rc) rc = make_tmap_4d(&a.tm_k, p.k, p.dtype, p.Z, p.Hkv, p.N, D, p.ks, 64, kT);
  if (!rc) rc = make_tmap_4d(&a.tm_v, p.v, p.dtype, p.Z, p.Hkv, p.N, D, p.vs, 64, kT);
  // The shape passed the eligibility checks: a failure here is an error, never a silent
  // hand-off to the CUDA-core kernel.
  if (rc) return fail(SA_ELAUNCH, std::string("forward tensor maps: ") + sa_last_error());
  a.Z = p.Z;
  a.H = p.H;
  a.Hkv = p.Hkv;
  a.N = p.N;
  a.RB = p.RB;
  a.NB = p.NB;
  a.QT = (p.N + kT - 1) / kT;
  a.lists = p.lists;
  a.list_stride = p.list_stride;
  a.counts = p.counts;
  a.bias = p.bias;
  a.bias_dtype = p.bias_dtype;
  for (int i = 0; i < 4; ++i) {
    a.bs[i] = p.bs[i];
    a.os[i] = p.os[i];
  }
  a.out = p.out;
  a.lse = p.lse;
  a.causal = p.causal;
  a.scale = p.scale;
  a.accumulate = p.accumulate;
  a.status = p.status;
  const int64_t items = a.Z * a.H * a.QT;
  const int grid = (int)std::min<int64_t>(items, device_sm_count());
  a.sched = SchedArgs{nullptr, nullptr, items};
  if (p.plan_fwd) {
    const PlanPtrs pp = plan_carve(p.plan_fwd, kPlanFwd, items, grid, D);
    rc = launch_plan(kPlanFwd, p, items, grid, pp, stream);
    if (rc) return rc;
    a.sched = SchedArgs{pp.header, pp.queue, items};
  }
  auto kern = fwd_sm100_kernel<D, BF16>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FwdLayout<D>::kAlloc);
  kern<<<grid, kFwdThreads, FwdLayout<D>::kAlloc, stream>>>(a);
  return check_launch("fwd_sm100_kernel");
}

}  // namespace

int64_t fwd_plan_bytes(int64_t Z, int64_t H, int64_t N, int64_t D) {
  const int64_t items = Z * H * ((N + kT - 1) / kT);
  return plan_workspace_bytes(kPlanFwd, items, (int)std::min<int64_t>(items, device_sm_count()), D);
}

int launch_fwd_sm100(const AttnParams& p, cudaStream_t stream) {
  if (p.dtype != SA_BF16 && p.dtype != SA_F16) return SA_EUNSUPPORTED;
  if (p.D != 64 && p.D != 128) return SA_EUNSUPPORTED;
  if (p.RB % kT) return SA_EUNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(p.out) % 16) return SA_EUNSUPPORTED;
  for (int i = 0; i < 3; ++i)
    if (p.os[i] % 8 || p.qs[i] % 8 || p.ks[i] % 8 || p.vs[i] % 8) return SA_EUNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(p.q) % 16 || reinterpret_cast<uintptr_t>(p.k) % 16 ||
      reinterpret_cast<uintptr_t>(p.v) % 16)
    return SA_EUNSUPPORTED;
  if (p.N > INT32_MAX || p.H > INT32_MAX) return SA_EUNSUPPORTED;
  const bool bf = p.dtype == SA_BF16;
  if (p.D == 64) return bf ? launch_t<64, true>(p, stream) : launch_t<64, false>(p, stream);
  return bf ? launch_t<128, true>(p, stream) : launch_t<128, false>(p, stream);
}

}  // namespace sa

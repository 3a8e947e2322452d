// Block-list attention forward on sm_100a: TMA + tcgen05 (TMEM accumulators).
//
// Same semantics as src/ultrametric/block_list.py:387-470 of sparse-ai (walk only the
// query block's own list, token-level causal and tail masks, exp2 online softmax, empty rows
// -> 0 / lse -inf, natural-log LSE, optional per-(row block, slot) logit bias).
//
// Persistent kernel, one CTA per SM, 12 warps (softmax warpgroups raised to 216 registers with
// setmaxnreg, the control warpgroup lowered to 72):
//   warp 10     scheduler: takes work entries (queue atomic or round-robin), computes each
//               item's indices once, reads its list 32 entries per coalesced warp load and
//               pushes one key start (+ soft bias) per key tile into an 8-slot shared ring,
//               and prefetches each item's Q tile into L2 (an L2 prefetch of every K/V tile as
//               well measured slower: it shares the SM's TMA throughput with the loads).
//   warp 8      TMA producer: Q tile once per work item, K tiles into a 2-stage ring and V
//               tiles into another, as three channels polled without blocking (each in order,
//               none waiting behind another); it never touches global memory itself.
//   warp 9      TMEM owner + QK issuer (one thread): S[g] = Q K_t^T (M=128, N=128, K=D; fp32
//               in TMEM), every key tile in order as soon as its K stage and S[g] are free.
//   warp 11     PV issuer (one thread): O[g] += P_t V_t (M=128, N=D, K=128; fp32 in TMEM), every
//               key tile in order as soon as the group's P and the tile's V are in shared
//               memory.  A thread issuing tcgen05.mma is held at each issue while the tensor
//               pipe is busy; with both kinds on one thread the pipe idled through every wait,
//               fence and commit between its MMA blocks (~45 % of each tile pair, traced).
//               Key tiles alternate between the two softmax groups (g = running tile index
//               mod 2, across items).
//   warps 0-7   two softmax groups of 4 warps, each with its own running max / sum and O[g].
//               Thread = query row (TMEM lane); tcgen05.ld of S, masking (-inf in place),
//               row max, exp2, P (bf16/fp16) into the group's shared-memory P buffer in the
//               MMA's swizzled K-major layout; O[g] rescaled in TMEM only when the row max
//               grows by more than 2^8 (lazy rescale).
//               Epilogue of an item of >= 2 tiles: the groups swap (max, sum) per row through
//               shared memory and each merges O[0] and O[1] for half of the head dim; of a
//               one-tile item: its owner alone.  O / l is staged (128B swizzle) in the P
//               buffer and written by TMA tile stores; LSE.
// Work item = (query tile of 128 rows, z, h).  With a planner workspace the items come
// heaviest-first from the device-built queue (one atomic per item; two per atomic when every
// item has the same weight of at most one list entry); without one, round-robin with late
// (heavier, under causal masking) query tiles first.
#include <string>
#include <type_traits>

#include "sched.cuh"

namespace sa {
namespace {

constexpr int kT = 128;           // rows of a query tile and of a key tile
constexpr int kFwdThreads = 384;  // 12 warps
constexpr int kProducerWarp = 8, kMmaWarp = 9, kSchedWarp = 10, kPvWarp = 11;
// Register split: the launch gives every thread kLaunchRegs; the control warpgroup (warps
// 8-11) drops to kCtrlRegs and the two softmax warpgroups take what it frees.
constexpr int kLaunchRegs = 168, kCtrlRegs = 72, kSoftmaxRegs = 216;
static_assert(4 * 32 * kCtrlRegs + 8 * 32 * kSoftmaxRegs <= kFwdThreads * kLaunchRegs,
              "register split exceeds the launch allocation");
constexpr int kGroupThreads = 128;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;    // S[g] at kColS + g * kT
constexpr uint32_t kColO = 256;  // O[g] at kColO + g * D
constexpr int kKeyRing = 8;  // key tiles the scheduler may run ahead of the V loads
constexpr uint32_t kMaxSmem = 232448;      // opt-in dynamic shared memory per block
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct FwdArgs {
  CUtensorMap tm_q, tm_k, tm_v, tm_o;
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

// barrier slots
enum {
  B_QFULL = 0, B_QEMPTY,
  B_KFULL0, B_KEMPTY0 = B_KFULL0 + 2, B_VFULL0 = B_KEMPTY0 + 2, B_VEMPTY0 = B_VFULL0 + 2,
  B_SFULL0 = B_VEMPTY0 + 2, B_SEMPTY0 = B_SFULL0 + 2, B_PFULL0 = B_SEMPTY0 + 2,
  B_ODONE0 = B_PFULL0 + 2, B_XCH = B_ODONE0 + 2, B_EPI, B_EPI1_0,
  B_OFULL0 = B_EPI1_0 + 2, B_ODRAIN0 = B_OFULL0 + 2, B_KEYFULL0 = B_ODRAIN0 + 2,
  B_KEYEMPTY0 = B_KEYFULL0 + kKeyRing,
  B_WFULL0 = B_KEYEMPTY0 + kKeyRing, B_WEMPTY0 = B_WFULL0 + kRing, B_NUM = B_WEMPTY0 + kRing
};

template <int D>
struct FwdLayout {
  static constexpr uint32_t kTileBytes = kT * D * 2;  // one 128 x D half-precision tile
  static constexpr uint32_t kPBytes = kT * kT * 2;    // one 128 x 128 P tile
  static constexpr uint32_t kQ = 0;
  static constexpr uint32_t kK0 = kQ + kTileBytes;
  static constexpr uint32_t kV0 = kK0 + 2 * kTileBytes;
  static constexpr uint32_t kP0 = kV0 + 2 * kTileBytes;  // P[2], one per softmax group
  static constexpr uint32_t kBars = kP0 + 2 * kPBytes;
  static constexpr uint32_t kKeys = kBars + 448;              // TileKey[kKeyRing]
  static constexpr uint32_t kRingOff = kKeys + kKeyRing * 16;  // WorkEntry[kRing]
  static constexpr uint32_t kPos = kRingOff + 64;               // ItemPos[kRing]
  static constexpr uint32_t kML = kPos + 64;                    // float2 [2][kT]: (max, sum)
  static constexpr uint32_t kTmemSlot = kML + 2 * kT * 8;
  static constexpr uint32_t kBytes = kTmemSlot + 16;
  // up to 1024 bytes of slack for aligning the tiles, as far as the opt-in limit allows; the
  // kernel checks the padding it needs against %dynamic_smem_size
  static constexpr uint32_t kAlloc = kBytes + 1024 <= kMaxSmem ? kBytes + 1024 : kMaxSmem;
  static_assert(kBytes <= kMaxSmem, "forward shared-memory layout too large");
  static_assert(B_NUM * 8 <= 448, "barrier area too small");
  static_assert(kRing * 16 <= 64, "work ring area too small");
};

// Per key tile: what the scheduler read from the lists, handed to the producer (K and V loads)
// and to the owning softmax group (masking, bias) through a shared-memory ring, so that
// neither reads the lists from global memory on its critical path.
struct TileKey {
  int key_start;  // < N <= INT32_MAX (checked at launch)
  float b2;       // soft-bias * log2(e) of the block pair
  int hk, z;      // KV head and batch index of the tile's item
};

struct ItemInfo {
  int64_t z, h, hk, q_start, qb, row_id;
};

// What the softmax groups need of a work item, computed once by the producer beside the work
// entry (no 64-bit index division on the groups' path between items).
struct ItemPos {
  int z, h, hk, q_start;
};

// Item indices are int (WorkEntry), so the index arithmetic runs in 32 bits: the scheduler
// decodes one item per work entry on its serial path, where 64-bit divisions cost hundreds of
// cycles each.
__device__ __forceinline__ ItemInfo item_info(const FwdArgs& a, int64_t item) {
  ItemInfo it;
  const uint32_t i = (uint32_t)item, zh_total = (uint32_t)(a.Z * a.H), H = (uint32_t)a.H;
  const uint32_t qi = i / zh_total, zh = i - qi * zh_total;
  const uint32_t qt = (uint32_t)a.QT - 1 - qi;
  const uint32_t z = zh / H, h = zh - z * H;
  it.z = z;
  it.h = h;
  it.hk = h / (H / (uint32_t)a.Hkv);
  it.q_start = (int64_t)qt * kT;
  it.qb = qt / (uint32_t)(a.RB / kT);
  it.row_id = (int64_t)zh * a.NB + it.qb;
  return it;
}

// 128-key tiles of an item (its whole list): the static-schedule weight.
__device__ __forceinline__ int item_tiles(const FwdArgs& a, int64_t item) {
  const ItemInfo it = item_info(a, item);
  return a.counts[it.row_id] * (int)(a.RB / kT);
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
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
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
  TileKey* keys = reinterpret_cast<TileKey*>(sm + L::kKeys);
  WorkEntry* ring = reinterpret_cast<WorkEntry*>(sm + L::kRingOff);
  ItemPos* pos = reinterpret_cast<ItemPos*>(sm + L::kPos);
  float2* s_ml = reinterpret_cast<float2*>(sm + L::kML);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::kTmemSlot);

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
      mbar_init(&bars[B_SEMPTY0 + i], kGroupThreads);
      mbar_init(&bars[B_PFULL0 + i], kGroupThreads);
      mbar_init(&bars[B_ODONE0 + i], 1);
    }
    mbar_init(&bars[B_XCH], 2 * kGroupThreads);
    mbar_init(&bars[B_EPI], 2 * kGroupThreads);
    mbar_init(&bars[B_EPI1_0], kGroupThreads);  // a one-tile item's owner has read O[0]
    mbar_init(&bars[B_EPI1_0 + 1], kGroupThreads);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[B_OFULL0 + i], kGroupThreads);  // output rows staged for the TMA store
      mbar_init(&bars[B_ODRAIN0 + i], 1);             // that store has read its staging buffer
    }
    for (int i = 0; i < kKeyRing; ++i) {
      mbar_init(&bars[B_KEYFULL0 + i], 1);
      mbar_init(&bars[B_KEYEMPTY0 + i], 1 + kGroupThreads);  // the producer (after V), the owning group
    }
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&bars[B_WFULL0 + i], 1);
      mbar_init(&bars[B_WEMPTY0 + i], 3 + 2 * kGroupThreads);  // producer, QK and PV issuers, both groups
    }
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp >= kProducerWarp) {
    // control warpgroup: the whole warpgroup lowers its registers, then warps 8 / 9 work
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kCtrlRegs));
  if (warp == kSchedWarp) {
    // ------------------------------------------------------------------ scheduler
    if (lane == 0) {
      prefetch_tmap(&a.tm_q);
      prefetch_tmap(&a.tm_k);
      prefetch_tmap(&a.tm_v);
    }
    // Work entries: the CTA's first is item blockIdx.x (while the planner, this grid's
    // programmatic prerequisite, orders the rest), then one queue atomic per entry -- or
    // round-robin without a planner.  After a one-tile entry the atomic for the next one is
    // issued before this entry's list is read and its key pushed, and resolved after them.
    const SchedArgs& S = a.sched;
    const bool dyn = S.header != nullptr;
    int n_entries = 0, natural = 0;
    bool planner_ready = !dyn || !S.first_static;
    if (dyn && planner_ready && lane == 0) {
      n_entries = S.header->n_entries;
      natural = S.header->natural;
    }
    auto whole = [&](int64_t item) -> WorkEntry {
      return item < S.items ? WorkEntry{(int)item, 0, item_tiles(a, item), -1} : no_work();
    };
    auto resolve = [&](int idx) -> WorkEntry {
      if (idx >= n_entries) return no_work();
      if (natural) {  // every queued item weighs natural - 1 tiles: no count to load
        const int64_t item = (S.first_static ? (int64_t)gridDim.x : 0) + idx;
        return item < S.items ? WorkEntry{(int)item, 0, natural - 1, -1} : no_work();
      }
      return S.queue[idx];
    };
    WorkEntry e_next{};
    if (lane == 0) {
      if (!dyn || S.first_static) {
        e_next = whole(blockIdx.x);
      } else {
        e_next = resolve(atomicAdd(&S.header->counter, 1));
      }
    }
    const int spb = (int)(a.RB / kT);  // key tiles per list entry
    uint32_t kq = 0;                   // key tiles pushed
    bool ok = true, batch = false;
    uint32_t w = 0;  // ring entries pushed
    for (; ok; ++w) {
      WorkEntry e{};
      e.item = __shfl_sync(0xffffffffu, e_next.item, 0);
      e.begin = __shfl_sync(0xffffffffu, e_next.begin, 0);
      e.end = __shfl_sync(0xffffffffu, e_next.end, 0);
      e.slot = __shfl_sync(0xffffffffu, e_next.slot, 0);
      // An entry of one key tile is over in about the scheduler's own serial latency per entry
      // (atomic, index decode, list load): take the next entry's atomic now and use it after
      // this entry's key.  Longer entries reserve after their keys as before: reserved any
      // earlier, an entry sits unstarted while other CTAs may run dry (measured slower at C2).
      const bool early = dyn && e.item >= 0 && planner_ready && e.end - e.begin <= 1;
      int idx_next = 0;
      if (lane == 0 && early) idx_next = atomicAdd(&S.header->counter, 1);
      ItemInfo it{};
      if (e.item >= 0) it = item_info(a, e.item);
      if (lane == 0) {
        const uint32_t slot = w % kRing;
        ok = mbar_wait(&bars[B_WEMPTY0 + slot], ((w / kRing) & 1) ^ 1, a.status);
        if (ok) {
          ring[slot] = e;
          pos[slot] = ItemPos{(int)it.z, (int)it.h, (int)it.hk, (int)it.q_start};
          mbar_arrive(&bars[B_WFULL0 + slot]);
          if (e.item >= 0 && e.end > e.begin)
            for (int c = 0; c < D / 64; ++c)
              tma_prefetch_4d(&a.tm_q, c * 64, (int)it.q_start, (int)it.h, (int)it.z);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok || e.item < 0) break;
      // list entries [p0, p1) cover the entry's key tiles; one coalesced load per 32
      const int p0 = e.begin / spb, p1 = e.end > e.begin ? (e.end - 1) / spb + 1 : p0;
      for (int pc = p0; pc < p1 && ok; pc += 32) {
        const int p = pc + lane;
        int kb = 0;
        float bb = 0.f;
        if (p < p1) {
          kb = a.lists[it.row_id * a.list_stride + p];
          if (a.bias)
            bb = load_any_f32(a.bias, a.bias_dtype,
                              it.z * a.bs[0] + it.h * a.bs[1] + it.qb * a.bs[2] + (int64_t)p * a.bs[3]) *
                 kLog2e;
        }
        const int t_lo = max(e.begin, pc * spb), t_hi = min(e.end, (pc + 32) * spb);
        for (int t = t_lo; t < t_hi; ++t) {
          const int src = t / spb - pc;
          const int64_t ks = (int64_t)__shfl_sync(0xffffffffu, kb, src) * a.RB + (int64_t)(t % spb) * kT;
          const float b2 = __shfl_sync(0xffffffffu, bb, src);
          if (lane == 0) {
            const uint32_t slot = kq % kKeyRing;
            ok = mbar_wait(&bars[B_KEYEMPTY0 + slot], ((kq / kKeyRing) & 1) ^ 1, a.status);
            if (ok) {
              keys[slot] = TileKey{(int)ks, b2, (int)it.hk, (int)it.z};
              mbar_arrive(&bars[B_KEYFULL0 + slot]);
            }
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) break;
          ++kq;
        }
      }
      if (lane == 0) {
        if (!dyn) {
          e_next = whole((int64_t)blockIdx.x + (int64_t)(w + 1) * gridDim.x);
        } else if (early) {
          e_next = resolve(idx_next);
        } else if (planner_ready) {
          e_next = resolve(atomicAdd(&S.header->counter, 1));
        } else {
          // after the first-wave item: the planner's queue and header are complete from here
          pdl_wait();
          planner_ready = true;
          n_entries = S.header->n_entries;
          natural = S.header->natural;
          // every remaining item the same weight, within one list entry: batches below
          batch = natural > 0 && natural - 1 <= spb;
          if (!batch) e_next = resolve(atomicAdd(&S.header->counter, 1));
        }
      }
      if (__shfl_sync(0xffffffffu, batch ? 1 : 0, 0)) {
        ++w;
        break;
      }
    }
    if (__shfl_sync(0xffffffffu, batch ? 1 : 0, 0) && ok) {
      // Uniform small items (very sparse lists, e.g. one key tile per query tile): one queue
      // atomic per kBatch items, taken a batch ahead, and the batch's indices, list entries
      // and biases decoded by kBatch lanes at once, so that a CTA's scheduler is not the
      // serial bottleneck (atomic, index decode, list load per item) of one-tile items.
      // Batches of 4 (up to 8 items held per CTA) left a longer tail at the end of the queue
      // than they saved: 98.4 % forward 0.064 -> 0.069 ms, against 0.063 with 2.
      constexpr int kBatch = 2;
      const int64_t base = (int64_t)gridDim.x;  // natural order: entry k is item grid + k
      const int wu = __shfl_sync(0xffffffffu, natural - 1, 0);
      const int n_ent = __shfl_sync(0xffffffffu, n_entries, 0);
      int idx = 0;
      if (lane == 0) idx = atomicAdd(&S.header->counter, kBatch);
      idx = __shfl_sync(0xffffffffu, idx, 0);
      while (ok && idx < n_ent) {
        int idx_nx = 0;
        if (lane == 0) idx_nx = atomicAdd(&S.header->counter, kBatch);
        ItemInfo itj{};
        int kbj = 0;
        float bbj = 0.f;
        if (lane < kBatch && idx + lane < n_ent) {
          itj = item_info(a, base + idx + lane);
          if (wu > 0) {
            kbj = a.lists[itj.row_id * a.list_stride];
            if (a.bias)
              bbj = load_any_f32(a.bias, a.bias_dtype, itj.z * a.bs[0] + itj.h * a.bs[1] + itj.qb * a.bs[2]) *
                    kLog2e;
          }
        }
        for (int jj = 0; jj < kBatch && ok && idx + jj < n_ent; ++jj, ++w) {
          const int z = __shfl_sync(0xffffffffu, (int)itj.z, jj), h = __shfl_sync(0xffffffffu, (int)itj.h, jj);
          const int hk = __shfl_sync(0xffffffffu, (int)itj.hk, jj);
          const int q_start = __shfl_sync(0xffffffffu, (int)itj.q_start, jj);
          const int kb = __shfl_sync(0xffffffffu, kbj, jj);
          const float b2 = __shfl_sync(0xffffffffu, bbj, jj);
          if (lane == 0) {
            const uint32_t slot = w % kRing;
            ok = mbar_wait(&bars[B_WEMPTY0 + slot], ((w / kRing) & 1) ^ 1, a.status);
            if (ok) {
              ring[slot] = WorkEntry{(int)(base + idx + jj), 0, wu, -1};
              pos[slot] = ItemPos{z, h, hk, q_start};
              mbar_arrive(&bars[B_WFULL0 + slot]);
              if (wu > 0)
                for (int c = 0; c < D / 64; ++c) tma_prefetch_4d(&a.tm_q, c * 64, q_start, h, z);
            }
            for (int tt = 0; tt < wu && ok; ++tt, ++kq) {
              const uint32_t ks_slot = kq % kKeyRing;
              ok = mbar_wait(&bars[B_KEYEMPTY0 + ks_slot], ((kq / kKeyRing) & 1) ^ 1, a.status);
              if (ok) {
                keys[ks_slot] = TileKey{(int)((int64_t)kb * a.RB + (int64_t)tt * kT), b2, hk, z};
                mbar_arrive(&bars[B_KEYFULL0 + ks_slot]);
              }
            }
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
        }
        idx = __shfl_sync(0xffffffffu, idx_nx, 0);
      }
      // the terminating entry ends every role's loop
      if (ok && lane == 0) {
        const uint32_t slot = w % kRing;
        if (mbar_wait(&bars[B_WEMPTY0 + slot], ((w / kRing) & 1) ^ 1, a.status)) {
          ring[slot] = no_work();
          mbar_arrive(&bars[B_WFULL0 + slot]);
        }
      }
    }
  } else if (warp == kProducerWarp) {
    // ------------------------------------------------------------------ TMA producer
    // Three load channels, each in order, polled without blocking so that none holds up the
    // others: Q once per work item (its slot frees when the item's last QK completes), K per
    // key tile (its stage frees when QK of the tile two back completes) and V per key tile
    // (when PV of the tile two back completes).  The PVs trail the QKs by a softmax pass, so a
    // producer that waited for each V stage in turn delayed the next K loads and with them
    // the QKs.  A key tile's start, KV head and batch index come from the scheduler's key
    // ring; the slot is handed back after the tile's V load.
    if (lane == 0) {
      uint32_t w = 0, jq = 0, uk = 0, uv = 0, tiles = 0;
      bool ended = false, ok = true;
      // work items read whose Q is not loaded yet (at most two: a Q waits for the previous
      // item's last QK, which waits for at most two K tiles beyond it)
      ItemPos q0{}, q1{};
      int nq = 0;
      long long idle_since = clock64();
      while (true) {
        bool busy = false;
        if (!ended && nq < 2) {
          const uint32_t slot = w % kRing;
          if (mbar_test(&bars[B_WFULL0 + slot], (w / kRing) & 1)) {
            const WorkEntry e = ring[slot];
            const ItemPos ip = pos[slot];
            mbar_arrive(&bars[B_WEMPTY0 + slot]);
            ++w;
            if (e.item < 0) {
              ended = true;
            } else if (e.end > e.begin) {
              tiles += (uint32_t)(e.end - e.begin);
              if (nq == 0) q0 = ip;
              else q1 = ip;
              ++nq;
            }
            busy = true;
          }
        }
        if (nq > 0 && mbar_test(&bars[B_QEMPTY], (jq & 1) ^ 1)) {
          mbar_arrive_expect_tx(&bars[B_QFULL], L::kTileBytes);
          for (int c = 0; c < D / 64; ++c)
            tma_load_4d(sm + L::kQ + c * kT * 128, &a.tm_q, &bars[B_QFULL], c * 64, q0.q_start, q0.h, q0.z);
          q0 = q1;
          --nq;
          ++jq;
          busy = true;
        }
        if (uk < tiles) {
          const uint32_t ks_slot = uk % kKeyRing, st = uk & 1;
          if (mbar_test(&bars[B_KEYFULL0 + ks_slot], (uk / kKeyRing) & 1) &&
              mbar_test(&bars[B_KEMPTY0 + st], ((uk >> 1) & 1) ^ 1)) {
            const TileKey k = keys[ks_slot];
            mbar_arrive_expect_tx(&bars[B_KFULL0 + st], L::kTileBytes);
            for (int c = 0; c < D / 64; ++c)
              tma_load_4d(sm + L::kK0 + st * L::kTileBytes + c * kT * 128, &a.tm_k,
                          &bars[B_KFULL0 + st], c * 64, k.key_start, k.hk, k.z);
            ++uk;
            busy = true;
          }
        }
        if (uv < uk) {
          const uint32_t ks_slot = uv % kKeyRing, st = uv & 1;
          if (mbar_test(&bars[B_VEMPTY0 + st], ((uv >> 1) & 1) ^ 1)) {
            const TileKey k = keys[ks_slot];
            mbar_arrive_expect_tx(&bars[B_VFULL0 + st], L::kTileBytes);
            for (int c = 0; c < D / 64; ++c)
              tma_load_4d(sm + L::kV0 + st * L::kTileBytes + c * kT * 128, &a.tm_v,
                          &bars[B_VFULL0 + st], c * 64, k.key_start, k.hk, k.z);
            mbar_arrive(&bars[B_KEYEMPTY0 + ks_slot]);  // the tile's key slot is done
            ++uv;
            busy = true;
          }
        }
        if (ended && nq == 0 && uv == tiles) break;
        if (busy) {
          idle_since = clock64();
        } else if (clock64() - idle_since > (1ll << 31)) {
          raise_status(a.status, kStatusWaitTimeout);
          ok = false;
          break;
        }
      }
      (void)ok;
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ QK issuer
    // S[g] = Q K^T for every key tile, in order.  The PVs have their own issuing thread
    // (warp kPvWarp): a thread that issues tcgen05.mma is held at each issue while the tensor
    // pipe is busy, so one thread issuing both would leave the pipe idle through every wait,
    // fence and commit between its MMA blocks.  The two threads' MMAs touch disjoint TMEM
    // (S[g] and O[g]) and meet only through the mbarriers below.
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_f16(kT, kT, BF16, false, false);
      const uint64_t qd = smem_desc(smem_u32(sm + L::kQ), 16, 1024);
      uint32_t kv = 0, jq = 0, sq0 = 0, sq1 = 0;
      bool ok = true;
      for (uint32_t w = 0; ok; ++w) {
        WorkEntry e;
        if (!(ok = ring_get(ring, &bars[B_WFULL0], &bars[B_WEMPTY0], w, e, a.status))) break;
        if (e.item < 0) break;
        const int n_sub = e.end - e.begin;
        if (n_sub == 0) continue;
        ok = mbar_wait(&bars[B_QFULL], jq & 1, a.status);
        ++jq;
        if (!ok) break;
        const int gb = (int)(kv & 1);  // tile t goes to group (gb + t) & 1
        for (int t = 0; t < n_sub && ok; ++t) {
          const uint32_t u = kv + t, g = (gb + t) & 1;
          const uint32_t st = u & 1, ph = (u >> 1) & 1;
          ok = mbar_wait(&bars[B_KFULL0 + st], ph, a.status) &&
               mbar_wait(&bars[B_SEMPTY0 + g], ((g ? sq1 : sq0) & 1) ^ 1, a.status);
          if (!ok) break;
          tc_fence_after();
          const uint64_t kd = smem_desc(smem_u32(sm + L::kK0 + st * L::kTileBytes), 16, 1024);
          const uint32_t d_s = tmem + kColS + g * kT;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * (kT * 128) + (kk & 3) * 32;
            tc_mma_f16(d_s, desc_add(qd, off), desc_add(kd, off), idesc_qk, kk > 0 ? 1u : 0u);
          }
          tc_commit(&bars[B_SFULL0 + g]);
          tc_commit(&bars[B_KEMPTY0 + st]);
          if (t == n_sub - 1) tc_commit(&bars[B_QEMPTY]);
          if (g) ++sq1; else ++sq0;
        }
        kv += n_sub;
      }
    }
  } else if (warp == kPvWarp) {
    // ------------------------------------------------------------------ PV issuer
    // O[g] += P[g] V for every key tile, in order, as soon as the group's P and the tile's V
    // are in shared memory.
    if (lane == 0) {
      constexpr uint32_t idesc_pv = idesc_f16(kT, D, BF16, false, true);
      uint32_t kv = 0, pv0 = 0, pv1 = 0, n_multi = 0, n_solo0 = 0, n_solo1 = 0;
      // O[g] is free for a new item once the readers of its last item are done: that item's
      // epilogue barrier and phase (EPI for items of >= 2 tiles, EPI1[g] for one-tile items)
      int guard_bar0 = -1, guard_bar1 = -1;
      uint32_t guard_ph0 = 0, guard_ph1 = 0;
      bool ok = true;
      for (uint32_t w = 0; ok; ++w) {
        WorkEntry e;
        if (!(ok = ring_get(ring, &bars[B_WFULL0], &bars[B_WEMPTY0], w, e, a.status))) break;
        if (e.item < 0) break;
        const int n_sub = e.end - e.begin;
        if (n_sub == 0) continue;
        const int gb = (int)(kv & 1);
        for (int t = 0; t < n_sub && ok; ++t) {
          const uint32_t u = kv + t, g = (gb + t) & 1;
          const uint32_t st = u & 1, ph = (u >> 1) & 1;
          // the group's first PV of the item waits for O[g]'s guard and, unless O[g] was
          // seeded with the previous output (accumulate mode, the first tile's group),
          // starts it afresh
          const bool first_of_g = t < 2, seeded = a.accumulate && t == 0;
          const int gbar = g ? guard_bar1 : guard_bar0;
          const uint32_t gph = g ? guard_ph1 : guard_ph0;
          ok = (!first_of_g || gbar < 0 || mbar_wait(&bars[gbar], gph & 1, a.status)) &&
               mbar_wait(&bars[B_PFULL0 + g], (g ? pv1 : pv0) & 1, a.status) &&
               mbar_wait(&bars[B_VFULL0 + st], ph, a.status);
          if (!ok) break;
          tc_fence_after();
          const uint64_t pd = smem_desc(smem_u32(sm + L::kP0 + g * L::kPBytes), 16, 1024);
          const uint64_t vd = smem_desc(smem_u32(sm + L::kV0 + st * L::kTileBytes), kT * 128, 1024);
          const uint32_t d_o = tmem + kColO + g * D;
          const bool first = first_of_g && !seeded;
#pragma unroll
          for (int kk = 0; kk < kT / 16; ++kk)
            tc_mma_f16(d_o, desc_add(pd, (kk >> 2) * (kT * 128) + (kk & 3) * 32),
                       desc_add(vd, kk * 16 * 128), idesc_pv, (!first || kk > 0) ? 1u : 0u);
          tc_commit(&bars[B_ODONE0 + g]);
          tc_commit(&bars[B_VEMPTY0 + st]);
          if (g) ++pv1; else ++pv0;
        }
        if (!ok) break;
        if (n_sub == 1) {
          if (gb) {
            guard_bar1 = B_EPI1_0 + 1;
            guard_ph1 = n_solo1++;
          } else {
            guard_bar0 = B_EPI1_0;
            guard_ph0 = n_solo0++;
          }
        } else {
          guard_bar0 = guard_bar1 = B_EPI;
          guard_ph0 = guard_ph1 = n_multi++;
        }
        kv += n_sub;
      }
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    // ------------------------------------------------------------------ softmax groups
    const int grp = warp >> 2;
    const int quarter = warp & 3;
    const int rl = quarter * 32 + lane;  // row within the tile == TMEM lane
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    const uint32_t col_s = kColS + grp * kT;
    const uint32_t col_o = kColO + grp * D, col_oo = kColO + (grp ^ 1) * D;
    const float scale2 = a.scale * kLog2e;
    const bool neg_scale = scale2 < 0.f;
    // |scale| (a sign flip of the scores handles a negative one); a zero scale becomes 1e-30,
    // which keeps -inf * scale = -inf for masked keys and changes nothing else representable
    const float sc2 = fmaxf(fabsf(scale2), 1e-30f);
    unsigned char* p_tile = sm + L::kP0 + grp * L::kPBytes;
    const bool issuer = quarter == 0 && lane == 0;  // issues this group's output store
    // n_multi: items of >= 2 tiles so far (XCH / EPI phases); n_solo: one-tile items owned
    uint32_t sc = 0, od = 0, kv = 0, n_multi = 0, n_solo = 0, n_store = 0, n_drain = 0;
    // P[g] is rewritten (P tiles, or the next output staging) only after this group's last
    // output store has read it
    auto drain = [&]() -> bool {
      if (n_drain == n_store) return true;
      if (issuer) {
        tma_store_wait_read();
        mbar_arrive(&bars[B_ODRAIN0 + grp]);
      }
      if (!mbar_wait_warp(&bars[B_ODRAIN0 + grp], n_drain & 1, a.status)) return false;
      ++n_drain;
      return true;
    };
    bool ok = true;
    for (uint32_t w = 0; ok; ++w) {
      WorkEntry e;
      ItemPos ip;
      {
        const uint32_t slot = w % kRing;
        if (!(ok = mbar_wait_warp(&bars[B_WFULL0 + slot], (w / kRing) & 1, a.status))) break;
        e = ring[slot];
        ip = pos[slot];
        mbar_arrive(&bars[B_WEMPTY0 + slot]);
      }
      if (e.item < 0) break;
      const int n_sub = e.end - e.begin;
      const int64_t row = (int64_t)ip.q_start + rl;
      const int64_t zh = (int64_t)ip.z * a.H + ip.h;
      T* orow = static_cast<T*>(a.out) + ip.z * a.os[0] + ip.h * a.os[1] + row * a.os[2];
      if (n_sub == 0) {
        // no key at all: O = 0, lse = -inf (in accumulate mode out / lse stay as they are)
        if (!a.accumulate && row < a.N) {
#pragma unroll
          for (int v = 0; v < D / 16; ++v)
            *reinterpret_cast<uint4*>(orow + grp * (D / 2) + v * 8) = make_uint4(0, 0, 0, 0);
          if (grp == 0 && a.lse) a.lse[zh * a.N + row] = -INFINITY;
        }
        continue;
      }
      // tile t goes to group (gb + t) & 1 (the alternation runs on across items); an item of
      // one tile is finished by its owner alone, the other group skips it
      const int gb = (int)(kv & 1);
      const bool solo = n_sub == 1;
      if (solo && grp != gb) {
        kv += 1;
        continue;
      }
      const int first_t = (grp ^ gb) & 1;
      const int n_mine = n_sub > first_t ? (n_sub - first_t + 1) >> 1 : 0;
      float m_used = -INFINITY, l_sum = 0.f;
      if (a.accumulate && grp == gb) {
        // Seed TMEM O[g] and this group's softmax state with the previous (normalised) output
        // and its LSE: with the reference max at the LSE, that output has weight 1 (l = 1).
        // O[g] is free once the readers of the last multi-tile item are done (a one-tile item
        // that used O[g] was this group's own).
        if (n_multi > 0 && !mbar_wait_warp(&bars[B_EPI], (n_multi - 1) & 1, a.status)) { ok = false; break; }
        const float lp = row < a.N ? a.lse[zh * a.N + row] : -INFINITY;
        if (lp != -INFINITY) {
          m_used = lp * kLog2e;
          l_sum = 1.f;
        }
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 wv = make_uint4(0, 0, 0, 0);
            if (lp != -INFINITY) wv = *reinterpret_cast<const uint4*>(orow + c * 32 + v * 8);
            const T* ev = reinterpret_cast<const T*>(&wv);
#pragma unroll
            for (int i = 0; i < 8; ++i) o[v * 8 + i] = to_f32<T>(ev[i]);
          }
          tmem_st32(lane_addr + col_o + c * 32, o);
        }
        tmem_wait_st();
      }
      for (int j = 0; j < n_mine && ok; ++j) {
        const uint32_t u = kv + first_t + 2 * j;
        if (!mbar_wait_warp(&bars[B_SFULL0 + grp], sc & 1, a.status)) { ok = false; break; }
        ++sc;
        tc_fence_after();
        float s[kT];
#pragma unroll
        for (int c = 0; c < kT / 32; ++c) {
          float chunk[32];
          tmem_ld32(lane_addr + col_s + c * 32, chunk);
#pragma unroll
          for (int i = 0; i < 32; ++i) s[c * 32 + i] = chunk[i];
        }
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&bars[B_SEMPTY0 + grp]);

        const uint32_t ks_slot = u % kKeyRing;
        if (!mbar_wait_warp(&bars[B_KEYFULL0 + ks_slot], (u / kKeyRing) & 1, a.status)) { ok = false; break; }
        const int64_t ks = keys[ks_slot].key_start;
        const float b2 = keys[ks_slot].b2;
        mbar_arrive(&bars[B_KEYEMPTY0 + ks_slot]);
        // keys key_start + c are visible for c <= lim (int32, clamped once per tile); masked
        // scores become -inf in place, so one exp path serves every tile
        int64_t lim64 = a.N - 1 - ks;
        if (a.causal) lim64 = min(lim64, row - ks);
        const int lim = (int)max((int64_t)-1, min((int64_t)kT, lim64));
        if (neg_scale || lim < kT - 1) {
#pragma unroll
          for (int c = 0; c < kT; ++c) {
            const float v = neg_scale ? -s[c] : s[c];
            s[c] = c <= lim ? v : -INFINITY;
          }
        }
        // row max of the raw scores: three-input max, eight independent chains
        float mx[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx[i] = fmaxf(s[2 * i], s[2 * i + 1]);
#pragma unroll
        for (int c = 16; c < kT; c += 2) mx[(c >> 1) & 7] = fmax3(mx[(c >> 1) & 7], s[c], s[c + 1]);
        const float mraw = fmaxf(fmax3(mx[0], mx[1], mx[2]), fmax3(fmax3(mx[3], mx[4], mx[5]), mx[6], mx[7]));
        const float mt = fmaf(mraw, sc2, b2);  // -inf when every key of the tile is masked
        // lazy rescale: move the reference max only when it grows by > 2^8
        float m_new = m_used;
        if (mt > -INFINITY && (m_used == -INFINITY || mt > m_used + kRescaleThreshold)) m_new = mt;
        const float m_ref = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = (m_used == -INFINITY) ? 1.f : fast_exp2(m_used - m_ref);
        const bool rescale = (m_new != m_used) && (m_used != -INFINITY);
        const float bm = b2 - m_ref;
        // exponent arguments and row sums two lanes at a time (f32x2 FMA / add)
        const uint64_t scale_x2 = f32x2(sc2, sc2), bias_x2 = f32x2(bm, bm);
        uint64_t rs[4] = {0, 0, 0, 0};
        uint32_t pk[kT / 2];
#pragma unroll
        for (int c = 0; c < kT; c += 2) {
          float x0, x1;
          f32x2_split(fma_f32x2(f32x2(s[c], s[c + 1]), scale_x2, bias_x2), x0, x1);
          const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
          rs[(c >> 1) & 3] = add_f32x2(rs[(c >> 1) & 3], f32x2(p0, p1));
          pk[c / 2] = pack2(p0, p1, BF16);
        }
        // P[g] and O[g] are free once the group's previous PV completed (a seeded O is ours
        // from the start)
        if (j > 0) {
          if (!mbar_wait_warp(&bars[B_ODONE0 + grp], od & 1, a.status)) { ok = false; break; }
          ++od;
          tc_fence_after();
        }
        if (j > 0 || (a.accumulate && grp == gb)) {
          if (__any_sync(0xffffffffu, rescale)) {
            const float f = rescale ? alpha : 1.f;
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
              float o[32];
              tmem_ld32(lane_addr + col_o + c * 32, o);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] *= f;
              tmem_st32(lane_addr + col_o + c * 32, o);
            }
            tmem_wait_st();
          }
        }
        if (j == 0 && !drain()) { ok = false; break; }
        // P row -> shared memory, 128-byte swizzled K-major (two 64-key chunks)
#pragma unroll
        for (int q = 0; q < kT / 8; ++q) {
          const int kc = q >> 3, unit = q & 7;
          const uint32_t off = kc * (kT * 128) + rl * 128 + ((unit ^ (rl & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(p_tile + off)),
                       "r"(pk[q * 4 + 0]), "r"(pk[q * 4 + 1]), "r"(pk[q * 4 + 2]),
                       "r"(pk[q * 4 + 3])
                       : "memory");
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&bars[B_PFULL0 + grp]);
        float r0, r1;
        f32x2_split(add_f32x2(add_f32x2(rs[0], rs[1]), add_f32x2(rs[2], rs[3])), r0, r1);
        l_sum = (m_used == -INFINITY ? 0.f : l_sum * alpha) + (r0 + r1);
        if (rescale || m_used == -INFINITY) m_used = m_new;
      }
      if (!ok) break;
      // ---------------------------------------------------------------- epilogue
      if (n_mine > 0) {
        if (!mbar_wait_warp(&bars[B_ODONE0 + grp], od & 1, a.status)) { ok = false; break; }
        ++od;
        tc_fence_after();
      }
      // An item of >= 2 tiles: the groups swap (max, sum) per row; the (max, sum) slots are
      // reused once both groups finished the previous such item.  A one-tile item: the owner's
      // own state is the whole result.
      float2 other = make_float2(-INFINITY, 0.f);
      if (!solo) {
        if (n_multi > 0 && !mbar_wait_warp(&bars[B_EPI], (n_multi - 1) & 1, a.status)) { ok = false; break; }
        s_ml[grp * kT + rl] = make_float2(m_used, l_sum);
        mbar_arrive(&bars[B_XCH]);
        if (!mbar_wait_warp(&bars[B_XCH], n_multi & 1, a.status)) { ok = false; break; }
        other = s_ml[(grp ^ 1) * kT + rl];
      }
      const float m = fmaxf(m_used, other.x);
      const float f_s = m == -INFINITY ? 0.f : fast_exp2(m_used - m);
      const float f_o = m == -INFINITY ? 0.f : fast_exp2(other.x - m);
      const float l = l_sum * f_s + other.y * f_o;
      const float inv = 1.f / (l == 0.f ? 1.f : l);
      const float w_s = f_s * inv, w_o = f_o * inv;
      // Columns this group stages: all of them for a one-tile item; otherwise its 64-column half
      // (D = 128) or, for D = 64, group 0 all.  Staging goes to the group's P buffer (free: its
      // last PV completed, the previous store out of it drained) in the TMA store's 128-byte
      // swizzled layout, one 128 x 64 box per 16 KB; one thread then stores the boxes.
      const int cols_lo = solo ? 0 : (D == 128 ? grp * 64 : 0);
      const int n_chunks = solo ? D / 32 : ((D == 128 || grp == 0) ? 2 : 0);
      // both O buffers hold this item's data for a multi-tile item; a one-tile item reads its
      // own twice (weight 0 on the second)
      const uint32_t col_other = solo ? col_o : col_oo;
      if (n_chunks > 0) {
        if (!drain()) { ok = false; break; }
#pragma unroll 1
        for (int c = 0; c < n_chunks; ++c) {
          const uint32_t col = cols_lo + c * 32;
          float os[32], oo[32];
          tmem_ld32(lane_addr + col_o + col, os);
          tmem_ld32(lane_addr + col_other + col, oo);
          tmem_wait_ld();
          unsigned char* box = p_tile + (c >> 1) * (kT * 128);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            float r[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) r[i] = os[v * 8 + i] * w_s + oo[v * 8 + i] * w_o;
            const uint32_t off = rl * 128 + (((((c & 1) * 4) + v) ^ (rl & 7)) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(box + off)),
                         "r"(pack2(r[0], r[1], BF16)), "r"(pack2(r[2], r[3], BF16)),
                         "r"(pack2(r[4], r[5], BF16)), "r"(pack2(r[6], r[7], BF16))
                         : "memory");
          }
        }
        fence_proxy_async_smem();
      }
      tc_fence_before();
      // O[0] / O[1] (and the (max, sum) slots) are read
      mbar_arrive(solo ? &bars[B_EPI1_0 + grp] : &bars[B_EPI]);
      if (n_chunks > 0) {
        mbar_arrive(&bars[B_OFULL0 + grp]);
        if (issuer) {
          if (mbar_wait(&bars[B_OFULL0 + grp], n_store & 1, a.status)) {
            for (int b = 0; b < n_chunks / 2; ++b)
              tma_store_4d(&a.tm_o, p_tile + b * (kT * 128), cols_lo + b * 64, ip.q_start, ip.h, ip.z);
          } else {
            ok = false;
          }
        }
        __syncwarp();
        ok = __all_sync(0xffffffffu, ok);
        ++n_store;
        if (!ok) break;
      }
      if ((solo || grp == 0) && a.lse && row < a.N)
        a.lse[zh * a.N + row] = m == -INFINITY ? -INFINITY : (m + log2f(l)) * kLn2;
      kv += n_sub;
      if (solo)
        ++n_solo;
      else
        ++n_multi;
    }
  }

  // output stores still in flight must have read their staging buffers (and finished) before
  // the CTA's shared memory goes away
  if (warp < kProducerWarp && (warp & 3) == 0 && lane == 0)
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
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
  if (!rc) rc = make_tmap_4d(&a.tm_o, p.out, p.dtype, p.Z, p.H, p.N, D, p.os, 64, kT);
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
  auto kern = fwd_sm100_kernel<D, BF16>;
  // setmaxnreg.inc waits until the registers it asks for are free: launch only when the
  // per-thread launch allocation is the one the split was sized against.
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess || fa.numRegs != kLaunchRegs)
    return fail(SA_ELAUNCH, "forward kernel: launch register count " + std::to_string(fa.numRegs) +
                                " differs from the register split's " + std::to_string(kLaunchRegs));
  a.sched = SchedArgs{nullptr, nullptr, items, 0};
  if (p.plan_fwd) {
    // Each CTA's first item is its own index (the static order starts with the late query
    // tiles, heavy under causal masking); the planner orders the rest heaviest-first while
    // that first wave runs: the kernel is its programmatic dependent and waits for it only
    // before the second fetch.
    const PlanPtrs pp = plan_carve(p.plan_fwd, kPlanFwd, items, grid, D);
    rc = launch_plan(kPlanFwd, p, items, grid, pp, stream, grid);
    if (rc) return rc;
    a.sched = SchedArgs{pp.header, pp.queue, items, 1};
  }
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FwdLayout<D>::kAlloc);
  if (p.plan_fwd)
    return launch_dependent(kern, dim3(grid), dim3(kFwdThreads), FwdLayout<D>::kAlloc, stream,
                            "fwd_sm100_kernel", a);
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

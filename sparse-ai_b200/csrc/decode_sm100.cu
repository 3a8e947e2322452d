// Routed paged decode, B200 fast path: page selection inside a persistent streaming kernel,
// TMA page streaming, and the score / value products on the tensor cores.
//
// Semantics are those of src/ultrametric/kernel_decode.py:23-124 in sparse-ai (and of the
// general path in decode.cu): request b, query head h attends the logical pages whose
// routing vector (router[phys, h, :r], indexed by the PHYSICAL page id) equals
// q_router[b, h, :r], plus logical page 0 (sink) and the last `local_blocks` pages; tokens
// >= context_lens[b] are masked; a request with no attended token gets zeros.
//
// A "unit" is one (request b, KV head g), bg = b * Hkv + g.  A work item is one unit's part
// of PP consecutive logical pages (PP chosen on the host so that there are a few items per
// SM).  Three kernels, each launched as the programmatic dependent of the one before:
//
//  1. decode_init_kernel (one CTA): zeroes the item queue and lists the (request, part)
//     pairs that hold pages (a scan over the requests' context lengths), so the items are
//     the pairs x KV heads with no empty ones in between.
//  2. decode_stream_kernel, one persistent CTA per SM taking items from an atomic queue.
//     Warp 6 (scheduler) selects each item's pages itself, up to three items ahead of the
//     producer: the item's block-table entries (a lane per page), then the group's routing
//     words of those pages against the query's, giving per page the mask of the group's
//     query heads that attend it; the selected pages are compacted in order into a
//     descriptor {physical page, head mask | valid tokens << 16}.  An item that selects
//     nothing marks its partial empty and costs no streaming.  Warp 0 streams each item's
//     K/V pages with TMA (4-D tensor maps over the paged caches) into a ring of 64-token
//     tiles and the group's G query rows with a bulk copy.  Warps 1-4 each own 16 token rows
//     of every tile: S = Q K^T and O += P V as m16n8k16 MMAs whose 16 rows are the group's
//     query heads (so K and V bytes are read once per KV head), online softmax in registers in
//     the log2 domain.  At an item's end they hand their states to warp 5 through a
//     double-buffered shared area; warp 5 merges them into one partial (m, l, acc[D]) per
//     query head.  The products are < 1 % of the tensor pipe at HBM speed, so the warp-level
//     MMA is enough; what matters is that the ring keeps ~200 KB of loads in flight per SM.
//  3. decode_unit_combine_kernel, one CTA per unit: merges the unit's part partials by
//     log-sum-exp weights and writes its G output rows (zeros when nothing was attended).
#include <algorithm>
#include <string>
#include <type_traits>
#include <utility>

#include "decode.cuh"

namespace sa {
namespace {

constexpr int kTile = 64;           // token rows per ring stage
constexpr int kMaxPP = 64;          // logical pages per work item (at most)
constexpr int kInitThreads = 1024;
constexpr int kMaxHeads = 128;
constexpr int kMaxSelLevels = 16;   // routing levels compared (req_depth)
constexpr int kCw = 4;              // consumer warps (16 token rows each)
constexpr int kSched = 4;           // scheduler warps (items selected concurrently)
constexpr int kStreamThreads = 32 * (2 + kCw + kSched);  // + producer, epilogue, schedulers
constexpr int kSchedWarp = 2 + kCw;  // the first scheduler warp
constexpr int kMaxG = 16;           // MMA rows = query heads of a group
constexpr int kMaxStages = 8;
constexpr int kQBufs = 4;   // query buffers: the producer may run 3 chunks ahead of the consumers
constexpr int kDescs = 2 * kSched;  // item descriptors: two per scheduler warp
constexpr int kFirst = 1, kLast = 2, kEnd = 4;

struct DecHeader {
  int next;   // queue counter of the stream kernel
  int n_rp;   // (request, part) pairs that hold pages
  int pad[62];
};
static_assert(sizeof(DecHeader) == 256, "DecHeader");

// Items: index i -> (request, part) pair rp[i / Hkv], KV head i % Hkv.  Part j of request b
// covers logical pages [j * PP, min(n_logical, (j + 1) * PP)).
struct FastWs {
  DecHeader* hdr;
  int4* rp;     // [B * NP] {request, part, n_logical, context length}, request-major
  float* part;  // [BG][NP][G][D + 4]: m (log2 units; -inf = nothing attended), l, 0, 0, acc[D]
  int NP, PP;
};

struct TileMeta {
  int chunk;
  int flags;
  int vr;               // valid token rows (a prefix of the tile)
  int pad[3];
  uint16_t wmask[kCw];  // head mask of the page holding each consumer warp's 16 rows
};
static_assert(sizeof(TileMeta) == 32, "TileMeta");

// A reserved item with its selected pages, prepared by the scheduler warp.
struct ChunkDesc {
  int chunk;  // partial slot bg * NP + part, or -1 (no more work)
  int bg, n, pad;
  int2 sel[kMaxPP];  // {physical page, head mask | valid tokens << 16}
};

struct StreamArgs {
  CUtensorMap tm_k, tm_v;
  const void* q;
  int64_t qs0, qs1;
  void* out;
  int64_t os0, os1;
  int64_t Hkv, page;
  int G, ppt, stages;
  float scale2;
  FastWs w;
  // selection inputs (DecodeParams subset)
  const int32_t* bt;
  int64_t bts0, bts1;
  const int32_t* ctx;
  const void* router;
  int router_dtype;
  int64_t rs0, rs1, rs2;
  const void* qrouter;
  int qrouter_dtype;
  int64_t qrs0, qrs1, qrs2;
  int64_t maxL, local_blocks;
  int r, sink;
  unsigned* status;
};

inline size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

// Logical pages per work item: 64, halved (down to 8) while the batch would give fewer than
// about four items per SM.
int pages_per_item(int64_t B, int64_t Hkv, int64_t maxL, int sms) {
  int pp = kMaxPP;
  while (pp > 8 && B * Hkv * ((std::max<int64_t>(maxL, 1) + pp - 1) / pp) < 4 * (int64_t)sms) pp /= 2;
  return pp;
}

// Workspace layout; returns its size.  Fills *w when base is given.
size_t carve(void* base, int64_t B, int64_t Hkv, int64_t maxL, int64_t G, int64_t D, int PP, FastWs* w) {
  const int64_t BG = B * Hkv;
  const int NP = (int)((std::max<int64_t>(maxL, 1) + PP - 1) / PP);
  char* c = static_cast<char*>(base);
  size_t o = 0;
  auto take = [&](size_t bytes) {
    char* r = c ? c + o : nullptr;
    o += al256(bytes);
    return r;
  };
  FastWs t;
  t.hdr = reinterpret_cast<DecHeader*>(take(sizeof(DecHeader)));
  t.rp = reinterpret_cast<int4*>(take((size_t)B * NP * 16));
  t.part = reinterpret_cast<float*>(take((size_t)BG * NP * G * (D + 4) * 4));
  t.NP = NP;
  t.PP = PP;
  if (w) *w = t;
  return o;
}

// ---------------------------------------------------------------------------------------
// 1. the item list
// ---------------------------------------------------------------------------------------
// One CTA: the (request, part) pairs holding pages, request-major, by an exclusive scan of
// the parts per request over the batch.
__global__ void __launch_bounds__(kInitThreads) decode_init_kernel(FastWs w, const int32_t* ctx,
                                                                   int64_t B, int64_t page,
                                                                   int64_t maxL) {
  pdl_trigger();
  __shared__ int s_warp[kInitThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int run = 0;
  for (int64_t b0 = 0; b0 < B; b0 += kInitThreads) {
    const int64_t b = b0 + tid;
    int np = 0, nlog = 0, c = 0;
    if (b < B) {
      c = ctx[b];
      nlog = c > 0 ? (int)min((c + page - 1) / page, maxL) : 0;
      np = (nlog + w.PP - 1) / w.PP;
    }
    int x = np;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    int base = 0, tot = 0;
    for (int i = 0; i < kInitThreads / 32; ++i) {
      base += i < warp ? s_warp[i] : 0;
      tot += s_warp[i];
    }
    __syncthreads();
    const int first = run + base + x - np;
    for (int j = 0; j < np; ++j) w.rp[first + j] = make_int4((int)b, j, nlog, c);
    run += tot;
  }
  if (tid == 0) {
    w.hdr->next = 0;
    w.hdr->n_rp = run;
  }
}

// ---------------------------------------------------------------------------------------
// 3. streaming
// ---------------------------------------------------------------------------------------
template <bool BF16>
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  uint32_t r;
  if constexpr (BF16)
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

template <bool BF16>
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  if constexpr (BF16)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Byte offset of (row, d) in a [64 rows][D] tile stored as D/64 chunks of 128-byte rows
// with the TMA 128-byte swizzle (16-byte unit index XOR row % 8).
__device__ __forceinline__ uint32_t swz(int row, int d) {
  return (uint32_t)((d >> 6) * (kTile * 128) + row * 128 + ((((d & 63) >> 3) ^ (row & 7)) << 4));
}

// Which of the group's heads disagree with the query on two pages: bit (i / r) of miss0 /
// miss1 is set when routing word i (head i / r, level i % r) of the page differs from the
// query's.  The loads are issued 16 + 16 at a time with no branch between them (the element
// type is a template parameter, not a run-time switch), so one memory latency covers them.
template <typename RT>
__device__ __forceinline__ void route_misses(const RT* __restrict__ router, int64_t base0, int64_t base1,
                                             bool in0, bool in1, int GR, int r, int64_t rs1,
                                             int64_t rs2, const int32_t* s_qr, unsigned& miss0,
                                             unsigned& miss1) {
  for (int i0 = 0; i0 < GR; i0 += 16) {
    RT v0[16], v1[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int i = min(i0 + u, GR - 1);  // in range; the word is ignored when i0 + u >= GR
      const int64_t off = (i / r) * rs1 + (i % r) * rs2;
      v0[u] = __ldg(router + (in0 ? base0 + off : 0));
      v1[u] = __ldg(router + (in1 ? base1 + off : 0));
    }
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int i = i0 + u;
      if (i < GR) {
        const int64_t q = s_qr[i];
        if ((int64_t)v0[u] != q) miss0 |= 1u << (i / r);
        if ((int64_t)v1[u] != q) miss1 |= 1u << (i / r);
      }
    }
  }
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kStreamThreads, 1)
    decode_stream_kernel(const __grid_constant__ StreamArgs a) {
  pdl_trigger();  // the unit merge may launch now; it waits for this grid to complete
  constexpr int KC = D / 64;
  constexpr uint32_t kHalf = kTile * D * 2;  // K (or V) bytes of one stage
  constexpr uint32_t kStage = 2 * kHalf;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int stages = a.stages, G = a.G;
  constexpr int RS = D + 4;  // state / partial row: m, l, 0, 0, acc[D]
  const uint32_t kQBuf = (uint32_t)G * D * 2;  // one chunk's G query rows (a multiple of 128 B)
  unsigned char* ring = sm;
  unsigned char* qbuf = sm + stages * kStage;  // kQBufs x [G][D]
  float* mbuf = reinterpret_cast<float*>(qbuf + kQBufs * kQBuf);  // 2 x [kCw][G][RS]
  TileMeta* meta = reinterpret_cast<TileMeta*>(mbuf + 2 * kCw * G * RS);
  uint64_t* full = reinterpret_cast<uint64_t*>(meta + stages);
  uint64_t* empty = full + stages;
  uint64_t* qfull = empty + stages;
  uint64_t* qempty = qfull + kQBufs;
  uint64_t* mfull = qempty + kQBufs;
  uint64_t* mempty = mfull + 2;
  int* einfo = reinterpret_cast<int*>(mempty + 2);   // [2] chunk handed to the epilogue warp
  ChunkDesc* desc = reinterpret_cast<ChunkDesc*>(einfo + 4);  // [kDescs] scheduler -> producer
  uint64_t* dfull = reinterpret_cast<uint64_t*>(desc + kDescs);
  uint64_t* dempty = dfull + kDescs;
  // per scheduler warp: the item's query routing words [G][r]
  int32_t* s_qr_all = reinterpret_cast<int32_t*>(dempty + kDescs);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCw);
    }
    for (int i = 0; i < kQBufs; ++i) {
      mbar_init(&qfull[i], 1);
      mbar_init(&qempty[i], kCw);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&mfull[i], kCw);
      mbar_init(&mempty[i], 1);
    }
    for (int i = 0; i < kDescs; ++i) {
      mbar_init(&dfull[i], 1);
      mbar_init(&dempty[i], 1);
    }
    fence_mbar_init();
    prefetch_tmap(&a.tm_k);
    prefetch_tmap(&a.tm_v);
  }
  __syncthreads();
  pdl_wait();  // the init kernel's item list and queue header are complete from here on

  if (warp == 0) {
    // ---------------- producer ----------------
    uint32_t tile = 0, qi = 0;
    bool ok = true;
    // descriptor d comes from scheduler d % kSched; each scheduler ends with one end marker,
    // after which its slots are skipped
    unsigned ended = 0;
    for (uint32_t d = 0; ok && ended != (1u << kSched) - 1u; ++d) {
      const uint32_t ds = d % kDescs;
      if (ended & (1u << (d % kSched))) continue;
      if (!(ok = mbar_wait_warp(&dfull[ds], (d / kDescs) & 1, a.status))) break;
      const ChunkDesc& cd = desc[ds];
      const int c = cd.chunk;
      if (c < 0) {
        ended |= 1u << (d % kSched);
        continue;
      }
      const int bg = cd.bg, nsel = cd.n;
      const int64_t b = bg / a.Hkv, g = bg % a.Hkv;
      if (lane == 0) {
        const uint32_t qb = qi % kQBufs;
        ok = mbar_wait(&qempty[qb], ((qi / kQBufs) & 1) ^ 1, a.status);
        if (ok) {
          mbar_arrive_expect_tx(&qfull[qb], (uint32_t)(G * D * 2));
          const char* src = static_cast<const char*>(a.q) + (b * a.qs0 + g * G * a.qs1) * 2;
          for (int hh = 0; hh < G; ++hh)
            bulk_load(qbuf + qb * kQBuf + hh * D * 2, src + hh * a.qs1 * 2, D * 2, &qfull[qb]);
        }
        const int2* bsel = cd.sel;
        if (a.page >= kTile) {
          // a page is page/64 tiles; tiles past the context end are skipped
          for (int k = 0; k < nsel && ok; ++k) {
            const int2 e = bsel[k];
            const int valid = (int)((unsigned)e.y >> 16);
            const uint16_t mk = (uint16_t)(e.y & 0xffff);
            for (int t0 = 0; t0 < valid; t0 += kTile, ++tile) {
              const uint32_t st = tile % stages;
              if (!(ok = mbar_wait(&empty[st], ((tile / stages) & 1) ^ 1, a.status))) break;
              TileMeta& m = meta[st];
              const bool last = k == nsel - 1 && t0 + kTile >= valid;
              m.chunk = c;
              m.flags = (k == 0 && t0 == 0 ? kFirst : 0) | (last ? kLast : 0);
              m.vr = min(kTile, valid - t0);
#pragma unroll
              for (int q = 0; q < kCw; ++q) m.wmask[q] = mk;
              mbar_arrive_expect_tx(&full[st], kStage);
              unsigned char* sk = ring + st * kStage;
#pragma unroll
              for (int ch = 0; ch < KC; ++ch) {
                tma_load_4d(sk + ch * (kTile * 128), &a.tm_k, &full[st], ch * 64, t0, (int)g, e.x);
                tma_load_4d(sk + kHalf + ch * (kTile * 128), &a.tm_v, &full[st], ch * 64, t0,
                            (int)g, e.x);
              }
            }
          }
        } else {
          // ppt = 64/page selected pages per tile
          const int ppt = a.ppt, page = (int)a.page;
          for (int k = 0; k < nsel && ok; k += ppt, ++tile) {
            const int n = min(ppt, nsel - k);
            const uint32_t st = tile % stages;
            if (!(ok = mbar_wait(&empty[st], ((tile / stages) & 1) ^ 1, a.status))) break;
            TileMeta& m = meta[st];
            m.chunk = c;
            m.flags = (k == 0 ? kFirst : 0) | (k + n == nsel ? kLast : 0);
            m.vr = (n - 1) * page + (int)((unsigned)bsel[k + n - 1].y >> 16);
#pragma unroll
            for (int q = 0; q < kCw; ++q) {
              const int j = q * 16 / page;
              m.wmask[q] = j < n ? (uint16_t)(bsel[k + j].y & 0xffff) : (uint16_t)0;
            }
            mbar_arrive_expect_tx(&full[st], (uint32_t)(n * page * D * 2 * 2));
            unsigned char* sk = ring + st * kStage;
            for (int j = 0; j < n; ++j) {
              const int phys = bsel[k + j].x;
#pragma unroll
              for (int ch = 0; ch < KC; ++ch) {
                tma_load_4d(sk + ch * (kTile * 128) + j * page * 128, &a.tm_k, &full[st], ch * 64, 0,
                            (int)g, phys);
                tma_load_4d(sk + kHalf + ch * (kTile * 128) + j * page * 128, &a.tm_v, &full[st],
                            ch * 64, 0, (int)g, phys);
              }
            }
          }
        }
      }
      ++qi;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[ds]);  // the descriptor's entries are no longer read
    }
    // tell the consumers that the queue is drained
    if (lane == 0 && ok) {
      const uint32_t st = tile % stages;
      if (mbar_wait(&empty[st], ((tile / stages) & 1) ^ 1, a.status)) {
        meta[st].flags = kEnd;
        mbar_arrive(&full[st]);
      }
    }
  } else if (warp <= kCw) {
    // ---------------- consumers: 16 token rows each ----------------
    const int cw = warp - 1;
    const int gq = lane >> 2, cq = lane & 3;
    const uint32_t ring_u = smem_u32(ring);
    uint32_t tile = 0, qi = 0, ei = 0;
    uint32_t qa[D / 16][4];
    float o[D / 8][4];
    float mr[2] = {-INFINITY, -INFINITY}, lr[2] = {0.f, 0.f};
    for (;;) {
      const uint32_t st = tile % stages;
      if (!mbar_wait_warp(&full[st], (tile / stages) & 1, a.status)) break;
      ++tile;
      const int flags = meta[st].flags;
      if (flags & kEnd) {
        // pass the end on to the epilogue warp
        const uint32_t eb = ei & 1;
        if (!mbar_wait_warp(&mempty[eb], ((ei >> 1) & 1) ^ 1, a.status)) break;
        if (cw == 0 && lane == 0) einfo[eb] = -1;
        __syncwarp();
        if (lane == 0) mbar_arrive(&mfull[eb]);
        break;
      }
      if (flags & kFirst) {
        const uint32_t qb = qi % kQBufs;
        if (!mbar_wait_warp(&qfull[qb], (qi / kQBufs) & 1, a.status)) break;
        // MMA rows >= G (no query head) are zero
        const bool v0 = gq < G, v1 = gq + 8 < G;
        const uint32_t* r0 = reinterpret_cast<const uint32_t*>(qbuf + qb * kQBuf + (v0 ? gq : 0) * D * 2);
        const uint32_t* r1 =
            reinterpret_cast<const uint32_t*>(qbuf + qb * kQBuf + (v1 ? gq + 8 : 0) * D * 2);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          qa[ks][0] = v0 ? r0[ks * 8 + cq] : 0u;
          qa[ks][1] = v1 ? r1[ks * 8 + cq] : 0u;
          qa[ks][2] = v0 ? r0[ks * 8 + 4 + cq] : 0u;
          qa[ks][3] = v1 ? r1[ks * 8 + 4 + cq] : 0u;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&qempty[qb]);
        ++qi;
#pragma unroll
        for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
        mr[0] = mr[1] = -INFINITY;
        lr[0] = lr[1] = 0.f;
      }
      const int vw = min(16, max(0, meta[st].vr - 16 * cw));
      const unsigned hm = meta[st].wmask[cw];
      const int chunk = meta[st].chunk;
      bool zeroed = false;
      if (vw > 0) {
        const uint32_t sk = ring_u + st * kStage, sv = sk + kHalf;
        if (vw < 16) {
          // rows past the context end (or of a page the tile does not hold): V := 0 so
          // that P = 0 there cannot meet a non-finite value
          unsigned char* vb = ring + st * kStage + kHalf;
          const int nz = (16 - vw) * KC * 8;
          for (int i = lane; i < nz; i += 32) {
            const int rr = 16 * cw + vw + i / (KC * 8), ch = (i / 8) % KC, u = i % 8;
            *reinterpret_cast<uint4*>(vb + ch * (kTile * 128) + rr * 128 + u * 16) =
                make_uint4(0, 0, 0, 0);
          }
          zeroed = true;
          __syncwarp();
        }
        float s[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
        for (int kc = 0; kc < D / 32; ++kc) {
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            uint32_t bfr[4];
            ldsm_x4(sk + swz(16 * cw + nt * 8 + (lane & 7), kc * 32 + (lane >> 3) * 8), bfr);
            mma16816<BF16>(s[nt], qa[2 * kc], bfr[0], bfr[1]);
            mma16816<BF16>(s[nt], qa[2 * kc + 1], bfr[2], bfr[3]);
          }
        }
        const bool h0 = (hm >> gq) & 1u, h1 = (hm >> (gq + 8)) & 1u;
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const bool v = nt * 8 + 2 * cq + e < vw;
            s[nt][e] = v && h0 ? s[nt][e] * a.scale2 : -INFINITY;
            s[nt][2 + e] = v && h1 ? s[nt][2 + e] * a.scale2 : -INFINITY;
            mx0 = fmaxf(mx0, s[nt][e]);
            mx1 = fmaxf(mx1, s[nt][2 + e]);
          }
#pragma unroll
        for (int o2 = 1; o2 <= 2; o2 <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o2));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o2));
        }
        const float mn0 = fmaxf(mr[0], mx0), mn1 = fmaxf(mr[1], mx1);
        const float ref0 = mn0 == -INFINITY ? 0.f : mn0, ref1 = mn1 == -INFINITY ? 0.f : mn1;
        const float al0 = fast_exp2(mr[0] - ref0), al1 = fast_exp2(mr[1] - ref1);
        mr[0] = mn0;
        mr[1] = mn1;
        float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            s[nt][e] = fast_exp2(s[nt][e] - ref0);
            s[nt][2 + e] = fast_exp2(s[nt][2 + e] - ref1);
            ps0 += s[nt][e];
            ps1 += s[nt][2 + e];
          }
        lr[0] = lr[0] * al0 + ps0;
        lr[1] = lr[1] * al1 + ps1;
        if (__any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {
#pragma unroll
          for (int n = 0; n < D / 8; ++n) {
            o[n][0] *= al0;
            o[n][1] *= al0;
            o[n][2] *= al1;
            o[n][3] *= al1;
          }
        }
        uint32_t pa[4];
        pa[0] = pack_half2<BF16>(s[0][0], s[0][1]);
        pa[1] = pack_half2<BF16>(s[0][2], s[0][3]);
        pa[2] = pack_half2<BF16>(s[1][0], s[1][1]);
        pa[3] = pack_half2<BF16>(s[1][2], s[1][3]);
#pragma unroll
        for (int dp = 0; dp < D / 16; ++dp) {
          uint32_t bfr[4];
          ldsm_x4_t(sv + swz(16 * cw + (lane & 7) + ((lane >> 3) & 1) * 8, dp * 16 + (lane >> 4) * 8),
                    bfr);
          mma16816<BF16>(o[2 * dp], pa, bfr[0], bfr[1]);
          mma16816<BF16>(o[2 * dp + 1], pa, bfr[2], bfr[3]);
        }
      }
      if (zeroed) fence_proxy_async_smem();  // our stores, then the next TMA into the stage
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      if (!(flags & kLast)) continue;

      // ---- end of a chunk: hand this warp's state to the epilogue warp
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        lr[i] += __shfl_xor_sync(0xffffffffu, lr[i], 1);
        lr[i] += __shfl_xor_sync(0xffffffffu, lr[i], 2);
      }
      const uint32_t eb = ei & 1;
      if (!mbar_wait_warp(&mempty[eb], ((ei >> 1) & 1) ^ 1, a.status)) break;
      ++ei;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int hh = gq + 8 * half;
        if (hh < G) {
          float* row = mbuf + ((eb * kCw + cw) * G + hh) * RS;
          if (cq == 0) *reinterpret_cast<float4*>(row) = make_float4(mr[half], lr[half], 0.f, 0.f);
#pragma unroll
          for (int n = 0; n < D / 8; ++n)
            *reinterpret_cast<float2*>(row + 4 + n * 8 + 2 * cq) =
                make_float2(o[n][2 * half], o[n][2 * half + 1]);
        }
      }
      if (cw == 0 && lane == 0) einfo[eb] = chunk;
      __syncwarp();
      if (lane == 0) mbar_arrive(&mfull[eb]);
    }
  } else if (warp >= kSchedWarp) {
    // ---------------- schedulers: take items and select their pages ----------------
    // kSched warps work on different items at once; scheduler w fills descriptors
    // w, w + kSched, ... (each up to two items ahead of the producer).  The first items
    // are static (w * gridDim.x + CTA); the queue counter hands out the rest.  Per item:
    // its {request, part, n_logical, context} entry, then together the query's routing words
    // of the group's heads and the block-table entries of the part's pages (a lane per page,
    // two rounds of 32), then each page's routing words of the group's heads; the pages that
    // some head attends are compacted in logical order into the descriptor.
    const int sw = warp - kSchedWarp;
    int32_t* s_qr = s_qr_all + sw * kMaxG * kMaxSelLevels;
    const int n_rp = __ldcg(&a.w.hdr->n_rp);
    const int64_t n_items = (int64_t)n_rp * a.Hkv;
    const int PP = a.w.PP, NP = a.w.NP, r = a.r, GR = G * r;
    constexpr int RSP = D + 4;
    bool first = true;
    for (uint32_t k = 0;; ++k) {
      const uint32_t d = sw + k * kSched, ds = d % kDescs;
      if (!mbar_wait_warp(&dempty[ds], ((d / kDescs) & 1) ^ 1, a.status)) break;
      ChunkDesc& cd = desc[ds];
      int slot = -1, bg = 0, nsel = 0;
      for (;;) {
        int64_t idx = 0;
        if (lane == 0)
          idx = first ? (int64_t)sw * gridDim.x + blockIdx.x
                      : (int64_t)kSched * gridDim.x + atomicAdd(&a.w.hdr->next, 1);
        first = false;
        idx = __shfl_sync(0xffffffffu, idx, 0);
        if (idx >= n_items) break;
        const int4 rp = __ldcg(a.w.rp + idx / a.Hkv);
        const int64_t b = rp.x, g = idx % a.Hkv, nlog = rp.z, cx = rp.w;
        const int part = rp.y;
        bg = (int)(b * a.Hkv + g);
        const int64_t lo = (int64_t)part * PP, hi = min(nlog, lo + PP);
        // query routing words and block-table entries, loads in flight together
        int32_t qv[kMaxG * kMaxSelLevels / 32];
        if (a.qrouter_dtype == SA_I64) {
#pragma unroll
          for (int j = 0; j < kMaxG * kMaxSelLevels / 32; ++j) {
            const int i = min(lane + 32 * j, GR - 1);
            qv[j] = GR > 0 ? (int32_t)__ldg(static_cast<const int64_t*>(a.qrouter) + b * a.qrs0 +
                                            (g * G + i / r) * a.qrs1 + (i % r) * a.qrs2)
                           : 0;
          }
        } else {
#pragma unroll
          for (int j = 0; j < kMaxG * kMaxSelLevels / 32; ++j) {
            const int i = min(lane + 32 * j, GR - 1);
            qv[j] = GR > 0 ? __ldg(static_cast<const int32_t*>(a.qrouter) + b * a.qrs0 +
                                   (g * G + i / r) * a.qrs1 + (i % r) * a.qrs2)
                           : 0;
          }
        }
        const int64_t pg0 = lo + lane, pg1 = lo + 32 + lane;
        const bool in0 = pg0 < hi, in1 = pg1 < hi;
        const int ph0 = in0 ? a.bt[b * a.bts0 + pg0 * a.bts1] : 0;
        const int ph1 = in1 ? a.bt[b * a.bts0 + pg1 * a.bts1] : 0;
#pragma unroll
        for (int j = 0; j < kMaxG * kMaxSelLevels / 32; ++j)
          if (lane + 32 * j < GR) s_qr[lane + 32 * j] = qv[j];
        __syncwarp();
        // both pages' routing words of the group's heads, 16 + 16 loads in flight at a time
        const int64_t base0 = (int64_t)ph0 * a.rs0 + g * G * a.rs1;
        const int64_t base1 = (int64_t)ph1 * a.rs0 + g * G * a.rs1;
        unsigned miss0 = 0, miss1 = 0;
        if (a.router_dtype == SA_I64)
          route_misses(static_cast<const int64_t*>(a.router), base0, base1, in0, in1, GR, r, a.rs1,
                       a.rs2, s_qr, miss0, miss1);
        else
          route_misses(static_cast<const int32_t*>(a.router), base0, base1, in0, in1, GR, r, a.rs1,
                       a.rs2, s_qr, miss0, miss1);
        const unsigned all = (1u << G) - 1u;
        nsel = 0;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int64_t pg = half ? pg1 : pg0;
          const bool in = half ? in1 : in0;
          const bool forced = (a.sink && pg == 0) || (a.local_blocks > 0 && pg >= nlog - a.local_blocks);
          const unsigned mask = !in ? 0u : forced ? all : (~(half ? miss1 : miss0) & all);
          const unsigned bal = __ballot_sync(0xffffffffu, mask != 0u);
          if (mask) {
            const int valid = (int)min(a.page, cx - pg * a.page);
            cd.sel[nsel + __popc(bal & ((1u << lane) - 1u))] =
                make_int2(half ? ph1 : ph0, (int)(mask | ((unsigned)valid << 16)));
          }
          nsel += __popc(bal);
        }
        __syncwarp();  // s_qr is rewritten for the next item
        slot = bg * NP + part;
        if (nsel > 0) break;
        // nothing attended in this part: its partial is marked empty, no streaming
        if (lane < G) a.w.part[((int64_t)slot * G + lane) * RSP] = -INFINITY;
        slot = -1;
      }
      if (lane == 0) {
        cd.chunk = slot;
        cd.bg = bg;
        cd.n = nsel;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&dfull[ds]);
      if (slot < 0) break;
    }
  } else {
    // ---------------- epilogue warp: chunk partials ----------------
    for (uint32_t ei = 0;; ++ei) {
      const uint32_t eb = ei & 1;
      if (!mbar_wait_warp(&mfull[eb], (ei >> 1) & 1, a.status)) break;
      const int chunk = einfo[eb];
      if (chunk < 0) break;
      // merge the four consumer warps' states (float4 columns; column 0 = {m, l, 0, 0})
      const float* mb = mbuf + eb * kCw * G * RS;
      float4* dst = reinterpret_cast<float4*>(a.w.part + (int64_t)chunk * G * RS);
      for (int i = lane; i < G * (RS / 4); i += 32) {
        const int hh = i / (RS / 4), c4 = i % (RS / 4);
        float mq[kCw], M = -INFINITY;
#pragma unroll
        for (int q = 0; q < kCw; ++q) {
          mq[q] = mb[(q * G + hh) * RS];
          M = fmaxf(M, mq[q]);
        }
        const float Mr = M == -INFINITY ? 0.f : M;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int q = 0; q < kCw; ++q) {
          const float wq = fast_exp2(mq[q] - Mr);
          const float4 x = *reinterpret_cast<const float4*>(mb + (q * G + hh) * RS + 4 * c4);
          v.x += x.x * wq;
          v.y += x.y * wq;
          v.z += x.z * wq;
          v.w += x.w * wq;
        }
        if (c4 == 0) v = make_float4(M, v.y, 0.f, 0.f);
        dst[i] = v;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&mempty[eb]);  // the shared states are consumed
    }
  }
}

// ---------------------------------------------------------------------------------------
// 3. per-unit merge of the part partials (a programmatic dependent of the stream kernel)
// ---------------------------------------------------------------------------------------
// One CTA per unit, one thread per float4 output column of the unit's G heads; the unit's
// parts (those holding pages: ceil(n_logical / PP)) are merged online with eight parts'
// loads in flight.  Parts (or heads) that attended nothing have m = -inf and are skipped
// (their other fields are not written); a unit with nothing attended gets zeros.
template <typename T, int D>
__global__ void __launch_bounds__(kMaxG * D / 4) decode_unit_combine_kernel(const FastWs w,
                                                                          const int32_t* ctx,
                                                                          int64_t page, int64_t maxL,
                                                                          void* out_, int64_t os0,
                                                                          int64_t os1, int64_t Hkv,
                                                                          int G) {
  constexpr int RS = D + 4;
  pdl_wait();
  const int64_t bg = blockIdx.x;
  const int i = threadIdx.x;
  if (i >= G * (D / 4)) return;
  const int64_t cx = ctx[bg / Hkv];
  const int64_t nlog = cx > 0 ? min((cx + page - 1) / page, maxL) : 0;
  const int nparts = (int)((nlog + w.PP - 1) / w.PP);
  const int hh = i / (D / 4), d4 = i % (D / 4);
  const float* ph = w.part + (int64_t)bg * w.NP * G * RS + hh * RS;
  const int64_t CS = (int64_t)G * RS;
  float M = -INFINITY, L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  constexpr int NU = 8;
  for (int k0 = 0; k0 < nparts; k0 += NU) {
    float2 ml[NU];
    float4 x[NU];
#pragma unroll
    for (int u = 0; u < NU; ++u) {
      const int k = min(k0 + u, nparts - 1);
      ml[u] = __ldcg(reinterpret_cast<const float2*>(ph + k * CS));
      x[u] = __ldcg(reinterpret_cast<const float4*>(ph + k * CS + 4 + 4 * d4));
    }
#pragma unroll
    for (int u = 0; u < NU; ++u) {
      if (k0 + u >= nparts) break;
      if (ml[u].x == -INFINITY) continue;  // nothing attended by this head in this part
      const float mn = fmaxf(M, ml[u].x);
      const float so = fast_exp2(M - mn), sn = fast_exp2(ml[u].x - mn);
      acc.x = acc.x * so + x[u].x * sn;
      acc.y = acc.y * so + x[u].y * sn;
      acc.z = acc.z * so + x[u].z * sn;
      acc.w = acc.w * so + x[u].w * sn;
      L = L * so + ml[u].y * sn;
      M = mn;
    }
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  const int64_t b = bg / Hkv, g = bg % Hkv;
  T* o4 = static_cast<T*>(out_) + b * os0 + (g * G + hh) * os1 + 4 * d4;
  o4[0] = from_f32<T>(acc.x * inv);
  o4[1] = from_f32<T>(acc.y * inv);
  o4[2] = from_f32<T>(acc.z * inv);
  o4[3] = from_f32<T>(acc.w * inv);
}

template <int D, bool BF16>
int launch_stream(StreamArgs& a, int grid, cudaStream_t stream) {
  constexpr size_t kStage = 2 * (size_t)kTile * D * 2;
  // alignment slack, query buffers, 2 merge buffers, then Q / merge barriers, hand-off
  // records, the producer's page batch and the scheduler's descriptors with barriers
  static_assert((2 * kQBufs + 4) * 8 + 16 + kDescs * (sizeof(ChunkDesc) + 16) +
                    kSched * kMaxG * kMaxSelLevels * 4 <= 9216,
                "decode: barrier, descriptor and query-route area");
  const size_t fixed = 1024 + kQBufs * (size_t)a.G * D * 2 + 2 * (size_t)kCw * a.G * (D + 4) * 4 + 9216;
  const size_t per_stage = kStage + sizeof(TileMeta) + 16;
  const int stages = (int)std::min<size_t>(kMaxStages, (226 * 1024 - fixed) / per_stage);
  if (stages < 2) return fail(SA_EUNSUPPORTED, "decode: shared memory too small for the ring");
  a.stages = stages;
  const size_t smem = fixed + (size_t)stages * per_stage;
  auto kern = decode_stream_kernel<D, BF16>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  return launch_dependent(kern, dim3(grid), dim3(kStreamThreads), smem, stream, "decode_stream_kernel", a);
}

}  // namespace

bool decode_fast_eligible(const DecodeParams& p, int dtype) {
  if (dtype != SA_BF16 && dtype != SA_F16) return false;
  if (p.D != 64 && p.D != 128) return false;
  if (p.G < 1 || p.G > kMaxG || p.H > kMaxHeads || p.r > kMaxSelLevels) return false;
  if (!(p.page == 16 || p.page == 32 || (p.page % kTile == 0 && p.page < 65536))) return false;
  if (p.num_pages < 1 || p.num_pages > INT32_MAX || p.Hkv > INT32_MAX || p.maxL > 65535) return false;
  if (p.qs[2] != 1 || reinterpret_cast<uintptr_t>(p.q) % 16 || (p.qs[0] * 2) % 16 ||
      (p.qs[1] * 2) % 16)
    return false;
  return true;
}

int64_t decode_fast_workspace_bytes(int64_t B, int64_t H, int64_t Hkv, int64_t D, int64_t maxL) {
  if (B <= 0 || H <= 0 || Hkv <= 0 || D <= 0) return 0;
  return (int64_t)carve(nullptr, B, Hkv, maxL, H / Hkv, D,
                        pages_per_item(B, Hkv, maxL, device_sm_count()), nullptr);
}

int launch_decode_fast(const DecodeParams& p, int dtype, void* workspace, int64_t workspace_bytes,
                       cudaStream_t stream) {
  const int64_t BG = p.B * p.Hkv;
  const int sms = device_sm_count();
  FastWs w;
  const size_t need = carve(workspace, p.B, p.Hkv, p.maxL, p.G, p.D,
                            pages_per_item(p.B, p.Hkv, p.maxL, sms), &w);
  if ((int64_t)need > workspace_bytes || !workspace)
    return fail(SA_EWORKSPACE, "decode: workspace too small (" + std::to_string(workspace_bytes) +
                                   " < " + std::to_string(need) + ")");
  if (p.B > 65535) return fail(SA_EUNSUPPORTED, "decode: more than 65535 requests");
  if (BG * w.NP > INT32_MAX) return fail(SA_EUNSUPPORTED, "decode: too many work items");
  StreamArgs a{};
  a.status = device_status_ptr();
  if (!a.status) return fail(SA_ELAUNCH, std::string("decode: ") + sa_last_error());
  const uint32_t box_n = (uint32_t)std::min<int64_t>(p.page, kTile);
  int rc = make_tmap_4d(&a.tm_k, p.kc, dtype, p.num_pages, p.Hkv, p.page, p.D, p.ks, 64, box_n);
  if (!rc) rc = make_tmap_4d(&a.tm_v, p.vc, dtype, p.num_pages, p.Hkv, p.page, p.D, p.vs, 64, box_n);
  if (rc) return fail(SA_ELAUNCH, std::string("decode: tensor map: ") + sa_last_error());

  decode_init_kernel<<<1, kInitThreads, 0, stream>>>(w, p.ctx, p.B, p.page, p.maxL);
  rc = check_launch("decode_init_kernel");
  if (rc) return rc;

  a.q = p.q;
  a.qs0 = p.qs[0];
  a.qs1 = p.qs[1];
  a.out = p.out;
  a.os0 = p.os[0];
  a.os1 = p.os[1];
  a.Hkv = p.Hkv;
  a.page = p.page;
  a.G = (int)p.G;
  a.ppt = p.page >= kTile ? 1 : (int)(kTile / p.page);
  a.scale2 = (1.0f / sqrtf((float)p.D)) * kLog2e;
  a.w = w;
  a.bt = p.bt;
  a.bts0 = p.bts[0];
  a.bts1 = p.bts[1];
  a.ctx = p.ctx;
  a.router = p.router;
  a.router_dtype = p.router_dtype;
  a.rs0 = p.rs[0];
  a.rs1 = p.rs[1];
  a.rs2 = p.rs[2];
  a.qrouter = p.qrouter;
  a.qrouter_dtype = p.qrouter_dtype;
  a.qrs0 = p.qrs[0];
  a.qrs1 = p.qrs[1];
  a.qrs2 = p.qrs[2];
  a.maxL = p.maxL;
  a.local_blocks = p.local_blocks;
  a.r = (int)p.r;
  a.sink = p.sink;
  const int grid = (int)std::min<int64_t>(sms, BG * w.NP);
  const bool bf = dtype == SA_BF16;
  if (p.D == 64)
    rc = bf ? launch_stream<64, true>(a, grid, stream) : launch_stream<64, false>(a, grid, stream);
  else
    rc = bf ? launch_stream<128, true>(a, grid, stream) : launch_stream<128, false>(a, grid, stream);
  if (rc) return rc;
  const dim3 cg((unsigned)BG), cb((unsigned)(p.G * p.D / 4));
  const char* cn = "decode_unit_combine_kernel";
  if (p.D == 64)
    return bf ? launch_dependent(decode_unit_combine_kernel<__nv_bfloat16, 64>, cg, cb, 0, stream, cn, w,
                                 p.ctx, p.page, p.maxL, p.out, p.os[0], p.os[1], p.Hkv, (int)p.G)
              : launch_dependent(decode_unit_combine_kernel<__half, 64>, cg, cb, 0, stream, cn, w, p.ctx,
                                 p.page, p.maxL, p.out, p.os[0], p.os[1], p.Hkv, (int)p.G);
  return bf ? launch_dependent(decode_unit_combine_kernel<__nv_bfloat16, 128>, cg, cb, 0, stream, cn, w,
                               p.ctx, p.page, p.maxL, p.out, p.os[0], p.os[1], p.Hkv, (int)p.G)
            : launch_dependent(decode_unit_combine_kernel<__half, 128>, cg, cb, 0, stream, cn, w, p.ctx,
                               p.page, p.maxL, p.out, p.os[0], p.os[1], p.Hkv, (int)p.G);
}

}  // namespace sa

// Routed paged decode, B200 fast path: balanced page chunks on a dynamic queue, TMA page
// streaming, and the score / value products on the tensor cores.
//
// Semantics are those of src/ultrametric/kernel_decode.py:23-124 in sparse-ai (and of the
// general path in decode.cu): request b, query head h attends the logical pages whose
// routing vector (router[phys, h, :r], indexed by the PHYSICAL page id) equals
// q_router[b, h, :r], plus logical page 0 (sink) and the last `local_blocks` pages; tokens
// >= context_lens[b] are masked; a request with no attended token gets zeros.
//
// A "unit" is one (request b, KV head g), bg = b * Hkv + g.  Four kernels, the last three
// launched as programmatic dependents of the one before (their prologues overlap it):
//
//  1. decode_init_kernel: zeroes the work header (selection count, queue counter).
//  2. decode_select_kernel, one CTA per (request, part of its logical pages): one pass over
//     the part's pages (a warp per 8 pages; each page's [H][TD] routing block read as
//     coalesced 128-byte runs) writes, per KV head, the ascending list of the part's pages
//     selected by ANY query head of the group as {physical page, head mask | valid tokens
//     << 16}.  The last CTA to finish (one 64-bit atomic) cuts every list into chunks of `chp`
//     pages, chp chosen so that the batch has about kChunkTarget chunks whatever the spread
//     of context lengths, writes the chunk table, and zeroes the output rows of units that
//     attend no page.
//  3. decode_stream_kernel, one persistent CTA per SM taking chunks from an atomic queue.
//     Warp 6 reserves the next chunk and fetches its table entry and first page entries
//     one chunk ahead of warp 0, which streams each chunk's K/V pages with TMA (4-D tensor
//     maps over the paged caches) into a ring of 64-token tiles and the chunk's G query rows
//     with a bulk copy.  Warps 1-4 each own 16 token rows of every tile: S = Q K^T and
//     O += P V as m16n8k16 MMAs whose 16 rows are the group's query heads (so K and V bytes
//     are read once per KV head), online softmax in registers in the log2 domain.  At a
//     chunk's end they hand their states to warp 5 through a double-buffered shared area
//     and go on; warp 5 merges them into one partial (m, l, acc[D]) per query head.  The
//     products are < 1 % of the tensor pipe at HBM speed, so the warp-level MMA is enough;
//     what matters is that the ring keeps ~200 KB of loads in flight per SM.
//  4. decode_unit_combine_kernel, one CTA per unit: merges the unit's chunk partials by
//     log-sum-exp weights (spread over kMaxG / G thread groups, then folded through shared
//     memory) and writes its G output rows.
#include <algorithm>
#include <string>
#include <type_traits>
#include <utility>

#include "decode.cuh"

namespace sa {
namespace {

constexpr int kTile = 64;           // token rows per ring stage
constexpr int kChunkTarget = 2048;  // chunks per batch; bounds the partials workspace
constexpr int kMaxUnitChunks = 32;  // chunks per unit; bounds the final merge
constexpr int kSelThreads = 256;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kSelTile = kSelThreads;  // pages per pass of the selection kernel
constexpr int kSelSplitCtas = 296;     // selection CTAs at most: 2 resident per SM, one wave
constexpr int kMaxParts = 16;          // parts per request
constexpr int kMaxHeadWords = 4;       // query heads <= 128
constexpr int kMaxHeads = kMaxHeadWords * 32;
constexpr int kMaxSelLevels = 16;      // routing levels compared (req_depth)
constexpr int kCw = 4;              // consumer warps (16 token rows each)
constexpr int kStreamThreads = 32 * (3 + kCw);  // + producer, epilogue and scheduler warps
constexpr int kSchedWarp = 2 + kCw;
constexpr int kMaxG = 16;           // MMA rows = query heads of a group
constexpr int kMaxStages = 8;
constexpr int kQBufs = 4;   // query buffers: the producer may run 3 chunks ahead of the consumers
constexpr int kDescs = 4;   // chunk descriptors: the scheduler reserves up to 3 chunks ahead
constexpr int kFirst = 1, kLast = 2, kEnd = 4;
constexpr int kTickShift = 40;  // DecHeader::total: CTA count above, pair count below

struct DecHeader {
  unsigned spare;
  int n_chunks;
  int chp;          // pages per chunk
  int next;         // queue counter of the stream kernel
  unsigned long long total;  // select CTAs finished << kTickShift | selected (unit, page) pairs
  int pad[58];
};
static_assert(sizeof(DecHeader) == 256, "DecHeader");

// A request's logical pages are selected in P parts of `seg` pages (one CTA each); part q of
// unit bg writes its list at sel[bg][q * seg ...] and its length at count[bg][q].
struct FastWs {
  DecHeader* hdr;
  int* count;   // [BG][P] selected pages of each unit's parts
  int2* uinfo;  // [BG] {first chunk, chunks} of each unit
  int4* table;  // [max chunks] {unit, first | end list index << 16, unit's first chunk, chunks}
  int2* sel;    // [BG][P * seg] {physical page, head mask | valid tokens << 16}
  float* part;  // [max chunks][G][D + 4]: m (log2 units), l, 0, 0, acc[D]
  int P, seg;
};

struct TileMeta {
  int chunk;
  int flags;
  int vr;               // valid token rows (a prefix of the tile)
  int pad[3];
  uint16_t wmask[kCw];  // head mask of the page holding each consumer warp's 16 rows
};
static_assert(sizeof(TileMeta) == 32, "TileMeta");

// A reserved chunk with its first 32 list entries, prepared by the scheduler warp.
struct ChunkDesc {
  int chunk, bg, p0, p1;
  int2 sel[32];
};

struct StreamArgs {
  CUtensorMap tm_k, tm_v;
  const void* q;
  int64_t qs0, qs1;
  void* out;
  int64_t os0, os1;
  int64_t Hkv, sel_row, page;
  int G, ppt, stages;
  float scale2;
  FastWs w;
  unsigned* status;
};

inline size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

// Parts per request: enough selection CTAs to cover the GPU, parts of >= 64 pages.
int sel_parts(int64_t B, int64_t maxL) {
  const int64_t want = kSelSplitCtas / std::max<int64_t>(B, 1);
  const int64_t cap = std::max<int64_t>(1, (maxL + 63) / 64);
  return (int)std::max<int64_t>(1, std::min<int64_t>({kMaxParts, want, cap}));
}

// Chunks never span two parts: a unit has <= (its pages / chunk pages) + P chunks.
int64_t max_chunks(int64_t BG, int64_t maxL, int P) {
  return BG * P + std::min<int64_t>(kChunkTarget, BG * std::max<int64_t>(maxL, 1));
}

// Workspace layout; returns its size.  Fills *w when base is given.
size_t carve(void* base, int64_t B, int64_t Hkv, int64_t maxL, int64_t G, int64_t D, FastWs* w) {
  const int64_t BG = B * Hkv;
  const int P = sel_parts(B, maxL);
  const int seg = (int)((std::max<int64_t>(maxL, 1) + P - 1) / P);
  const int64_t mc = max_chunks(BG, maxL, P);
  char* c = static_cast<char*>(base);
  size_t o = 0;
  auto take = [&](size_t bytes) {
    char* r = c ? c + o : nullptr;
    o += al256(bytes);
    return r;
  };
  FastWs t;
  t.hdr = reinterpret_cast<DecHeader*>(take(sizeof(DecHeader)));
  t.count = reinterpret_cast<int*>(take((size_t)BG * P * 4));
  t.uinfo = reinterpret_cast<int2*>(take((size_t)BG * 8));
  t.table = reinterpret_cast<int4*>(take((size_t)mc * 16));
  t.sel = reinterpret_cast<int2*>(take((size_t)BG * P * seg * 8));
  t.part = reinterpret_cast<float*>(take((size_t)mc * G * (D + 4) * 4));
  t.P = P;
  t.seg = seg;
  if (w) *w = t;
  return o;
}

// ---------------------------------------------------------------------------------------
// 1-2. page selection and chunking
// ---------------------------------------------------------------------------------------
__global__ void decode_init_kernel(DecHeader* hdr) {
  pdl_trigger();
  hdr->next = 0;
  hdr->total = 0;
}

// Exclusive prefix of v over the CTA (kSelThreads threads); *total gets the sum.
__device__ __forceinline__ int cta_excl_scan(int v, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  int base = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < kSelThreads / 32; ++w) {
    const int t = s_warp[w];
    base += w < warp ? t : 0;
    tot += t;
  }
  __syncthreads();  // s_warp may be rewritten by the next call
  *total = tot;
  return base + x - v;
}

// One CTA per request.  Pass 1 (per 512-page tile): each warp takes 4 pages at a time, its
// lanes the query heads, so a page's routing vectors for all heads are read as one
// contiguous run; a ballot per page gives the H-bit mask of heads that select it.  Pass 2:
// one thread per page, per KV group a warp ballot + per-warp counts give the ascending
// compaction of the group's selected pages into the unit's list.
template <typename RT, int PP, int KK>
__global__ void __launch_bounds__(kSelThreads, 2) decode_select_kernel(const DecodeParams p,
                                                                    const FastWs w, int ppt) {
  const RT* router = static_cast<const RT*>(p.router);
  pdl_trigger();
  const int part = blockIdx.x;
  const int64_t b = blockIdx.y;
  const int H = (int)p.H, G = (int)p.G, r = (int)p.r, Hkv = (int)p.Hkv;
  const int HW = (H + 31) / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ uint32_t s_hmask[kSelTile][kMaxHeadWords];
  __shared__ int s_phys[kSelTile];
  __shared__ int s_valid[kSelTile];
  __shared__ int32_t s_qr[kMaxHeads][kMaxSelLevels + 1];  // padded: lanes over heads, distinct banks
  __shared__ uint8_t s_miss[kSelWarps][PP * kMaxHeads];  // per warp: [page of the step][head]
  __shared__ int s_cnt[kSelWarps][kMaxHeadWords * 32];
  __shared__ int s_run[kMaxHeadWords * 32];
  __shared__ int s_warp[kSelWarps];
  __shared__ long long s_sum[kSelWarps];
  __shared__ int s_last;
  __shared__ long long s_total;
  const int64_t ctx = p.ctx[b];
  // Lanes run over the (head, level < r) pairs that are compared, KK words per lane and PP
  // pages per step: the loads of one step (PP * KK per lane) are all in flight together.
  constexpr int NST = 32 / PP;  // steps covered by one block-table load per lane
  const int64_t lo = (int64_t)part * w.seg;
  // Warp w takes a tile's pages s * 8PP + w * PP + [0, PP) in steps s < NST; one block-table
  // load per lane covers all NST steps.  The first tile's load is issued with the context
  // length's: it reads within the part and the table's width, and entries past the context
  // are never used.
  const int my_lt = (lane / PP) * (kSelWarps * PP) + warp * PP + (lane % PP);
  int my_phys_next =
      my_lt < min((int64_t)min(kSelTile, w.seg), p.maxL - lo) ? p.bt[b * p.bts[0] + (lo + my_lt) * p.bts[1]] : 0;
  for (int i = tid; i < H * r; i += kSelThreads) {
    const int h = i / r, lvl = i % r;
    s_qr[h][lvl] = (int32_t)load_any_i64(p.qrouter, p.qrouter_dtype,
                                         b * p.qrs[0] + h * p.qrs[1] + lvl * p.qrs[2]);
  }
  for (int g = tid; g < Hkv; g += kSelThreads) s_run[g] = 0;
  __syncthreads();
  // logical pages past the block table's width are not read (a consistent request has none)
  const int64_t nlog = ctx > 0 ? min((ctx + p.page - 1) / p.page, p.maxL) : 0;
  const int HR = H * r;
  uint8_t* mflag = s_miss[warp];
  const int64_t hi = min(nlog, lo + w.seg);
  const int64_t row = (int64_t)w.P * w.seg;  // one unit's list row
  for (int64_t t0 = lo; t0 < hi; t0 += kSelTile) {
    const int tn = (int)min((int64_t)kSelTile, hi - t0);
    // ---- pass 1: head masks
    const int my_phys = my_phys_next;  // entries past tn are never used
    if (t0 + kSelTile < hi) {
      const int64_t nt = min((int64_t)kSelTile, hi - t0 - kSelTile);
      my_phys_next = my_lt < nt ? p.bt[b * p.bts[0] + (t0 + kSelTile + my_lt) * p.bts[1]] : 0;
    }
    for (int st = 0; st < NST; ++st) {
      const int lt = st * (kSelWarps * PP) + warp * PP;  // first page of this step
      if (lt >= tn) break;
      int ph[PP];  // pages past the tile's end repeat the step's first page (ignored)
#pragma unroll
      for (int u = 0; u < PP; ++u) ph[u] = __shfl_sync(0xffffffffu, my_phys, st * PP + (lt + u < tn ? u : 0));
      for (int x = lane; x < PP * kMaxHeads / 4; x += 32) reinterpret_cast<uint32_t*>(mflag)[x] = 0u;
      __syncwarp();
      for (int k0 = 0; k0 < HR; k0 += 32 * KK) {
        int64_t off[KK];
#pragma unroll
        for (int kk = 0; kk < KK; ++kk) {
          const int jp = min(k0 + kk * 32 + lane, HR - 1);
          const int h = jp / r, lvl = jp - h * r;
          off[kk] = h * p.rs[1] + lvl * p.rs[2];
        }
        RT v[PP][KK];
#pragma unroll
        for (int u = 0; u < PP; ++u)
#pragma unroll
          for (int kk = 0; kk < KK; ++kk) v[u][kk] = __ldg(router + (int64_t)ph[u] * p.rs[0] + off[kk]);
#pragma unroll
        for (int kk = 0; kk < KK; ++kk) {
          const int jp = k0 + kk * 32 + lane;
          if (jp < HR) {
            const int h = jp / r, lvl = jp - h * r;
            const int64_t q = s_qr[h][lvl];
#pragma unroll
            for (int u = 0; u < PP; ++u)
              if ((int64_t)v[u][kk] != q) mflag[u * kMaxHeads + h] = 1;
          }
        }
      }
      __syncwarp();
      for (int hc = 0; hc < HW; ++hc) {
        const int h = hc * 32 + lane;
        const bool active = h < H;
#pragma unroll
        for (int u = 0; u < PP; ++u) {
          const int64_t l = t0 + lt + u;
          const bool forced = (p.sink && l == 0) || (p.local_blocks > 0 && l >= nlog - p.local_blocks);
          const bool match = active && (forced || !mflag[u * kMaxHeads + (active ? h : 0)]);
          const unsigned m = __ballot_sync(0xffffffffu, match);
          if (lane == 0 && lt + u < tn) s_hmask[lt + u][hc] = m;
        }
      }
      const int phys_l = __shfl_sync(0xffffffffu, my_phys, st * PP + (lane % PP));  // all lanes
      if (lane < PP && lt + lane < tn) {
        s_phys[lt + lane] = phys_l;
        s_valid[lt + lane] = (int)min(p.page, ctx - (t0 + lt + lane) * p.page);
      }
    }
    __syncthreads();
    // ---- pass 2: per-group ascending compaction of this tile (one thread per page)
    const int i = tid;
    auto group_bits = [&](int g) -> unsigned {
      if (i >= tn) return 0u;
      const int bit = g * G, wd = bit >> 5, off = bit & 31;
      uint64_t x = s_hmask[i][wd];
      if (wd + 1 < HW) x |= (uint64_t)s_hmask[i][wd + 1] << 32;
      return (unsigned)((x >> off) & ((1ull << G) - 1ull));
    };
    for (int g = 0; g < Hkv; ++g) {
      const unsigned bl = __ballot_sync(0xffffffffu, group_bits(g) != 0u);
      if (lane == 0) s_cnt[warp][g] = __popc(bl);
    }
    __syncthreads();
    for (int g = tid; g < Hkv; g += kSelThreads) {  // exclusive prefix over the warp slices
      int run = s_run[g];
      for (int q = 0; q < kSelWarps; ++q) {
        const int c = s_cnt[q][g];
        s_cnt[q][g] = run;
        run += c;
      }
      s_run[g] = run;
    }
    __syncthreads();
    for (int g = 0; g < Hkv; ++g) {
      const unsigned gb = group_bits(g);
      const unsigned bl = __ballot_sync(0xffffffffu, gb != 0u);
      if (gb) {
        const int pos = s_cnt[warp][g] + __popc(bl & ((1u << lane) - 1u));
        w.sel[(b * Hkv + g) * row + (int64_t)part * w.seg + pos] =
            make_int2(s_phys[i], (int)(gb | ((unsigned)s_valid[i] << 16)));
      }
    }
    __syncthreads();  // the tile's shared arrays are rewritten by the next tile
  }
  long long mine = 0;
  for (int g = tid; g < Hkv; g += kSelThreads) {
    w.count[(b * Hkv + g) * w.P + part] = s_run[g];
    mine += s_run[g];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
  if (lane == 0) s_sum[warp] = mine;

  // The CTA adds its selected pairs and itself to the header's count; the last CTA
  // to finish cuts the lists into chunks (the header was zeroed by the init kernel, which
  // must have completed).
  pdl_wait();
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    long long cta = 0;
    for (int i = 0; i < kSelWarps; ++i) cta += s_sum[i];
    // one atomic: CTAs finished in the top 24 bits, selected pairs in the low 40, so the CTA
    // that finishes last learns so, and the complete total, from the value it replaced
    const unsigned long long old =
        atomicAdd(&w.hdr->total, (1ull << kTickShift) | (unsigned long long)cta);
    s_last = (old >> kTickShift) == gridDim.x * gridDim.y - 1;
    s_total = (long long)(old & ((1ull << kTickShift) - 1ull)) + cta;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int64_t BG = p.B * p.Hkv;
  const int P = w.P;
  // each round's loads of the next round's part lengths go out before its scan: one
  // dependent round trip instead of one per round
  const long long total = s_total;
  int cnt_next[kMaxParts];
#pragma unroll
  for (int q = 0; q < kMaxParts; ++q) cnt_next[q] = tid < BG && q < P ? __ldcg(w.count + (int64_t)tid * P + q) : 0;
  int chp = (int)std::max<long long>(ppt, (total + kChunkTarget - 1) / kChunkTarget);
  chp = (chp + ppt - 1) / ppt * ppt;
  int run = 0;
  uint16_t* out = static_cast<uint16_t*>(p.out);
  for (int64_t i0 = 0; i0 < BG; i0 += kSelThreads) {
    const int64_t i = i0 + tid;
    int cnt[kMaxParts];  // this unit's part lengths
#pragma unroll
    for (int q = 0; q < kMaxParts; ++q) cnt[q] = cnt_next[q];
    const int64_t inext = i + kSelThreads;
#pragma unroll
    for (int q = 0; q < kMaxParts; ++q)
      cnt_next[q] = inext < BG && q < P ? __ldcg(w.count + inext * P + q) : 0;
    int cu_tot = 0;
#pragma unroll
    for (int q = 0; q < kMaxParts; ++q) cu_tot += cnt[q];
    // a long list gets longer chunks so that its final merge reads about kMaxUnitChunks
    // partials; chunks never span two parts
    int cu = max(chp, (cu_tot + kMaxUnitChunks - 1) / kMaxUnitChunks);
    cu = (cu + ppt - 1) / ppt * ppt;
    int n = 0;
#pragma unroll
    for (int q = 0; q < kMaxParts; ++q) n += (cnt[q] + cu - 1) / cu;
    int t;
    const int base = run + cta_excl_scan(n, s_warp, &t);
    if (i < BG) {
      w.uinfo[i] = make_int2(base, n);
      int k = 0;
#pragma unroll
      for (int q = 0; q < kMaxParts; ++q) {
        const int c = cnt[q], off = q * w.seg;
        for (int pb = 0; pb < c; pb += cu, ++k) {
          const int pe = off + min(c, pb + cu);
          w.table[base + k] = make_int4((int)i, (off + pb) | (pe << 16), base, n);
        }
      }
      if (cu_tot == 0) {  // a unit with no page: its rows are zero (no chunk writes them)
        const int64_t b = i / p.Hkv, g = i % p.Hkv;
        for (int j = 0; j < G * p.D; ++j)
          out[b * p.os[0] + (g * G + j / p.D) * p.os[1] + j % p.D] = 0;  // +0.0 in bf16 and fp16
      }
    }
    run += t;
  }
  if (tid == 0) {
    w.hdr->n_chunks = run;
    w.hdr->chp = chp;
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
  int2* s_sel = reinterpret_cast<int2*>(einfo + 4);  // [32] producer's page batch
  ChunkDesc* desc = reinterpret_cast<ChunkDesc*>(s_sel + 32);  // [kDescs] scheduler -> producer
  uint64_t* dfull = reinterpret_cast<uint64_t*>(desc + kDescs);
  uint64_t* dempty = dfull + kDescs;
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
  pdl_wait();  // the selection kernel's lists, table and header are complete from here on

  if (warp == 0) {
    // ---------------- producer ----------------
    uint32_t tile = 0, qi = 0;
    bool ok = true;
    for (uint32_t d = 0; ok; ++d) {
      const uint32_t ds = d % kDescs;
      if (!(ok = mbar_wait_warp(&dfull[ds], (d / kDescs) & 1, a.status))) break;
      const ChunkDesc& cd = desc[ds];
      const int c = cd.chunk;
      if (c < 0) break;
      const int bg = cd.bg, p0 = cd.p0, p1 = cd.p1;
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
      }
      ++qi;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      const int2* sel = a.w.sel + (int64_t)bg * a.sel_row;
      for (int i0 = p0; i0 < p1 && ok; i0 += 32) {
        const int nb = min(32, p1 - i0);
        // the first 32 entries came with the descriptor; longer chunks load the rest here
        const int2* bsel = cd.sel;
        if (i0 != p0) {
          __syncwarp();
          if (lane < nb) s_sel[lane] = __ldcg(sel + i0 + lane);
          __syncwarp();
          bsel = s_sel;
        }
        if (lane == 0) {
          if (a.page >= kTile) {
            // a page is page/64 tiles; tiles past the context end are skipped
            for (int k = 0; k < nb && ok; ++k) {
              const int2 e = bsel[k];
              const int valid = (int)((unsigned)e.y >> 16);
              const uint16_t mk = (uint16_t)(e.y & 0xffff);
              for (int t0 = 0; t0 < valid; t0 += kTile, ++tile) {
                const uint32_t st = tile % stages;
                if (!(ok = mbar_wait(&empty[st], ((tile / stages) & 1) ^ 1, a.status))) break;
                TileMeta& m = meta[st];
                const bool last = i0 + k == p1 - 1 && t0 + kTile >= valid;
                m.chunk = c;
                m.flags = (i0 + k == p0 && t0 == 0 ? kFirst : 0) | (last ? kLast : 0);
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
            // ppt = 64/page pages per tile; chunk boundaries are multiples of ppt
            const int ppt = a.ppt, page = (int)a.page;
            for (int k = 0; k < nb && ok; k += ppt, ++tile) {
              const int n = min(ppt, nb - k);
              const uint32_t st = tile % stages;
              if (!(ok = mbar_wait(&empty[st], ((tile / stages) & 1) ^ 1, a.status))) break;
              TileMeta& m = meta[st];
              const bool last = i0 + k + n == p1;
              m.chunk = c;
              m.flags = (i0 + k == p0 ? kFirst : 0) | (last ? kLast : 0);
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
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
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
  } else if (warp == kSchedWarp) {
    // ---------------- scheduler: reserve the next chunk and fetch its entries ----------------
    // Up to kDescs - 1 descriptors ahead of the producer, so that runs of one-page chunks do
    // not wait on the queue's atomic -> table -> list chain.  CTA x takes chunk x first; the
    // queue counter hands out the rest from chunk gridDim.x on.
    // Near the queue's end (fewer than two chunks per CTA left) the lookahead shrinks to one:
    // the next chunk is reserved only once the producer has issued the previous one's loads,
    // so that the last chunks spread over the CTAs instead of waiting in one CTA's ring while
    // the others go idle.
    const int n_chunks = __ldcg(&a.w.hdr->n_chunks);
    int last_c = 0;
    for (uint32_t d = 0;; ++d) {
      const uint32_t ds = d % kDescs;
      if (!mbar_wait_warp(&dempty[ds], ((d / kDescs) & 1) ^ 1, a.status)) break;
      if (d > 0 && n_chunks - last_c < 2 * (int)gridDim.x &&
          !mbar_wait_warp(&dempty[(d - 1) % kDescs], ((d - 1) / kDescs) & 1, a.status))
        break;
      int c = 0;
      if (lane == 0) c = d == 0 ? (int)blockIdx.x : (int)gridDim.x + atomicAdd(&a.w.hdr->next, 1);
      c = __shfl_sync(0xffffffffu, c, 0);
      last_c = c;
      ChunkDesc& cd = desc[ds];
      if (c >= n_chunks) {
        if (lane == 0) {
          cd.chunk = -1;
          mbar_arrive(&dfull[ds]);
        }
        break;
      }
      const int4 ent = __ldcg(a.w.table + c);
      const int bg = ent.x, p0 = ent.y & 0xffff, p1 = (int)((unsigned)ent.y >> 16);
      if (lane < min(32, p1 - p0)) cd.sel[lane] = __ldcg(a.w.sel + (int64_t)bg * a.sel_row + p0 + lane);
      if (lane == 0) {
        cd.chunk = c;
        cd.bg = bg;
        cd.p0 = p0;
        cd.p1 = p1;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&dfull[ds]);
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
// 4. per-unit merge of the chunk partials (a programmatic dependent of the stream kernel)
// ---------------------------------------------------------------------------------------
// One CTA per unit.  Its kMaxG * D / 4 threads are CG = kMaxG / G groups of one thread per
// float4 output column of the unit's G heads; group c merges the unit's chunks c, c + CG, ...
// online (eight chunks' loads in flight, one round for most units), then the CG partial
// states are merged through shared memory.  A unit's long chunk list thus costs one round
// of loads instead of a chain of them.
template <typename T, int D>
__global__ void __launch_bounds__(kMaxG * D / 4) decode_unit_combine_kernel(const FastWs w, void* out_,
                                                                          int64_t os0, int64_t os1,
                                                                          int64_t Hkv, int G) {
  constexpr int RS = D + 4;
  constexpr int kThreads = kMaxG * D / 4;
  __shared__ float4 s_acc[kThreads];
  __shared__ float2 s_ml[kThreads];
  pdl_wait();
  const int64_t bg = blockIdx.x;
  const int per_unit = G * (D / 4);
  const int CG = (int)blockDim.x / per_unit;
  const int cg = (int)threadIdx.x / per_unit, i = (int)threadIdx.x % per_unit;
  const int2 ui = w.uinfo[bg];
  if (ui.y == 0) return;  // (CTA-uniform) a unit without pages was zeroed at selection
  const int hh = i / (D / 4), d4 = i % (D / 4);
  const float* ph = w.part + (int64_t)ui.x * G * RS + hh * RS;
  const int64_t CS = (int64_t)G * RS;
  float M = -INFINITY, L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  constexpr int NU = 8;
  const int mine = cg < ui.y ? (ui.y - cg + CG - 1) / CG : 0;  // chunks cg, cg + CG, ...
  for (int k0 = 0; k0 < mine; k0 += NU) {
    float2 ml[NU];
    float4 x[NU];
#pragma unroll
    for (int u = 0; u < NU; ++u) {
      const int k = cg + CG * min(k0 + u, mine - 1);
      ml[u] = __ldcg(reinterpret_cast<const float2*>(ph + k * CS));
      x[u] = __ldcg(reinterpret_cast<const float4*>(ph + k * CS + 4 + 4 * d4));
    }
#pragma unroll
    for (int u = 0; u < NU; ++u) {
      if (k0 + u >= mine) break;
      const float mn = fmaxf(M, ml[u].x);
      const float ref = mn == -INFINITY ? 0.f : mn;
      const float so = fast_exp2(M - ref), sn = fast_exp2(ml[u].x - ref);
      acc.x = acc.x * so + x[u].x * sn;
      acc.y = acc.y * so + x[u].y * sn;
      acc.z = acc.z * so + x[u].z * sn;
      acc.w = acc.w * so + x[u].w * sn;
      L = L * so + ml[u].y * sn;
      M = mn;
    }
  }
  if (threadIdx.x < (unsigned)(CG * per_unit)) {
    s_acc[threadIdx.x] = acc;
    s_ml[threadIdx.x] = make_float2(M, L);
  }
  __syncthreads();
  if (cg != 0) return;
  for (int c = 1; c < CG; ++c) {  // group 0 folds in the other groups' states
    const float2 ml = s_ml[c * per_unit + i];
    const float4 x = s_acc[c * per_unit + i];
    const float mn = fmaxf(M, ml.x);
    const float ref = mn == -INFINITY ? 0.f : mn;
    const float so = fast_exp2(M - ref), sn = fast_exp2(ml.x - ref);
    acc.x = acc.x * so + x.x * sn;
    acc.y = acc.y * so + x.y * sn;
    acc.z = acc.z * so + x.z * sn;
    acc.w = acc.w * so + x.w * sn;
    L = L * so + ml.y * sn;
    M = mn;
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
  static_assert((2 * kQBufs + 4) * 8 + 16 + 32 * 8 + kDescs * (sizeof(ChunkDesc) + 16) <= 2048,
                "decode: barrier and descriptor area");
  const size_t fixed = 1024 + kQBufs * (size_t)a.G * D * 2 + 2 * (size_t)kCw * a.G * (D + 4) * 4 + 2048;
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
  return (int64_t)carve(nullptr, B, Hkv, maxL, H / Hkv, D, nullptr);
}

int launch_decode_fast(const DecodeParams& p, int dtype, void* workspace, int64_t workspace_bytes,
                       cudaStream_t stream) {
  const int64_t BG = p.B * p.Hkv;
  FastWs w;
  const size_t need = carve(workspace, p.B, p.Hkv, p.maxL, p.G, p.D, &w);
  if ((int64_t)need > workspace_bytes || !workspace)
    return fail(SA_EWORKSPACE, "decode: workspace too small (" + std::to_string(workspace_bytes) +
                                   " < " + std::to_string(need) + ")");
  if (p.B > 65535) return fail(SA_EUNSUPPORTED, "decode: more than 65535 requests");
  StreamArgs a{};
  a.status = device_status_ptr();
  if (!a.status) return fail(SA_ELAUNCH, std::string("decode: ") + sa_last_error());
  const uint32_t box_n = (uint32_t)std::min<int64_t>(p.page, kTile);
  int rc = make_tmap_4d(&a.tm_k, p.kc, dtype, p.num_pages, p.Hkv, p.page, p.D, p.ks, 64, box_n);
  if (!rc) rc = make_tmap_4d(&a.tm_v, p.vc, dtype, p.num_pages, p.Hkv, p.page, p.D, p.vs, 64, box_n);
  if (rc) return fail(SA_ELAUNCH, std::string("decode: tensor map: ") + sa_last_error());

  decode_init_kernel<<<1, 1, 0, stream>>>(w.hdr);
  rc = check_launch("decode_init_kernel");
  if (rc) return rc;
  const int ppt = p.page >= kTile ? 1 : (int)(kTile / p.page);
  {
    // pages x compared words per lane and step: as many loads in flight as fit in registers
    const int64_t HR = p.H * p.r;
    const dim3 sg((unsigned)w.P, (unsigned)p.B), sb(kSelThreads);
    const char* sn = "decode_select_kernel";
    const bool i64 = p.router_dtype == SA_I64;
    if (HR <= 128)
      rc = i64 ? launch_dependent(decode_select_kernel<int64_t, 4, 4>, sg, sb, 0, stream, sn, p, w, ppt)
               : launch_dependent(decode_select_kernel<int32_t, 8, 4>, sg, sb, 0, stream, sn, p, w, ppt);
    else
      rc = i64 ? launch_dependent(decode_select_kernel<int64_t, 4, 4>, sg, sb, 0, stream, sn, p, w, ppt)
               : launch_dependent(decode_select_kernel<int32_t, 4, 8>, sg, sb, 0, stream, sn, p, w, ppt);
  }
  if (rc) return rc;

  a.q = p.q;
  a.qs0 = p.qs[0];
  a.qs1 = p.qs[1];
  a.out = p.out;
  a.os0 = p.os[0];
  a.os1 = p.os[1];
  a.Hkv = p.Hkv;
  a.sel_row = (int64_t)w.P * w.seg;
  a.page = p.page;
  a.G = (int)p.G;
  a.ppt = ppt;
  a.scale2 = (1.0f / sqrtf((float)p.D)) * kLog2e;
  a.w = w;
  const int grid = (int)std::min<int64_t>(device_sm_count(), max_chunks(BG, p.maxL, w.P));
  const bool bf = dtype == SA_BF16;
  if (p.D == 64)
    rc = bf ? launch_stream<64, true>(a, grid, stream) : launch_stream<64, false>(a, grid, stream);
  else
    rc = bf ? launch_stream<128, true>(a, grid, stream) : launch_stream<128, false>(a, grid, stream);
  if (rc) return rc;
  // one CTA per unit: kMaxG / G chunk groups of G * D / 4 threads (<= kMaxG * D / 4)
  const dim3 cg((unsigned)BG), cb((unsigned)((kMaxG / p.G) * p.G * p.D / 4));
  const char* cn = "decode_unit_combine_kernel";
  if (p.D == 64)
    return bf ? launch_dependent(decode_unit_combine_kernel<__nv_bfloat16, 64>, cg, cb, 0, stream, cn, w,
                                 p.out, p.os[0], p.os[1], p.Hkv, (int)p.G)
              : launch_dependent(decode_unit_combine_kernel<__half, 64>, cg, cb, 0, stream, cn, w, p.out,
                                 p.os[0], p.os[1], p.Hkv, (int)p.G);
  return bf ? launch_dependent(decode_unit_combine_kernel<__nv_bfloat16, 128>, cg, cb, 0, stream, cn, w,
                               p.out, p.os[0], p.os[1], p.Hkv, (int)p.G)
            : launch_dependent(decode_unit_combine_kernel<__half, 128>, cg, cb, 0, stream, cn, w, p.out,
                               p.os[0], p.os[1], p.Hkv, (int)p.G);
}

}  // namespace sa

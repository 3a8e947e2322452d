// Routed sparse paged decode (one query token per request), split-K over the routed pages.
//
// Semantics of src/ultrametric/kernel_decode.py:23-124 / :129-185 in sparse-ai: request b,
// query head h attends the logical pages whose routing vector (router[phys, h, :r], indexed
// by the PHYSICAL page id) equals q_router[b, h, :r], plus logical page 0 (sink) and the
// last `local_blocks` pages; tokens >= context_lens[b] are masked; ctx == 0 -> zeros.
//
// Work split: CTA = (split s, KV head g, request b).  Each CTA scans the request's logical
// pages once, keeps those selected by ANY query head of the GQA group (with a per-head
// bit mask), takes its contiguous share of that list, and streams the K/V pages of the
// KV head with 16-byte cp.async into a shared-memory ring.  Every loaded page serves all
// G query heads of the group (K/V bytes are read once per KV head).  Within the CTA each
// "token slot" (LPT lanes) runs its own online softmax; slots and splits are merged in
// fp32 by log-sum-exp weights (slots in the CTA epilogue, splits in a second kernel).
#include <string>

#include "decode.cuh"

namespace sa {
namespace {

constexpr int kDecThreads = 128;
constexpr int kMaxSplits = 64;



__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename T>
__device__ __forceinline__ void load_chunk(const T* src, float* dst) {
  // one 16-byte chunk -> 16/sizeof(T) floats
  const uint4 raw = *reinterpret_cast<const uint4*>(src);
  if constexpr (sizeof(T) == 4) {
    dst[0] = __uint_as_float(raw.x);
    dst[1] = __uint_as_float(raw.y);
    dst[2] = __uint_as_float(raw.z);
    dst[3] = __uint_as_float(raw.w);
  } else {
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = to_f32<T>(e[i]);
  }
}

// GT: compile-time max heads per group (runtime G <= GT); DPL: head dims per lane.
template <typename T, int D, int GT>
__global__ void __launch_bounds__(kDecThreads) decode_split_kernel(DecodeParams p) {
  constexpr int DPL = GT >= 8 ? 8 : 16;
  constexpr int LPT = D / DPL;              // lanes per token
  constexpr int CE = 16 / sizeof(T);        // elements per 16-byte chunk
  constexpr int NCH = DPL / CE;             // chunks per lane
  constexpr int SLOTS = kDecThreads / LPT;  // token slots per CTA
  static_assert(D % DPL == 0 && LPT >= 1 && LPT <= 32, "head_dim");

  extern __shared__ __align__(16) unsigned char dsm[];
  const int s_idx = blockIdx.x, g = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int G = (int)p.G;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t ctx = p.ctx[b];
  const int64_t nlog = ctx > 0 ? (ctx + p.page - 1) / p.page : 0;

  // ---- shared layout: [sel pages int32 maxL][sel masks uint8 maxL][pipeline stages]
  int32_t* s_pages = reinterpret_cast<int32_t*>(dsm);
  uint8_t* s_mask = reinterpret_cast<uint8_t*>(s_pages + p.maxL);
  __shared__ int s_warp_tot[kDecThreads / 32];
  __shared__ int s_count;
  __shared__ int32_t s_qr[8][32];  // query routes of the group's heads (first r <= 32 levels)
  const size_t route_bytes = ((size_t)p.maxL * 5 + 127) & ~(size_t)127;
  T* ring = reinterpret_cast<T*>(dsm + route_bytes);
  const int64_t page_elems = p.page * D;

  // ---- 1. route scan: ascending list of pages selected by any head of the group
  const int r = (int)p.r;
  for (int i = tid; i < G * r; i += kDecThreads) {
    const int hh = i / r, lvl = i % r;
    s_qr[hh][lvl] = (int32_t)load_any_i64(
        p.qrouter, p.qrouter_dtype, b * p.qrs[0] + (g * G + hh) * p.qrs[1] + lvl * p.qrs[2]);
  }
  if (tid == 0) s_count = 0;
  __syncthreads();
  for (int64_t l0 = 0; l0 < nlog; l0 += kDecThreads) {
    const int64_t l = l0 + tid;
    unsigned mask = 0;
    if (l < nlog) {
      const bool forced = (p.sink && l == 0) || (p.local_blocks > 0 && l >= nlog - p.local_blocks);
      if (forced) {
        mask = (1u << G) - 1u;
      } else {
        const int64_t phys = p.bt[b * p.bts[0] + l * p.bts[1]];
        for (int hh = 0; hh < G; ++hh) {
          bool ok = true;
          const int64_t rb = phys * p.rs[0] + (g * G + hh) * p.rs[1];
          for (int lvl = 0; lvl < r && ok; ++lvl)
            ok = load_any_i64(p.router, p.router_dtype, rb + lvl * p.rs[2]) == s_qr[hh][lvl];
          if (ok) mask |= 1u << hh;
        }
      }
    }
    const bool sel = mask != 0;
    const unsigned ball = __ballot_sync(0xffffffffu, sel);
    if (lane == 0) s_warp_tot[warp] = __popc(ball);
    __syncthreads();
    int base = s_count;
    for (int w = 0; w < warp; ++w) base += s_warp_tot[w];
    const int pos = base + __popc(ball & ((1u << lane) - 1u));
    if (sel) {
      s_pages[pos] = (int32_t)l;
      s_mask[pos] = (uint8_t)mask;
    }
    __syncthreads();  // every thread has read s_count and s_warp_tot
    if (tid == 0) {
      int tot = 0;
      for (int w = 0; w < kDecThreads / 32; ++w) tot += s_warp_tot[w];
      s_count += tot;
    }
    __syncthreads();
  }
  const int count = s_count;
  const int per = (count + p.S - 1) / p.S;
  const int beg = min(count, s_idx * per), end = min(count, beg + per);

  // ---- 2. per-lane query values (pre-scaled to log2 units)
  const int slot = tid / LPT, li = tid % LPT;
  const float qk_scale = (1.0f / sqrtf((float)D)) * kLog2e;
  float qv[GT][DPL];
#pragma unroll
  for (int hh = 0; hh < GT; ++hh) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
#pragma unroll
      for (int e = 0; e < CE; ++e) {
        const int d = (li + c * LPT) * CE + e;
        qv[hh][c * CE + e] =
            hh < G ? to_f32<T>(static_cast<const T*>(p.q)[b * p.qs[0] + (g * G + hh) * p.qs[1] + d]) *
                         qk_scale
                   : 0.f;
      }
    }
  }
  float m[GT], l[GT], acc[GT][DPL];
#pragma unroll
  for (int hh = 0; hh < GT; ++hh) {
    m[hh] = -INFINITY;
    l[hh] = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[hh][i] = 0.f;
  }

  // ---- 3. stream the pages [beg, end) through the ring
  auto issue = [&](int e, int stage) {
    if (e < end) {
      const int64_t lp = s_pages[e];
      const int64_t phys = p.bt[b * p.bts[0] + lp * p.bts[1]];
      const T* kb = static_cast<const T*>(p.kc) + phys * p.ks[0] + g * p.ks[1];
      const T* vb = static_cast<const T*>(p.vc) + phys * p.vs[0] + g * p.vs[1];
      T* sk = ring + (size_t)stage * 2 * page_elems;
      T* sv = sk + page_elems;
      const int chunks = (int)(page_elems / CE);
      for (int c = tid; c < chunks; c += kDecThreads) {
        const int64_t tok = (int64_t)c / (D / CE), dc = (int64_t)(c % (D / CE)) * CE;
        cp_async16(sk + tok * D + dc, kb + tok * p.ks[2] + dc);
        cp_async16(sv + tok * D + dc, vb + tok * p.vs[2] + dc);
      }
    }
    cp_async_commit();
  };
  const int stages = p.stages;
  for (int st = 0; st < stages - 1; ++st) issue(beg + st, st);
  for (int e = beg; e < end; ++e) {
    const int stage = (e - beg) % stages;
    issue(e + stages - 1, (e - beg + stages - 1) % stages);
    // the group issued for page e is now (stages - 1) groups old
    if (stages == 3) cp_async_wait<2>(); else cp_async_wait<1>();
    __syncthreads();
    const T* sk = ring + (size_t)stage * 2 * page_elems;
    const T* sv = sk + page_elems;
    const int64_t lp = s_pages[e];
    const unsigned hmask = s_mask[e];
    const int valid = (int)min((int64_t)p.page, ctx - lp * p.page);
    // warp-uniform trip count: the score reduction shuffles need every lane present
    for (int t0 = 0; t0 < valid; t0 += 4 * SLOTS) {
      float sc[4][GT];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int tok = t0 + slot + u * SLOTS;
        float kf[DPL];
        if (tok < valid) {
#pragma unroll
          for (int c = 0; c < NCH; ++c) load_chunk<T>(sk + tok * D + (li + c * LPT) * CE, kf + c * CE);
        } else {
#pragma unroll
          for (int i = 0; i < DPL; ++i) kf[i] = 0.f;
        }
#pragma unroll
        for (int hh = 0; hh < GT; ++hh) {
          float a = 0.f;
#pragma unroll
          for (int i = 0; i < DPL; ++i) a = fmaf(qv[hh][i], kf[i], a);
#pragma unroll
          for (int o = LPT / 2; o; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
          sc[u][hh] = (tok < valid && hh < G && ((hmask >> hh) & 1u)) ? a : -INFINITY;
        }
      }
#pragma unroll
      for (int hh = 0; hh < GT; ++hh) {
        const float mt = fmaxf(fmaxf(sc[0][hh], sc[1][hh]), fmaxf(sc[2][hh], sc[3][hh]));
        const float m_new = fmaxf(m[hh], mt);
        const float m_ref = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = fast_exp2(m[hh] - m_ref);
        m[hh] = m_new;
        l[hh] *= alpha;
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[hh][i] *= alpha;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          sc[u][hh] = fast_exp2(sc[u][hh] - m_ref);
          l[hh] += sc[u][hh];
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int tok = t0 + slot + u * SLOTS;
        if (tok >= valid) continue;
        float vf[DPL];
#pragma unroll
        for (int c = 0; c < NCH; ++c) load_chunk<T>(sv + tok * D + (li + c * LPT) * CE, vf + c * CE);
#pragma unroll
        for (int hh = 0; hh < GT; ++hh)
#pragma unroll
          for (int i = 0; i < DPL; ++i) acc[hh][i] = fmaf(sc[u][hh], vf[i], acc[hh][i]);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- 4. merge the token slots of this CTA and write the split partial
  float* red = reinterpret_cast<float*>(ring);  // [SLOTS][GT][D + 2]
  const int RS = D + 2;
#pragma unroll
  for (int hh = 0; hh < GT; ++hh) {
    float* rr = red + ((size_t)slot * GT + hh) * RS;
    if (li == 0) {
      rr[0] = m[hh];
      rr[1] = l[hh];
    }
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int e2 = 0; e2 < CE; ++e2) rr[2 + (li + c * LPT) * CE + e2] = acc[hh][c * CE + e2];
  }
  __syncthreads();
  float* outp = p.part + (((b * p.Hkv + g) * p.S + s_idx) * p.G) * RS;
  for (int i = tid; i < G * RS; i += kDecThreads) {
    const int hh = i / RS, c = i % RS;
    float M = -INFINITY;
    for (int sl = 0; sl < SLOTS; ++sl) M = fmaxf(M, red[((size_t)sl * GT + hh) * RS]);
    const float Mr = M == -INFINITY ? 0.f : M;
    float v = 0.f;
    if (c == 0) {
      v = M;
    } else {
      for (int sl = 0; sl < SLOTS; ++sl) {
        const float* rr = red + ((size_t)sl * GT + hh) * RS;
        v += rr[c] * fast_exp2(rr[0] - Mr);
      }
    }
    outp[(size_t)hh * RS + c] = v;
  }
}

// Merge the S split partials of (b, h) and write out[b, h, :].  grid (B, H), D threads.
template <typename T>
__global__ void decode_combine_kernel(DecodeParams p) {
  const int64_t b = blockIdx.x, h = blockIdx.y;
  const int64_t g = h / p.G, hh = h % p.G;
  const int RS = (int)p.D + 2;
  const float* base = p.part + ((b * p.Hkv + g) * p.S * p.G + hh) * RS;
  const size_t sstride = (size_t)p.G * RS;
  float M = -INFINITY;
  for (int s = 0; s < p.S; ++s) M = fmaxf(M, base[s * sstride]);
  const float Mr = M == -INFINITY ? 0.f : M;
  float L = 0.f;
  for (int s = 0; s < p.S; ++s) L += base[s * sstride + 1] * fast_exp2(base[s * sstride] - Mr);
  const float inv = L > 0.f ? 1.f / L : 0.f;
  T* o = static_cast<T*>(p.out) + b * p.os[0] + h * p.os[1];
  for (int d = threadIdx.x; d < p.D; d += blockDim.x) {
    float a = 0.f;
    for (int s = 0; s < p.S; ++s)
      a += base[s * sstride + 2 + d] * fast_exp2(base[s * sstride] - Mr);
    o[d] = from_f32<T>(p.ctx[b] > 0 ? a * inv : 0.f);
  }
}

int choose_splits(int64_t B, int64_t Hkv, int64_t maxL) {
  const int64_t units = B * Hkv;
  if (units <= 0) return 1;
  int64_t s = (4 * 148 + units - 1) / units;
  s = s < 1 ? 1 : s;
  const int64_t cap = maxL / 2 > 1 ? maxL / 2 : 1;
  if (s > cap) s = cap;
  if (s > kMaxSplits) s = kMaxSplits;
  return (int)s;
}

template <typename T, int D, int GT>
int launch_decode_t(DecodeParams& p, cudaStream_t stream) {
  const size_t route_bytes = ((size_t)p.maxL * 5 + 127) & ~(size_t)127;
  const size_t stage_bytes = (size_t)2 * p.page * D * sizeof(T);
  constexpr int DPL = GT >= 8 ? 8 : 16;
  const size_t red_bytes = (size_t)(kDecThreads / (D / DPL)) * GT * (D + 2) * sizeof(float);
  int stages = 3;
  size_t ring = stages * stage_bytes;
  if (route_bytes + ring > 200 * 1024) {
    stages = 2;
    ring = stages * stage_bytes;
  }
  if (ring < red_bytes) ring = red_bytes;
  const size_t smem = route_bytes + ring;
  if (smem > 220 * 1024)
    return fail(SA_EUNSUPPORTED, "decode: page_size * head_dim or max_logical_pages too large "
                                 "for the shared-memory ring");
  p.stages = stages;
  auto kern = decode_split_kernel<T, D, GT>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((unsigned)p.S, (unsigned)p.Hkv, (unsigned)p.B);
  kern<<<grid, kDecThreads, smem, stream>>>(p);
  int rc = check_launch("decode_split_kernel");
  if (rc) return rc;
  dim3 g2((unsigned)p.B, (unsigned)p.H);
  decode_combine_kernel<T><<<g2, D < 128 ? (unsigned)D : 128u, 0, stream>>>(p);
  return check_launch("decode_combine_kernel");
}

template <typename T, int D>
int dispatch_group(DecodeParams& p, cudaStream_t s) {
  if (p.G <= 1) return launch_decode_t<T, D, 1>(p, s);
  if (p.G <= 2) return launch_decode_t<T, D, 2>(p, s);
  if (p.G <= 4) return launch_decode_t<T, D, 4>(p, s);
  if (p.G <= 8) return launch_decode_t<T, D, 8>(p, s);
  return fail(SA_EUNSUPPORTED, "decode: more than 8 query heads per KV head");
}

template <typename T>
int dispatch_dim(DecodeParams& p, cudaStream_t s) {
  switch (p.D) {
    case 16: return dispatch_group<T, 16>(p, s);
    case 32: return dispatch_group<T, 32>(p, s);
    case 64: return dispatch_group<T, 64>(p, s);
    case 128: return dispatch_group<T, 128>(p, s);
    case 256: return dispatch_group<T, 256>(p, s);
  }
  return fail(SA_EUNSUPPORTED, "decode: head_dim not in {16,32,64,128,256}");
}

}  // namespace
}  // namespace sa

extern "C" {

int64_t sa_ultrametric_decode_workspace_bytes(int64_t B, int64_t H, int64_t Hkv, int64_t D,
                                              int64_t max_logical_pages) {
  if (B <= 0 || H <= 0 || Hkv <= 0 || D <= 0) return 0;
  const int S = sa::choose_splits(B, Hkv, max_logical_pages);
  const int64_t general = B * Hkv * (int64_t)S * (H / Hkv) * (D + 2) * (int64_t)sizeof(float);
  const int64_t fast = sa::decode_fast_workspace_bytes(B, H, Hkv, D, max_logical_pages);
  return general > fast ? general : fast;
}

int sa_ultrametric_decode(int dtype, int64_t B, int64_t H, int64_t Hkv, int64_t D,
                          int64_t page_size, int64_t num_pages, const void* q,
                          const int64_t* q_strides, const void* k_cache, const int64_t* k_strides,
                          const void* v_cache, const int64_t* v_strides,
                          const int32_t* block_tables, const int64_t* bt_strides,
                          int64_t max_logical_pages, const int32_t* context_lens,
                          const void* router, int router_dtype, const int64_t* router_strides,
                          const void* q_router, int q_router_dtype,
                          const int64_t* q_router_strides, int64_t TD, int64_t req_depth,
                          int64_t local_blocks, int sink_block, void* out,
                          const int64_t* out_strides, void* workspace, int64_t workspace_bytes,
                          void* stream) {
  using namespace sa;
  if (B < 0 || H <= 0 || Hkv <= 0 || D <= 0 || page_size <= 0 || TD < 1)
    return fail(SA_EINVAL, "decode: bad sizes");
  if (B == 0) return SA_OK;
  if (H % Hkv) return fail(SA_EINVAL, "decode: num_heads must be a multiple of the cache heads");
  if (dtype != SA_F32 && dtype != SA_F16 && dtype != SA_BF16)
    return fail(SA_EUNSUPPORTED, "decode: dtype must be fp32, fp16 or bf16");
  if ((router_dtype != SA_I32 && router_dtype != SA_I64) ||
      (q_router_dtype != SA_I32 && q_router_dtype != SA_I64))
    return fail(SA_EUNSUPPORTED, "decode: routing vectors must be int32 or int64");
  if (max_logical_pages > 16384) return fail(SA_EUNSUPPORTED, "decode: more than 16384 pages per request");
  const int64_t esz = dtype == SA_F32 ? 4 : 2;
  if (k_strides[3] != 1 || v_strides[3] != 1 || q_strides[2] != 1 || out_strides[2] != 1)
    return fail(SA_EUNSUPPORTED, "decode: head_dim must be the contiguous dimension");
  for (int i = 0; i < 3; ++i)
    if ((k_strides[i] * esz) % 16 || (v_strides[i] * esz) % 16)
      return fail(SA_EUNSUPPORTED, "decode: cache strides must be multiples of 16 bytes");
  if (reinterpret_cast<uintptr_t>(k_cache) % 16 || reinterpret_cast<uintptr_t>(v_cache) % 16)
    return fail(SA_EUNSUPPORTED, "decode: caches must be 16-byte aligned");
  const int64_t need = sa_ultrametric_decode_workspace_bytes(B, H, Hkv, D, max_logical_pages);
  if (workspace_bytes < need || (need && !workspace))
    return fail(SA_EWORKSPACE, "decode: workspace too small (" + std::to_string(workspace_bytes) +
                                   " < " + std::to_string(need) + ")");
  DecodeParams p{};
  p.B = B;
  p.H = H;
  p.Hkv = Hkv;
  p.G = H / Hkv;
  p.D = D;
  p.page = page_size;
  p.num_pages = num_pages;
  p.maxL = max_logical_pages > 0 ? max_logical_pages : 1;
  p.TD = TD;
  p.r = req_depth < 0 ? 0 : (req_depth > TD ? TD : req_depth);
  if (p.r > 32) return fail(SA_EUNSUPPORTED, "decode: req_depth above 32 levels");
  p.local_blocks = local_blocks;
  p.sink = sink_block;
  p.q = q;
  for (int i = 0; i < 3; ++i) p.qs[i] = q_strides[i];
  p.kc = k_cache;
  p.vc = v_cache;
  for (int i = 0; i < 4; ++i) {
    p.ks[i] = k_strides[i];
    p.vs[i] = v_strides[i];
  }
  p.bt = block_tables;
  p.bts[0] = bt_strides[0];
  p.bts[1] = bt_strides[1];
  p.ctx = context_lens;
  p.router = router;
  p.router_dtype = router_dtype;
  p.qrouter = q_router;
  p.qrouter_dtype = q_router_dtype;
  for (int i = 0; i < 3; ++i) {
    p.rs[i] = router_strides[i];
    p.qrs[i] = q_router_strides[i];
    p.os[i] = out_strides[i];
  }
  p.out = out;
  p.part = static_cast<float*>(workspace);
  p.S = choose_splits(B, Hkv, max_logical_pages);
  cudaStream_t s = (cudaStream_t)stream;
  if (decode_fast_eligible(p, dtype)) return launch_decode_fast(p, dtype, workspace, workspace_bytes, s);
  switch (dtype) {
    case SA_F32: return dispatch_dim<float>(p, s);
    case SA_F16: return dispatch_dim<__half>(p, s);
    default: return dispatch_dim<__nv_bfloat16>(p, s);
  }
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// Decode without any allocation by the caller.
//
// Some callers cannot allocate device memory when they decode: a serving loop whose device
// memory is carved up front by its own pool and that binds only this C ABI (it has no
// allocator to call for the split-K workspace), or a host that must not trigger
// cudaMalloc's implicit device synchronisation in the middle of a decode step.  This entry
// point takes its split-K workspace from a fixed, file-scope device array instead.
//
//  * The array holds kNoAllocScratchBytes (16 MiB).  Every GPU that loads this library
//    keeps it for the life of the process.
//  * Its device address is looked up once per device (cudaGetSymbolAddress, with that
//    device current) on the first call made on that device; make that first call before
//    any stream capture.
//  * Requests whose workspace would exceed the array are rejected with SA_EWORKSPACE.
//  * All calls share the one array: calls that overlap on the GPU (different streams, or
//    different host threads) race on it.  The decode kernel rewrites every slot it reads
//    in the same launch, so nothing needs clearing between calls.
//  * `stream` must belong to the current device (the array is looked up for the current
//    device); a stream of another device is rejected with SA_EINVAL.
// ---------------------------------------------------------------------------------------
#include <mutex>

namespace sa {
namespace {

constexpr int64_t kNoAllocScratchBytes = 16ll << 20;
__device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

void* decode_scratch_ptr() {
  constexpr int kMaxDev = 64;
  static void* ptrs[kMaxDev] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) {
      // clear the runtime's sticky last error, so that a later launch check does not
      // report it against an unrelated kernel; the message is kept here
      cudaGetLastError();
      set_error(std::string("decode scratch address: ") + cudaGetErrorString(e));
      return nullptr;
    }
    ptrs[dev] = p;
  }
  return ptrs[dev];
}

}  // namespace
}  // namespace sa

extern "C" {

int sa_ultrametric_decode_noalloc(int dtype, int64_t B, int64_t H, int64_t Hkv, int64_t D,
                                  int64_t page_size, int64_t num_pages, const void* q,
                                  const int64_t* q_strides, const void* k_cache,
                                  const int64_t* k_strides, const void* v_cache,
                                  const int64_t* v_strides, const int32_t* block_tables,
                                  const int64_t* bt_strides, int64_t max_logical_pages,
                                  const int32_t* context_lens, const void* router,
                                  int router_dtype, const int64_t* router_strides,
                                  const void* q_router, int q_router_dtype,
                                  const int64_t* q_router_strides, int64_t TD, int64_t req_depth,
                                  int64_t local_blocks, int sink_block, void* out,
                                  const int64_t* out_strides, void* stream) {
  using namespace sa;
  // the scratch address is looked up for the current device, so the stream must be its own
  if (int rc = check_stream_device(stream, "decode_noalloc")) return rc;
  if (H > 0 && Hkv > 0 && D > 0) {
    const int64_t need = sa_ultrametric_decode_workspace_bytes(B, H, Hkv, D, max_logical_pages);
    if (need > kNoAllocScratchBytes)
      return fail(SA_EWORKSPACE, "decode_noalloc: this request needs " + std::to_string(need) +
                                     " bytes of split-K workspace, above the fixed " +
                                     std::to_string(kNoAllocScratchBytes) +
                                     "-byte device array; use sa_ultrametric_decode with a "
                                     "caller-provided workspace");
  }
  void* scratch = decode_scratch_ptr();
  if (!scratch) return fail(SA_ELAUNCH, std::string("decode_noalloc: ") + sa_last_error());
  return sa_ultrametric_decode(dtype, B, H, Hkv, D, page_size, num_pages, q, q_strides, k_cache,
                               k_strides, v_cache, v_strides, block_tables, bt_strides,
                               max_logical_pages, context_lens, router, router_dtype,
                               router_strides, q_router, q_router_dtype, q_router_strides, TD,
                               req_depth, local_blocks, sink_block, out, out_strides, scratch,
                               kNoAllocScratchBytes, stream);
}

}  // extern "C"

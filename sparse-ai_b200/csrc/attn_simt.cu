// CUDA-core (FFMA) block-list attention: the fp32 path (accurate to ~1e-6 relative, which
// tcgen05's fp16/bf16/tf32 inputs cannot reach) and the path for shapes outside the
// tcgen05 kernels (head_dim < 64, route_block < 128).  Same semantics as the tcgen05
// kernels and as src/ultrametric/block_list.py:387-470 (forward), :494-584 (dQ),
// :586-681 (dK/dV) of sparse-ai.
#include <string>

#include "attn_params.cuh"

namespace sa {
namespace {

constexpr int kBM = 16;       // query rows per CTA (<= route_block, which is >= 16)
constexpr int kThreads = 128;  // 4 warps, 4 rows each

template <typename T>
__device__ __forceinline__ float ld(const void* p, int64_t off) {
  return to_f32<T>(static_cast<const T*>(p)[off]);
}

__device__ __forceinline__ float bias_log2(const AttnParams& p, int64_t z, int64_t h, int64_t qb,
                                           int t) {
  if (!p.bias) return 0.f;
  return load_any_f32(p.bias, p.bias_dtype,
                      z * p.bs[0] + h * p.bs[1] + qb * p.bs[2] + (int64_t)t * p.bs[3]) *
         kLog2e;
}

// grid (ceil(N / kBM), Z*H)
template <typename T, int D>
__global__ void __launch_bounds__(kThreads) fwd_simt_kernel(AttnParams p) {
  constexpr int DL = (D + 31) / 32;  // head dims per lane
  extern __shared__ float smem[];
  const int BN = p.RB < 32 ? (int)p.RB : 32;
  float* sQ = smem;                 // [kBM][D]
  float* sK = sQ + kBM * D;         // [32][D + 1]
  float* sV = sK + 32 * (D + 1);    // [32][D]
  const int64_t zh = blockIdx.y, z = zh / p.H, h = zh % p.H;
  const int64_t hk = h / (p.H / p.Hkv);
  const int64_t row0 = (int64_t)blockIdx.x * kBM;
  const int64_t qb = row0 / p.RB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float qk_scale = p.scale * kLog2e;

  for (int i = threadIdx.x; i < kBM * D; i += kThreads) {
    const int64_t r = row0 + i / D;
    sQ[i] = r < p.N ? ld<T>(p.q, z * p.qs[0] + h * p.qs[1] + r * p.qs[2] + (i % D)) : 0.f;
  }
  float m[4], l[4], acc[4][DL];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int e = 0; e < DL; ++e) acc[r][e] = 0.f;
  }
  const int64_t row_id = zh * p.NB + qb;
  const int count = p.counts[row_id];
  const int32_t* lst = p.lists + row_id * p.list_stride;
  for (int t = 0; t < count; ++t) {
    const int64_t kb = lst[t];
    const float b2 = bias_log2(p, z, h, qb, t);
    for (int64_t key0 = kb * p.RB; key0 < (kb + 1) * p.RB; key0 += BN) {
      __syncthreads();
      for (int i = threadIdx.x; i < BN * D; i += kThreads) {
        const int j = i / D, d = i % D;
        const int64_t key = key0 + j;
        const bool ok = key < p.N;
        sK[j * (D + 1) + d] = ok ? ld<T>(p.k, z * p.ks[0] + hk * p.ks[1] + key * p.ks[2] + d) : 0.f;
        sV[j * D + d] = ok ? ld<T>(p.v, z * p.vs[0] + hk * p.vs[1] + key * p.vs[2] + d) : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int rr = warp * 4 + r;
        const int64_t row = row0 + rr;
        const int64_t key = key0 + lane;
        float s = -INFINITY;
        if (lane < BN && key < p.N && (!p.causal || key <= row)) {
          float a = 0.f;
#pragma unroll 8
          for (int d = 0; d < D; ++d) a = fmaf(sQ[rr * D + d], sK[lane * (D + 1) + d], a);
          s = a * qk_scale + b2;
        }
        float mt = s;
#pragma unroll
        for (int o = 16; o; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
        const float m_new = fmaxf(m[r], mt);
        const float m_ref = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = exp2f(m[r] - m_ref);
        const float pj = exp2f(s - m_ref);
        float ps = pj;
#pragma unroll
        for (int o = 16; o; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
        l[r] = l[r] * alpha + ps;
        m[r] = m_new;
#pragma unroll
        for (int e = 0; e < DL; ++e) acc[r][e] *= alpha;
        for (int j = 0; j < BN; ++j) {
          const float pjj = __shfl_sync(0xffffffffu, pj, j);
#pragma unroll
          for (int e = 0; e < DL; ++e) {
            const int d = lane + 32 * e;
            if (d < D) acc[r][e] = fmaf(pjj, sV[j * D + d], acc[r][e]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t row = row0 + warp * 4 + r;
    if (row >= p.N) continue;
    const float inv = 1.f / (l[r] == 0.f ? 1.f : l[r]);
    T* o = static_cast<T*>(p.out) + z * p.os[0] + h * p.os[1] + row * p.os[2];
#pragma unroll
    for (int e = 0; e < DL; ++e) {
      const int d = lane + 32 * e;
      if (d < D) o[d] = from_f32<T>(acc[r][e] * inv);
    }
    if (p.lse && lane == 0) p.lse[zh * p.N + row] = (m[r] + log2f(l[r])) * kLn2;
  }
}

// Delta_i = sum_d dO_i,d * O_i,d in fp32 (block_list.py:785).  One warp per row; the grid
// covers the rows padded to a multiple of 64 so the row-stats array is fully written:
// stats[zh][row / 64] = {lse*log2e (0 for -inf rows, as lse_safe in block_list.py:553),
// Delta}, 64 + 64 floats per 64-row block, zeros for the padding rows.  The tcgen05 dK/dV
// kernel bulk-copies one 512-byte block per 64-row query sub-tile.
template <typename T>
__global__ void delta_kernel(AttnParams p) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t npad = (p.N + 63) / 64 * 64;
  if (gw >= p.Z * p.H * npad) return;
  const int64_t row = gw % npad, zh = gw / npad, z = zh / p.H, h = zh % p.H;
  float a = 0.f, l2 = 0.f;
  if (row < p.N) {
    const T* o = static_cast<const T*>(p.out) + z * p.os[0] + h * p.os[1] + row * p.os[2];
    const T* g = static_cast<const T*>(p.dout) + z * p.dos[0] + h * p.dos[1] + row * p.dos[2];
    for (int64_t d = lane; d < p.D; d += 32) a = fmaf(to_f32<T>(o[d]), to_f32<T>(g[d]), a);
#pragma unroll
    for (int off = 16; off; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
    const float lv = p.lse[zh * p.N + row];
    l2 = lv == -INFINITY ? 0.f : lv * kLog2e;
  }
  if (lane == 0) {
    if (row < p.N) p.delta[zh * p.N + row] = a;
    if (p.stats) {
      float* st = p.stats + (zh * (npad / 64) + row / 64) * 128;
      st[row % 64] = l2;
      st[64 + row % 64] = a;
    }
  }
}

// Vectorised Delta / row stats: LPR lanes per row, 16-byte loads of O and dO; same outputs
// as delta_kernel.  Rows (and their bases) must be 16-byte aligned.
template <typename T, int D>
__global__ void __launch_bounds__(256) delta_vec_kernel(AttnParams p) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int LPR = D / VEC;  // lanes per row (<= 32)
  constexpr int RPW = 32 / LPR;
  const int lane = threadIdx.x & 31;
  const int64_t npad = (p.N + 63) / 64 * 64;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t gr = gw * RPW + lane / LPR;  // padded row index over (Z*H, npad)
  const int li = lane % LPR;
  const bool in_range = gr < p.Z * p.H * npad;
  const int64_t row = in_range ? gr % npad : 0, zh = in_range ? gr / npad : 0;
  const int64_t z = zh / p.H, h = zh % p.H;
  float a = 0.f, l2 = 0.f;
  if (in_range && row < p.N) {
    const uint4 ov = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.out) + z * p.os[0] +
                                                     h * p.os[1] + row * p.os[2] + li * VEC);
    const uint4 gv = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.dout) + z * p.dos[0] +
                                                     h * p.dos[1] + row * p.dos[2] + li * VEC);
    const T* oe = reinterpret_cast<const T*>(&ov);
    const T* ge = reinterpret_cast<const T*>(&gv);
#pragma unroll
    for (int i = 0; i < VEC; ++i) a = fmaf(to_f32<T>(oe[i]), to_f32<T>(ge[i]), a);
  }
#pragma unroll
  for (int off = LPR / 2; off; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
  if (in_range && li == 0) {
    if (row < p.N) {
      const float lv = p.lse[zh * p.N + row];
      l2 = lv == -INFINITY ? 0.f : lv * kLog2e;
      p.delta[zh * p.N + row] = a;
    } else {
      a = 0.f;
    }
    if (p.stats) {
      float* st = p.stats + (zh * (npad / 64) + row / 64) * 128;
      st[row % 64] = l2;
      st[64 + row % 64] = a;
    }
  }
  if (p.dq_acc && in_range && row < p.N) {
    // fused backward: zero this row of the fp32 dQ accumulator
    float4* acc = reinterpret_cast<float4*>(p.dq_acc + (zh * p.N + row) * D) + li * (D / LPR / 4);
#pragma unroll
    for (int i = 0; i < D / LPR / 4; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// dQ over the forward lists (+ soft-bias gradient).  grid (ceil(N / kBM), Z*H).
template <typename T, int D>
__global__ void __launch_bounds__(kThreads) dq_simt_kernel(AttnParams p) {
  constexpr int DL = (D + 31) / 32;
  extern __shared__ float smem[];
  const int BN = p.RB < 32 ? (int)p.RB : 32;
  float* sQ = smem;               // [kBM][D]
  float* sG = sQ + kBM * D;       // dO [kBM][D]
  float* sK = sG + kBM * D;       // [32][D + 1]
  float* sV = sK + 32 * (D + 1);  // [32][D + 1]
  const int64_t zh = blockIdx.y, z = zh / p.H, h = zh % p.H;
  const int64_t hk = h / (p.H / p.Hkv);
  const int64_t row0 = (int64_t)blockIdx.x * kBM;
  const int64_t qb = row0 / p.RB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float qk_scale = p.scale * kLog2e;
  for (int i = threadIdx.x; i < kBM * D; i += kThreads) {
    const int64_t r = row0 + i / D;
    const bool ok = r < p.N;
    sQ[i] = ok ? ld<T>(p.q, z * p.qs[0] + h * p.qs[1] + r * p.qs[2] + (i % D)) : 0.f;
    sG[i] = ok ? ld<T>(p.dout, z * p.dos[0] + h * p.dos[1] + r * p.dos[2] + (i % D)) : 0.f;
  }
  float lse2[4], dl[4], dq[4][DL];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t row = row0 + warp * 4 + r;
    const float lv = row < p.N ? p.lse[zh * p.N + row] : -INFINITY;
    lse2[r] = lv == -INFINITY ? 0.f : lv * kLog2e;
    dl[r] = row < p.N ? p.delta[zh * p.N + row] : 0.f;
#pragma unroll
    for (int e = 0; e < DL; ++e) dq[r][e] = 0.f;
  }
  const int64_t row_id = zh * p.NB + qb;
  const int count = p.counts[row_id];
  const int32_t* lst = p.lists + row_id * p.list_stride;
  for (int t = 0; t < count; ++t) {
    const int64_t kb = lst[t];
    const float b2 = bias_log2(p, z, h, qb, t);
    float db = 0.f;
    for (int64_t key0 = kb * p.RB; key0 < (kb + 1) * p.RB; key0 += BN) {
      __syncthreads();
      for (int i = threadIdx.x; i < BN * D; i += kThreads) {
        const int j = i / D, d = i % D;
        const int64_t key = key0 + j;
        const bool ok = key < p.N;
        sK[j * (D + 1) + d] = ok ? ld<T>(p.k, z * p.ks[0] + hk * p.ks[1] + key * p.ks[2] + d) : 0.f;
        sV[j * (D + 1) + d] = ok ? ld<T>(p.v, z * p.vs[0] + hk * p.vs[1] + key * p.vs[2] + d) : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int rr = warp * 4 + r;
        const int64_t row = row0 + rr;
        const int64_t key = key0 + lane;
        float ds = 0.f;
        if (lane < BN && row < p.N && key < p.N && (!p.causal || key <= row)) {
          float s = 0.f, dp = 0.f;
#pragma unroll 8
          for (int d = 0; d < D; ++d) {
            s = fmaf(sQ[rr * D + d], sK[lane * (D + 1) + d], s);
            dp = fmaf(sG[rr * D + d], sV[lane * (D + 1) + d], dp);
          }
          const float pr = exp2f(s * qk_scale + b2 - lse2[r]);
          ds = pr * (dp - dl[r]);
        }
        db += ds;
        for (int j = 0; j < BN; ++j) {
          const float dsj = __shfl_sync(0xffffffffu, ds, j) * p.scale;
#pragma unroll
          for (int e = 0; e < DL; ++e) {
            const int d = lane + 32 * e;
            if (d < D) dq[r][e] = fmaf(dsj, sK[j * (D + 1) + d], dq[r][e]);
          }
        }
      }
    }
    if (p.dbias) {
#pragma unroll
      for (int o = 16; o; o >>= 1) db += __shfl_xor_sync(0xffffffffu, db, o);
      if (lane == 0) atomicAdd(&p.dbias[row_id * p.list_stride + t], db);
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t row = row0 + warp * 4 + r;
    if (row >= p.N) continue;
    T* o = static_cast<T*>(p.dq) + z * p.dqs[0] + h * p.dqs[1] + row * p.dqs[2];
#pragma unroll
    for (int e = 0; e < DL; ++e) {
      const int d = lane + 32 * e;
      if (d < D) o[d] = from_f32<T>(dq[r][e]);
    }
  }
}

constexpr int kBNK = 16;  // keys per dK/dV CTA (4 per warp)
constexpr int kBMQ = 32;  // query rows per inner step (one per lane)

// dK, dV over the transposed lists; one CTA per (key tile, z, KV head) accumulates over every
// query head of the GQA group.  grid (ceil(N / kBNK), Z*Hkv).
template <typename T, int D>
__global__ void __launch_bounds__(kThreads) dkdv_simt_kernel(AttnParams p) {
  constexpr int DL = (D + 31) / 32;
  extern __shared__ float smem[];
  float* sQ = smem;                 // [kBMQ][D + 1]
  float* sG = sQ + kBMQ * (D + 1);  // dO [kBMQ][D + 1]
  float* sK = sG + kBMQ * (D + 1);  // [kBNK][D]
  float* sV = sK + kBNK * D;        // [kBNK][D]
  float* sL = sV + kBNK * D;        // lse*log2e [kBMQ]
  float* sDl = sL + kBMQ;           // delta [kBMQ]
  const int64_t zg = blockIdx.y, z = zg / p.Hkv, hk = zg % p.Hkv;
  const int64_t group = p.H / p.Hkv;
  const int64_t key0 = (int64_t)blockIdx.x * kBNK;
  const int64_t kb = key0 / p.RB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float qk_scale = p.scale * kLog2e;
  const int rows_step = p.RB < kBMQ ? (int)p.RB : kBMQ;
  for (int i = threadIdx.x; i < kBNK * D; i += kThreads) {
    const int64_t key = key0 + i / D;
    const bool ok = key < p.N;
    sK[i] = ok ? ld<T>(p.k, z * p.ks[0] + hk * p.ks[1] + key * p.ks[2] + (i % D)) : 0.f;
    sV[i] = ok ? ld<T>(p.v, z * p.vs[0] + hk * p.vs[1] + key * p.vs[2] + (i % D)) : 0.f;
  }
  float dk[4][DL], dv[4][DL];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int e = 0; e < DL; ++e) dk[c][e] = dv[c][e] = 0.f;
  for (int64_t h = hk * group; h < (hk + 1) * group; ++h) {
    const int64_t zh = z * p.H + h;
    const int64_t krow = zh * p.NB + kb;
    const int qcount = p.q_counts[krow];
    for (int j = 0; j < qcount; ++j) {
      const int64_t qb = p.k_lists[krow * p.NB + j];
      const int slot = p.k_slots[krow * p.NB + j];
      const float b2 = bias_log2(p, z, h, qb, slot);
      for (int64_t r0 = qb * p.RB; r0 < (qb + 1) * p.RB; r0 += rows_step) {
        __syncthreads();
        for (int i = threadIdx.x; i < rows_step * D; i += kThreads) {
          const int64_t r = r0 + i / D;
          const int d = i % D;
          const bool ok = r < p.N;
          sQ[(i / D) * (D + 1) + d] = ok ? ld<T>(p.q, z * p.qs[0] + h * p.qs[1] + r * p.qs[2] + d) : 0.f;
          sG[(i / D) * (D + 1) + d] =
              ok ? ld<T>(p.dout, z * p.dos[0] + h * p.dos[1] + r * p.dos[2] + d) : 0.f;
        }
        for (int i = threadIdx.x; i < rows_step; i += kThreads) {
          const int64_t r = r0 + i;
          const float lv = r < p.N ? p.lse[zh * p.N + r] : -INFINITY;
          sL[i] = lv == -INFINITY ? 0.f : lv * kLog2e;
          sDl[i] = r < p.N ? p.delta[zh * p.N + r] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int kk = warp * 4 + c;
          const int64_t key = key0 + kk;
          const int64_t row = r0 + lane;
          float pr = 0.f, ds = 0.f;
          if (lane < rows_step && row < p.N && key < p.N && (!p.causal || key <= row)) {
            float s = 0.f, dp = 0.f;
#pragma unroll 8
            for (int d = 0; d < D; ++d) {
              s = fmaf(sQ[lane * (D + 1) + d], sK[kk * D + d], s);
              dp = fmaf(sG[lane * (D + 1) + d], sV[kk * D + d], dp);
            }
            pr = exp2f(s * qk_scale + b2 - sL[lane]);
            ds = pr * (dp - sDl[lane]) * p.scale;
          }
          for (int i = 0; i < rows_step; ++i) {
            const float pi = __shfl_sync(0xffffffffu, pr, i);
            const float dsi = __shfl_sync(0xffffffffu, ds, i);
#pragma unroll
            for (int e = 0; e < DL; ++e) {
              const int d = lane + 32 * e;
              if (d < D) {
                dv[c][e] = fmaf(pi, sG[i * (D + 1) + d], dv[c][e]);
                dk[c][e] = fmaf(dsi, sQ[i * (D + 1) + d], dk[c][e]);
              }
            }
          }
        }
      }
    }
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int64_t key = key0 + warp * 4 + c;
    if (key >= p.N) continue;
    T* ok = static_cast<T*>(p.dk) + z * p.dks[0] + hk * p.dks[1] + key * p.dks[2];
    T* ov = static_cast<T*>(p.dv) + z * p.dvs[0] + hk * p.dvs[1] + key * p.dvs[2];
#pragma unroll
    for (int e = 0; e < DL; ++e) {
      const int d = lane + 32 * e;
      if (d < D) {
        ok[d] = from_f32<T>(dk[c][e]);
        ov[d] = from_f32<T>(dv[c][e]);
      }
    }
  }
}

template <typename T, int D>
int launch_fwd_t(const AttnParams& p, cudaStream_t s) {
  const size_t smem = (size_t)(kBM * D + 32 * (D + 1) + 32 * D) * sizeof(float);
  auto kern = fwd_simt_kernel<T, D>;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((unsigned)((p.N + kBM - 1) / kBM), (unsigned)(p.Z * p.H));
  kern<<<grid, kThreads, smem, s>>>(p);
  return check_launch("fwd_simt_kernel");
}

template <typename T, int D>
int launch_bwd_t(const AttnParams& p, cudaStream_t s, int parts) {
  if (parts & kBwdDq) {
    const size_t smem = (size_t)(2 * kBM * D + 2 * 32 * (D + 1)) * sizeof(float);
    auto kern = dq_simt_kernel<T, D>;
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dim3 grid((unsigned)((p.N + kBM - 1) / kBM), (unsigned)(p.Z * p.H));
    kern<<<grid, kThreads, smem, s>>>(p);
    int rc = check_launch("dq_simt_kernel");
    if (rc) return rc;
  }
  if (parts & kBwdDkDv) {
    const size_t smem = (size_t)(2 * kBMQ * (D + 1) + 2 * kBNK * D + 2 * kBMQ) * sizeof(float);
    auto kern = dkdv_simt_kernel<T, D>;
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dim3 grid((unsigned)((p.N + kBNK - 1) / kBNK), (unsigned)(p.Z * p.Hkv));
    kern<<<grid, kThreads, smem, s>>>(p);
    return check_launch("dkdv_simt_kernel");
  }
  return SA_OK;
}

template <typename T>
int dispatch_fwd(const AttnParams& p, cudaStream_t s) {
  switch (p.D) {
    case 16: return launch_fwd_t<T, 16>(p, s);
    case 32: return launch_fwd_t<T, 32>(p, s);
    case 64: return launch_fwd_t<T, 64>(p, s);
    case 128: return launch_fwd_t<T, 128>(p, s);
    case 256: return launch_fwd_t<T, 256>(p, s);
  }
  return fail(SA_EUNSUPPORTED, "head_dim " + std::to_string(p.D) + " not in {16,32,64,128,256}");
}

template <typename T>
int dispatch_bwd(const AttnParams& p, cudaStream_t s, int parts) {
  switch (p.D) {
    case 16: return launch_bwd_t<T, 16>(p, s, parts);
    case 32: return launch_bwd_t<T, 32>(p, s, parts);
    case 64: return launch_bwd_t<T, 64>(p, s, parts);
    case 128: return launch_bwd_t<T, 128>(p, s, parts);
    case 256: return launch_bwd_t<T, 256>(p, s, parts);
  }
  return fail(SA_EUNSUPPORTED, "head_dim " + std::to_string(p.D) + " not in {16,32,64,128,256}");
}

}  // namespace

int launch_fwd_simt(const AttnParams& p, cudaStream_t s) {
  if (p.N == 0 || p.Z * p.H == 0) return SA_OK;
  switch (p.dtype) {
    case SA_F32: return dispatch_fwd<float>(p, s);
    case SA_F16: return dispatch_fwd<__half>(p, s);
    case SA_BF16: return dispatch_fwd<__nv_bfloat16>(p, s);
  }
  return fail(SA_EUNSUPPORTED, "dtype");
}

int launch_bwd_simt(const AttnParams& p, cudaStream_t s, int parts) {
  if (p.N == 0 || p.Z * p.H == 0) return SA_OK;
  switch (p.dtype) {
    case SA_F32: return dispatch_bwd<float>(p, s, parts);
    case SA_F16: return dispatch_bwd<__half>(p, s, parts);
    case SA_BF16: return dispatch_bwd<__nv_bfloat16>(p, s, parts);
  }
  return fail(SA_EUNSUPPORTED, "dtype");
}

template <typename T, int D>
int launch_delta_vec(const AttnParams& p, cudaStream_t s, int64_t rows) {
  constexpr int RPW = 32 / (D / (16 / (int)sizeof(T)));
  const int64_t warps = (rows + RPW - 1) / RPW;
  delta_vec_kernel<T, D><<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(p);
  return check_launch("delta_vec_kernel");
}

int launch_delta(const AttnParams& p, cudaStream_t s) {
  const int64_t rows = p.Z * p.H * ((p.N + 63) / 64 * 64);
  if (rows == 0) return SA_OK;
  const int esz = p.dtype == SA_F32 ? 4 : 2;
  bool vec = reinterpret_cast<uintptr_t>(p.out) % 16 == 0 &&
             reinterpret_cast<uintptr_t>(p.dout) % 16 == 0;
  for (int i = 0; i < 3; ++i) vec = vec && (p.os[i] * esz) % 16 == 0 && (p.dos[i] * esz) % 16 == 0;
  if (vec && p.dtype != SA_F32 && (p.D == 64 || p.D == 128)) {
    const bool bf = p.dtype == SA_BF16;
    if (p.D == 128) return bf ? launch_delta_vec<__nv_bfloat16, 128>(p, s, rows)
                              : launch_delta_vec<__half, 128>(p, s, rows);
    return bf ? launch_delta_vec<__nv_bfloat16, 64>(p, s, rows) : launch_delta_vec<__half, 64>(p, s, rows);
  }
  const int threads = 256;
  const int64_t blocks = (rows * 32 + threads - 1) / threads;
  switch (p.dtype) {
    case SA_F32: delta_kernel<float><<<(unsigned)blocks, threads, 0, s>>>(p); break;
    case SA_F16: delta_kernel<__half><<<(unsigned)blocks, threads, 0, s>>>(p); break;
    case SA_BF16: delta_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, s>>>(p); break;
    default: return fail(SA_EUNSUPPORTED, "dtype");
  }
  return check_launch("delta_kernel");
}

}  // namespace sa

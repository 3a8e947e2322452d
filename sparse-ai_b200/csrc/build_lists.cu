// Block-list compaction kernels: routing vectors -> ascending per-row key-block lists, and
// the transposition key block -> query blocks (with the forward slot of each pair).
//
// Integer work, HBM/latency bound: one warp per output row, 32 candidate columns per
// ballot, the row's codes staged once per CTA in shared memory.
#include <string>

#include "common.cuh"

namespace sa {
namespace {

constexpr int kBuildThreads = 256;
constexpr int kBuildRowsPerCta = 32;

struct BuildParams {
  const void* router;
  int router_dtype;
  int64_t rs[4];
  int64_t H, NB, TD;
  const int32_t* depth;
  uint64_t base;
  int use_codes, is_causal, sink_block;
  int64_t local_blocks;
  int32_t* lists;
  int64_t list_stride;
  int32_t* counts;
};

// Mixed-radix prefix code sum_{l<d} r_l * base^l in wrapping 64-bit arithmetic
// (src/ultrametric/block_list.py:224-229 computes it in torch int64, which wraps the same way).
__device__ __forceinline__ uint64_t prefix_code(const BuildParams& p, int64_t off, int d) {
  uint64_t code = 0, pw = 1;
  for (int l = 0; l < d; ++l) {
    code += (uint64_t)load_any_i64(p.router, p.router_dtype, off + l * p.rs[3]) * pw;
    pw *= p.base;
  }
  return code;
}

__device__ __forceinline__ bool levels_equal(const BuildParams& p, int64_t oa, int64_t ob, int d) {
  for (int l = 0; l < d; ++l)
    if (load_any_i64(p.router, p.router_dtype, oa + l * p.rs[3]) !=
        load_any_i64(p.router, p.router_dtype, ob + l * p.rs[3]))
      return false;
  return true;
}

// grid (ceil(NB / kBuildRowsPerCta), Z*H); the rule of block_list.py:37-38,107-118,149-156:
// match = equal prefix OR |i-j| <= local OR (sink and j == 0); AND j <= i when causal.
__global__ void __launch_bounds__(kBuildThreads) build_lists_kernel(BuildParams p) {
  extern __shared__ uint64_t s_codes[];
  // launched as a programmatic dependent (after the route vote), the routes are complete
  // only past this point; otherwise a no-op
  pdl_wait();
  const int64_t zh = blockIdx.y;
  const int64_t z = zh / p.H, h = zh % p.H;
  const int d = p.depth[h];
  const int64_t rbase = z * p.rs[0] + h * p.rs[1];
  if (p.use_codes) {
    for (int64_t j = threadIdx.x; j < p.NB; j += blockDim.x)
      s_codes[j] = prefix_code(p, rbase + j * p.rs[2], d);
    __syncthreads();
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row0 = (int64_t)blockIdx.x * kBuildRowsPerCta;
  for (int64_t i = row0 + warp; i < min(row0 + kBuildRowsPerCta, p.NB);
       i += kBuildThreads / 32) {
    const uint64_t qcode = p.use_codes ? s_codes[i] : 0;
    const int64_t qoff = rbase + i * p.rs[2];
    int32_t* lrow = p.lists + (zh * p.NB + i) * p.list_stride;
    int count = 0;
    const int64_t jend = p.is_causal ? i + 1 : p.NB;
    for (int64_t j0 = 0; j0 < jend; j0 += 32) {
      const int64_t j = j0 + lane;
      bool m = false;
      if (j < jend) {
        m = p.use_codes ? (s_codes[j] == qcode) : levels_equal(p, qoff, rbase + j * p.rs[2], d);
        const int64_t diff = i > j ? i - j : j - i;
        if (p.local_blocks > 0 && diff <= p.local_blocks) m = true;
        if (p.sink_block && j == 0) m = true;
      }
      const unsigned ball = __ballot_sync(0xffffffffu, m);
      const int pos = count + __popc(ball & ((1u << lane) - 1u));
      if (m && pos < p.list_stride) lrow[pos] = (int32_t)j;
      count += __popc(ball);
    }
    for (int64_t s = count + lane; s < p.list_stride; s += 32) lrow[s] = 0;
    if (lane == 0) p.counts[zh * p.NB + i] = count;
  }
}

constexpr int kTransRows = 8;  // key-block rows per CTA in the transposition

struct TransParams {
  const int32_t* lists;
  int64_t list_stride;
  const int32_t* counts;
  int64_t NBQ, NBK;
  int32_t* k_lists;
  int64_t k_list_stride;
  int32_t* q_counts;
  int32_t* k_slots;
  int pad;
};

// grid (ceil(NBK / kTransRows), ZH).  Phase 1 scatters every (qb, t) entry whose key block
// falls in this CTA's rows into a shared slot table (-1 = absent; the largest t wins on
// duplicates, as the last match wins in block_list.py:647-650).  Phase 2 compacts each
// key-block row ascending over qb (block_list.py:305-325).
__global__ void __launch_bounds__(256) transpose_lists_kernel(TransParams p) {
  extern __shared__ int32_t s_slot[];  // [kTransRows][NBQ]
  const int64_t zh = blockIdx.y;
  const int64_t kb0 = (int64_t)blockIdx.x * kTransRows;
  const int64_t nrows = min((int64_t)kTransRows, p.NBK - kb0);
  for (int64_t i = threadIdx.x; i < nrows * p.NBQ; i += blockDim.x) s_slot[i] = -1;
  __syncthreads();
  const int32_t* cnt = p.counts + zh * p.NBQ;
  const int32_t* lst = p.lists + zh * p.NBQ * p.list_stride;
  for (int64_t qb = threadIdx.x >> 5; qb < p.NBQ; qb += blockDim.x >> 5) {
    const int c = min((int64_t)cnt[qb], p.list_stride);
    for (int t = threadIdx.x & 31; t < c; t += 32) {
      const int64_t kb = lst[qb * p.list_stride + t];
      if (kb >= kb0 && kb < kb0 + nrows) atomicMax(&s_slot[(kb - kb0) * p.NBQ + qb], t);
    }
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < nrows; r += blockDim.x >> 5) {
    const int64_t kb = kb0 + r;
    int32_t* krow = p.k_lists + (zh * p.NBK + kb) * p.k_list_stride;
    int32_t* srow = p.k_slots ? p.k_slots + (zh * p.NBK + kb) * p.k_list_stride : nullptr;
    int count = 0;
    for (int64_t q0 = 0; q0 < p.NBQ; q0 += 32) {
      const int64_t qb = q0 + lane;
      const int slot = qb < p.NBQ ? s_slot[r * p.NBQ + qb] : -1;
      const bool m = slot >= 0;
      const unsigned ball = __ballot_sync(0xffffffffu, m);
      const int pos = count + __popc(ball & ((1u << lane) - 1u));
      if (m && pos < p.k_list_stride) {
        krow[pos] = (int32_t)qb;
        if (srow) srow[pos] = slot;
      }
      count += __popc(ball);
    }
    if (p.pad) {
      for (int64_t s = count + lane; s < p.k_list_stride; s += 32) {
        krow[s] = 0;
        if (srow) srow[s] = 0;
      }
    }
    if (lane == 0) p.q_counts[zh * p.NBK + kb] = count;
  }
}

}  // namespace

int launch_transpose_lists(const int32_t* lists, int64_t list_stride, const int32_t* counts,
                           int64_t ZH, int64_t NBQ, int64_t NBK, int32_t* k_lists,
                           int64_t k_list_stride, int32_t* q_counts, int32_t* k_slots, int pad,
                           cudaStream_t stream) {
  if (ZH <= 0 || NBK <= 0) return SA_OK;
  const size_t smem = (size_t)kTransRows * NBQ * sizeof(int32_t);
  if (smem > 200 * 1024)
    return fail(SA_EUNSUPPORTED, "transposed lists: too many query blocks (" +
                                     std::to_string(NBQ) + ") for the shared slot table");
  TransParams p{lists, list_stride, counts, NBQ, NBK, k_lists, k_list_stride, q_counts, k_slots, pad};
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(transpose_lists_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  dim3 grid((unsigned)((NBK + kTransRows - 1) / kTransRows), (unsigned)ZH);
  transpose_lists_kernel<<<grid, 256, smem, stream>>>(p);
  return check_launch("transpose_lists_kernel");
}

int launch_build_lists(const void* router, int router_dtype, const int64_t* router_strides,
                       int64_t Z, int64_t H, int64_t NB, int64_t TD, const int32_t* req_depth,
                       int64_t base, int use_codes, int is_causal, int sink_block,
                       int64_t local_blocks, int32_t* lists, int64_t list_stride,
                       int32_t* counts, cudaStream_t stream, bool dependent) {
  if (list_stride < 1) return fail(SA_EINVAL, "list_stride must be >= 1");
  if (use_codes && NB > 16384)
    return fail(SA_EUNSUPPORTED, "more than 16384 route blocks per head");
  if (Z * H > 65535) return fail(SA_EUNSUPPORTED, "Z*H exceeds 65535");
  BuildParams p{};
  p.router = router;
  p.router_dtype = router_dtype;
  for (int i = 0; i < 4; ++i) p.rs[i] = router_strides[i];
  p.H = H;
  p.NB = NB;
  p.TD = TD;
  p.depth = req_depth;
  p.base = (uint64_t)base;
  p.use_codes = use_codes;
  p.is_causal = is_causal;
  p.sink_block = sink_block;
  p.local_blocks = local_blocks;
  p.lists = lists;
  p.list_stride = list_stride;
  p.counts = counts;
  const size_t smem = use_codes ? (size_t)NB * sizeof(uint64_t) : 0;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(build_lists_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  dim3 grid((unsigned)((NB + kBuildRowsPerCta - 1) / kBuildRowsPerCta), (unsigned)(Z * H));
  if (dependent)
    return launch_dependent(build_lists_kernel, grid, dim3(kBuildThreads), smem, stream,
                            "build_lists_kernel", p);
  build_lists_kernel<<<grid, kBuildThreads, smem, stream>>>(p);
  return check_launch("build_lists_kernel");
}

}  // namespace sa

extern "C" {

int sa_build_block_lists(const void* router, int router_dtype, const int64_t* router_strides,
                         int64_t Z, int64_t H, int64_t NB, int64_t TD, const int32_t* req_depth,
                         int64_t base, int use_codes, int is_causal, int sink_block,
                         int64_t local_blocks, int32_t* lists, int64_t list_stride,
                         int32_t* counts, void* stream) {
  using namespace sa;
  if (Z < 0 || H < 0 || NB < 0 || TD < 0) return fail(SA_EINVAL, "negative size");
  if (Z * H * NB == 0) return SA_OK;
  if (!router || !req_depth || !lists || !counts || !router_strides)
    return fail(SA_EINVAL, "null pointer argument");
  if (router_dtype != SA_I32 && router_dtype != SA_I64)
    return fail(SA_EUNSUPPORTED, "router_indices must be int32 or int64");
  return launch_build_lists(router, router_dtype, router_strides, Z, H, NB, TD, req_depth, base,
                            use_codes, is_causal, sink_block, local_blocks, lists, list_stride,
                            counts, (cudaStream_t)stream, false);
}

int sa_build_transposed_block_lists(const int32_t* lists, int64_t list_stride,
                                    const int32_t* counts, int64_t ZH, int64_t NBQ, int64_t NBK,
                                    int32_t* k_lists, int64_t k_list_stride, int32_t* q_counts,
                                    int32_t* k_slots, void* stream) {
  using namespace sa;
  if (ZH < 0 || NBQ < 0 || NBK < 0) return fail(SA_EINVAL, "negative size");
  if (ZH * NBK == 0) return SA_OK;
  if (!k_lists || !q_counts || (NBQ > 0 && (!lists || !counts)))
    return fail(SA_EINVAL, "null pointer argument");
  if (k_list_stride < 1 || list_stride < 0) return fail(SA_EINVAL, "bad list stride");
  if (ZH > 65535) return fail(SA_EUNSUPPORTED, "Z*H exceeds 65535");
  return launch_transpose_lists(lists, list_stride, counts, ZH, NBQ, NBK, k_lists, k_list_stride,
                                q_counts, k_slots, 1, (cudaStream_t)stream);
}

}  // extern "C"

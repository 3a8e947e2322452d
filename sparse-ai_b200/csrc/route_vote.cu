// Surgery routing -> block lists in one C-ABI call (no torch glue in between):
//
//   1. route_vote_kernel: per route block, the per-level branch of its tokens' router
//      outputs by majority vote (src/llama_surgery/surgery.py:543-547 of sparse-ai:
//      token argmax over the p branches, one-hot votes summed over the block, argmax of the
//      votes, ties to the lowest branch id; tokens past S do not vote).  With one token per
//      block (the router already ran on pooled block descriptors, surgery.py:533-538) the
//      vote is that token's argmax.  Writes block_route (Z, H, NB, r) int32.
//   2. build_lists_kernel (build_lists.cu), launched as the vote kernel's programmatic
//      dependent: prefix codes of the first depth[h] levels and the ascending compaction,
//      exactly as sa_build_block_lists.
//
// Two launches, because the compaction of query block i needs the votes of every key
// block j <= i, a grid-wide dependency; programmatic dependent launch lets the second
// kernel's launch overlap the first one's tail.  Integer / byte work, HBM-bound on the
// router outputs (Z*H*S*r*p elements read once).
#include <cmath>
#include <string>

#include "common.cuh"

namespace sa {

int launch_build_lists(const void* router, int router_dtype, const int64_t* router_strides,
                       int64_t Z, int64_t H, int64_t NB, int64_t TD, const int32_t* req_depth,
                       int64_t base, int use_codes, int is_causal, int sink_block,
                       int64_t local_blocks, int32_t* lists, int64_t list_stride,
                       int32_t* counts, cudaStream_t stream, bool dependent);

namespace {

constexpr int kVoteThreads = 128;
constexpr int kMaxVoteLevels = 32;
constexpr int kMaxBranches = 16;

struct VoteParams {
  const void* a;
  int dtype;
  int64_t as[5];  // element strides of (Z, H, S, levels, p)
  int64_t H, S, T, NB;
  int r, P;
  int32_t* route;  // (Z, H, NB, r) contiguous
};

// argmax over the p branches of one (token, level): first maximum wins, and a NaN counts as
// the maximum (torch.argmax semantics).
__device__ __forceinline__ int branch_argmax(const VoteParams& p, int64_t off) {
  float best = load_any_f32(p.a, p.dtype, off);
  int arg = 0;
  for (int c = 1; c < p.P; ++c) {
    const float x = load_any_f32(p.a, p.dtype, off + c * p.as[4]);
    if (!isnan(best) && (x > best || isnan(x))) {
      best = x;
      arg = c;
    }
  }
  return arg;
}

// grid (NB, Z*H): one CTA per route block; thread = token, warp ballots per (level, branch).
__global__ void __launch_bounds__(kVoteThreads) route_vote_kernel(VoteParams p) {
  __shared__ unsigned s_cnt[kMaxVoteLevels * kMaxBranches];
  const int64_t zh = blockIdx.y, b = blockIdx.x;
  const int64_t z = zh / p.H, h = zh % p.H;
  for (int i = threadIdx.x; i < p.r * p.P; i += blockDim.x) s_cnt[i] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t t0 = b * p.T;
  const int64_t t1 = min(t0 + p.T, p.S);
  const int64_t base = z * p.as[0] + h * p.as[1];
  // every warp runs the same number of iterations, so the ballots stay warp-uniform
  for (int64_t tb = t0; tb < t0 + p.T; tb += blockDim.x) {
    const int64_t t = tb + threadIdx.x;
    const bool valid = t < t1;
    for (int l = 0; l < p.r; ++l) {
      const int c_mine = valid ? branch_argmax(p, base + t * p.as[2] + l * p.as[3]) : -1;
      for (int c = 0; c < p.P; ++c) {
        const unsigned bal = __ballot_sync(0xffffffffu, c_mine == c);
        if (lane == 0 && bal) atomicAdd(&s_cnt[l * p.P + c], __popc(bal));
      }
    }
  }
  __syncthreads();
  for (int l = threadIdx.x; l < p.r; l += blockDim.x) {
    unsigned best = s_cnt[l * p.P];
    int arg = 0;
    for (int c = 1; c < p.P; ++c) {
      const unsigned n = s_cnt[l * p.P + c];
      if (n > best) {
        best = n;
        arg = c;
      }
    }
    p.route[(zh * p.NB + b) * p.r + l] = arg;
  }
  // let the dependent compaction launch while the last vote CTAs finish
  pdl_trigger();
}

}  // namespace
}  // namespace sa

extern "C" {

int sa_build_block_lists_from_assignments(const void* assignments, int dtype,
                                          const int64_t* strides, int64_t Z, int64_t H, int64_t S,
                                          int64_t levels, int64_t num_branches,
                                          int64_t tokens_per_block, int64_t r,
                                          const int32_t* req_depth, int64_t arity, int is_causal,
                                          int sink_block, int64_t local_blocks,
                                          int32_t* block_route, int32_t* lists,
                                          int64_t list_stride, int32_t* counts, void* stream) {
  using namespace sa;
  if (Z < 0 || H < 0 || S < 0) return fail(SA_EINVAL, "negative size");
  if (tokens_per_block < 1) return fail(SA_EINVAL, "tokens_per_block must be >= 1");
  if (num_branches < 1 || num_branches > kMaxBranches)
    return fail(SA_EUNSUPPORTED, "number of branches must be in [1, 16]");
  if (r < 0 || r > levels || r > kMaxVoteLevels)
    return fail(SA_EINVAL, "r must be in [0, min(levels, 32)]");
  if (dtype != SA_F32 && dtype != SA_F16 && dtype != SA_BF16)
    return fail(SA_EUNSUPPORTED, "assignments must be fp32, fp16 or bf16");
  const int64_t NB = (S + tokens_per_block - 1) / tokens_per_block;
  if (Z * H * NB == 0) return SA_OK;
  if (!assignments || !strides || !req_depth || !block_route || !lists || !counts)
    return fail(SA_EINVAL, "null pointer argument");
  if (list_stride < 1) return fail(SA_EINVAL, "list_stride must be >= 1");
  if (Z * H > 65535) return fail(SA_EUNSUPPORTED, "Z*H exceeds 65535");
  if (NB > 16384) return fail(SA_EUNSUPPORTED, "more than 16384 route blocks per head");
  if (int rc = check_stream_device(stream, "build_block_lists_from_assignments")) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t base = arity > 2 ? arity : 2;
  if (r > 0) {
    VoteParams p{};
    p.a = assignments;
    p.dtype = dtype;
    for (int i = 0; i < 5; ++i) p.as[i] = strides[i];
    p.H = H;
    p.S = S;
    p.T = tokens_per_block;
    p.NB = NB;
    p.r = (int)r;
    p.P = (int)num_branches;
    p.route = block_route;
    route_vote_kernel<<<dim3((unsigned)NB, (unsigned)(Z * H)), kVoteThreads, 0, s>>>(p);
    if (int rc = check_launch("route_vote_kernel")) return rc;
  }
  // codes fit in 62 bits: compare codes; otherwise compare level by level
  // (block_list.py:226,256-258 of the reference)
  const int use_codes = (double)r * std::log2((double)base) < 62.0 ? 1 : 0;
  const int64_t rs[4] = {H * NB * r, NB * r, r, 1};
  return launch_build_lists(block_route, SA_I32, rs, Z, H, NB, r > 0 ? r : 1, req_depth, base,
                            use_codes, is_causal, sink_block, local_blocks, lists, list_stride,
                            counts, s, r > 0);
}

}  // extern "C"

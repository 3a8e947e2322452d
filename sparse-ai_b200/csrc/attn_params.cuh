// Argument bundle shared by the block-list attention kernels (forward and backward).
#pragma once

#include "common.cuh"

namespace sa {

struct AttnParams {
  int dtype;
  int64_t Z, H, Hkv, N, D, RB, NB;
  const void* q;
  int64_t qs[4];
  const void* k;
  int64_t ks[4];
  const void* v;
  int64_t vs[4];
  void* out;
  int64_t os[4];
  float* lse;  // (Z, H, N) contiguous or null
  const int32_t* lists;
  int64_t list_stride;
  const int32_t* counts;
  const void* bias;  // (Z, H, NB, list_stride) with bs strides, or null
  int bias_dtype;
  int64_t bs[4];
  int causal;
  float scale;
  int accumulate;  // forward: continue from the output / LSE already in out / lse
  // backward only
  const void* dout;
  int64_t dos[4];
  float* delta;  // (Z, H, N) fp32 workspace
  float* stats;  // (Z*H, ceil(N/64), {lse*log2e[64], delta[64]}) fp32 workspace
  const int32_t* k_lists;  // transposed lists (Z, H, NB, NB) + slots
  const int32_t* k_slots;
  const int32_t* q_counts;
  void* dq;
  int64_t dqs[4];
  void* dk;
  int64_t dks[4];
  void* dv;
  int64_t dvs[4];
  float* dbias;  // (Z, H, NB, list_stride) contiguous fp32, or null
  // fused backward: fp32 dQ accumulator (Z*H, N, D) contiguous (null on the two-kernel path)
  float* dq_acc;
  unsigned* status;
  // planner workspaces of the tcgen05 kernels (null: static round-robin scheduling)
  void* plan_fwd;
  void* plan_dq;
  void* plan_dkdv;
};

// backward parts (bitmask): the dQ and dK/dV kernels, or the fused single-pass kernel
constexpr int kBwdDq = 1, kBwdDkDv = 2, kBwdFused = 4;

int launch_fwd_simt(const AttnParams& p, cudaStream_t stream);
int launch_bwd_simt(const AttnParams& p, cudaStream_t stream, int parts);
int launch_delta(const AttnParams& p, cudaStream_t stream);
int launch_transpose_lists(const int32_t* lists, int64_t list_stride, const int32_t* counts,
                           int64_t ZH, int64_t NBQ, int64_t NBK, int32_t* k_lists,
                           int64_t k_list_stride, int32_t* q_counts, int32_t* k_slots, int pad,
                           cudaStream_t stream);
// The fused backward takes bf16/fp16, head_dim 128, route_block a multiple of 128.
bool bwd_fused_eligible(const AttnParams& p);
// tcgen05 kernels: return SA_EUNSUPPORTED (without launching) for shapes they do not take.
int launch_fwd_sm100(const AttnParams& p, cudaStream_t stream);
int launch_bwd_sm100(const AttnParams& p, cudaStream_t stream, int parts);
// Planner workspaces (bytes) of the tcgen05 kernels for these sizes on the current device,
// and the plan launches of the backward (run after the transposed lists exist).
int64_t fwd_plan_bytes(int64_t Z, int64_t H, int64_t N, int64_t D);
int64_t bwd_plan_bytes(int which, int64_t Z, int64_t H, int64_t Hkv, int64_t N, int64_t D);
// Work queues of the tcgen05 dQ (kBwdDq: needs the forward counts) and dK/dV (kBwdDkDv:
// needs the transposed counts) kernels.
int plan_bwd_sm100(const AttnParams& p, cudaStream_t stream, int which);

}  // namespace sa

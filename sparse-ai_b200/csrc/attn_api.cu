// C-ABI entry points of the block-list attention forward and backward: argument checks,
// workspace carving, and dispatch to the tcgen05 kernels (bf16/fp16, head_dim 64/128,
// route_block a multiple of 128) or to the CUDA-core kernels (everything else, fp32).
#include <string>

#include "attn_plan.cuh"

namespace sa {
namespace {

int fill_common(AttnParams& p, int dtype, int64_t Z, int64_t H, int64_t Hkv, int64_t N, int64_t D,
                int64_t RB, const void* q, const int64_t* qs, const void* k, const int64_t* ks,
                const void* v, const int64_t* vs, const int32_t* lists, int64_t list_stride,
                const int32_t* counts, const void* bias, int bias_dtype, const int64_t* bs,
                int causal, float scale) {
  if (Z < 0 || H <= 0 || Hkv <= 0 || N < 0) return fail(SA_EINVAL, "bad sizes");
  if (H % Hkv) return fail(SA_EINVAL, "num_heads must be a multiple of the K/V heads");
  if (D < 16 || (D & (D - 1))) return fail(SA_EINVAL, "head_dim must be a power of two >= 16");
  if (RB < 16 || (RB & (RB - 1))) return fail(SA_EINVAL, "route_block must be a power of two >= 16");
  if (dtype != SA_F32 && dtype != SA_F16 && dtype != SA_BF16)
    return fail(SA_EUNSUPPORTED, "dtype must be fp32, fp16 or bf16");
  if (!qs || !ks || !vs) return fail(SA_EINVAL, "null stride array");
  if (qs[3] != 1 || ks[3] != 1 || vs[3] != 1)
    return fail(SA_EUNSUPPORTED, "head_dim must be the contiguous dimension");
  if (list_stride < 0) return fail(SA_EINVAL, "negative list stride");
  if (bias && (bias_dtype < SA_F32 || bias_dtype > SA_BF16 || !bs))
    return fail(SA_EINVAL, "soft_block_bias must be a float tensor with strides");
  p.dtype = dtype;
  p.Z = Z;
  p.H = H;
  p.Hkv = Hkv;
  p.N = N;
  p.D = D;
  p.RB = RB;
  p.NB = (N + RB - 1) / RB;
  p.q = q;
  p.k = k;
  p.v = v;
  for (int i = 0; i < 4; ++i) {
    p.qs[i] = qs[i];
    p.ks[i] = ks[i];
    p.vs[i] = vs[i];
    p.bs[i] = bias ? bs[i] : 0;
  }
  p.lists = lists;
  p.list_stride = list_stride;
  p.counts = counts;
  p.bias = bias;
  p.bias_dtype = bias_dtype;
  p.causal = causal;
  p.scale = scale;
  p.status = device_status_ptr();
  if (!p.status) return fail(SA_ELAUNCH, std::string("attention: ") + sa_last_error());
  if (Z * H > 65535) return fail(SA_EUNSUPPORTED, "Z*H exceeds 65535");
  return SA_OK;
}

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

// Shapes the fused single-pass backward can take (dtype and alignment are checked at launch);
// their workspace carries its fp32 dQ accumulator.
bool fused_shape(int64_t D, int64_t RB) { return D == 128 && RB % 128 == 0; }
}  // namespace sa

extern "C" {

int sa_block_list_attention_fwd(int dtype, int64_t Z, int64_t H, int64_t Hkv, int64_t N,
                                int64_t D, int64_t route_block, const void* q,
                                const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                const void* v, const int64_t* v_strides, void* out,
                                const int64_t* out_strides, float* lse, const int32_t* lists,
                                int64_t list_stride, const int32_t* counts, const void* soft_bias,
                                int sb_dtype, const int64_t* sb_strides, int is_causal,
                                float sm_scale, void* workspace, int64_t workspace_bytes,
                                void* stream) {
  using namespace sa;
  AttnParams p{};
  int rc = fill_common(p, dtype, Z, H, Hkv, N, D, route_block, q, q_strides, k, k_strides, v,
                       v_strides, lists, list_stride, counts, soft_bias, sb_dtype, sb_strides,
                       is_causal, sm_scale);
  if (rc) return rc;
  if (!out_strides || out_strides[3] != 1)
    return fail(SA_EUNSUPPORTED, "out: head_dim must be the contiguous dimension");
  p.out = out;
  for (int i = 0; i < 4; ++i) p.os[i] = out_strides[i];
  p.lse = lse;
  if (Z * H * N == 0) return SA_OK;
  if (!q || !k || !v || !out || !lists || !counts) return fail(SA_EINVAL, "null pointer argument");
  if (workspace) {
    if (reinterpret_cast<uintptr_t>(workspace) % 256)
      return fail(SA_EINVAL, "workspace must be 256-byte aligned");
    if (workspace_bytes < fwd_plan_bytes(Z, H, N, D))
      return fail(SA_EWORKSPACE, "forward workspace too small");
    p.plan_fwd = workspace;
  }
  cudaStream_t s = (cudaStream_t)stream;
  rc = launch_fwd_sm100(p, s);
  if (rc != SA_EUNSUPPORTED) return rc;
  return launch_fwd_simt(p, s);
}

int sa_block_list_attention_fwd_accumulate(int dtype, int64_t Z, int64_t H, int64_t Hkv, int64_t N,
                                           int64_t D, int64_t route_block, const void* q,
                                           const int64_t* q_strides, const void* k,
                                           const int64_t* k_strides, const void* v,
                                           const int64_t* v_strides, void* out,
                                           const int64_t* out_strides, float* lse,
                                           const int32_t* lists, int64_t list_stride,
                                           const int32_t* counts, int is_causal, float sm_scale,
                                           void* workspace, int64_t workspace_bytes,
                                           void* stream) {
  using namespace sa;
  AttnParams p{};
  int rc = fill_common(p, dtype, Z, H, Hkv, N, D, route_block, q, q_strides, k, k_strides, v,
                       v_strides, lists, list_stride, counts, nullptr, 0, nullptr, is_causal,
                       sm_scale);
  if (rc) return rc;
  if (!out_strides || out_strides[3] != 1)
    return fail(SA_EUNSUPPORTED, "out: head_dim must be the contiguous dimension");
  p.out = out;
  for (int i = 0; i < 4; ++i) p.os[i] = out_strides[i];
  p.lse = lse;
  p.accumulate = 1;
  if (Z * H * N == 0) return SA_OK;
  if (!q || !k || !v || !out || !lse || !lists || !counts)
    return fail(SA_EINVAL, "null pointer argument (accumulate needs out and lse)");
  if (workspace) {
    if (reinterpret_cast<uintptr_t>(workspace) % 256)
      return fail(SA_EINVAL, "workspace must be 256-byte aligned");
    if (workspace_bytes < fwd_plan_bytes(Z, H, N, D))
      return fail(SA_EWORKSPACE, "forward workspace too small");
    p.plan_fwd = workspace;
  }
  rc = launch_fwd_sm100(p, (cudaStream_t)stream);
  if (rc == SA_EUNSUPPORTED)
    return fail(SA_EUNSUPPORTED, "accumulating forward: needs the tensor-core path (bf16/fp16, "
                                 "head_dim 64/128, route_block a multiple of 128, aligned rows)");
  return rc;
}

int64_t sa_block_list_attention_fwd_workspace_bytes(int64_t Z, int64_t H, int64_t N, int64_t D,
                                                    int64_t route_block) {
  if (Z <= 0 || H <= 0 || N <= 0 || D <= 0 || route_block <= 0) return 0;
  return sa::fwd_plan_bytes(Z, H, N, D);
}

int64_t sa_block_list_attention_bwd_workspace_bytes(int64_t Z, int64_t H, int64_t Hkv, int64_t N,
                                                    int64_t D, int64_t route_block) {
  using sa::align256;
  if (Z <= 0 || H <= 0 || Hkv <= 0 || N <= 0 || D <= 0 || route_block <= 0) return 0;
  const int64_t NB = (N + route_block - 1) / route_block;
  size_t b = align256((size_t)Z * H * N * sizeof(float));            // delta
  b += 2 * align256((size_t)Z * H * NB * NB * sizeof(int32_t));       // k_lists, k_slots
  b += align256((size_t)Z * H * NB * sizeof(int32_t));                // q_counts
  b += align256((size_t)Z * H * ((N + 63) / 64) * 128 * sizeof(float));  // row stats
  b += align256((size_t)sa::bwd_plan_bytes(sa::kPlanDq, Z, H, Hkv, N, D));
  b += align256((size_t)sa::bwd_plan_bytes(sa::kPlanDkdv, Z, H, Hkv, N, D));
  if (sa::fused_shape(D, route_block))
    b += align256((size_t)Z * H * N * D * sizeof(float));  // fp32 dQ accumulator
  return (int64_t)b;
}

int sa_block_list_attention_bwd_phase(int phase, int dtype, int64_t Z, int64_t H, int64_t Hkv,
                                      int64_t N, int64_t D, int64_t route_block, const void* q,
                                const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                const void* v, const int64_t* v_strides, const void* out,
                                const int64_t* out_strides, const void* dout,
                                const int64_t* dout_strides, const float* lse,
                                const int32_t* lists, int64_t list_stride, const int32_t* counts,
                                const void* soft_bias, int sb_dtype, const int64_t* sb_strides,
                                int is_causal, float sm_scale, void* dq,
                                const int64_t* dq_strides, void* dk, const int64_t* dk_strides,
                                void* dv, const int64_t* dv_strides, float* d_soft_bias,
                                void* workspace, int64_t workspace_bytes, void* stream) {
  using namespace sa;
  AttnParams p{};
  int rc = fill_common(p, dtype, Z, H, Hkv, N, D, route_block, q, q_strides, k, k_strides, v,
                       v_strides, lists, list_stride, counts, soft_bias, sb_dtype, sb_strides,
                       is_causal, sm_scale);
  if (rc) return rc;
  const int64_t* arrs[5] = {out_strides, dout_strides, dq_strides, dk_strides, dv_strides};
  for (auto a : arrs)
    if (!a || a[3] != 1) return fail(SA_EUNSUPPORTED, "gradients: head_dim must be contiguous");
  if (d_soft_bias && !soft_bias) return fail(SA_EINVAL, "d_soft_bias needs soft_bias");
  p.out = const_cast<void*>(out);
  p.dout = dout;
  p.dq = dq;
  p.dk = dk;
  p.dv = dv;
  for (int i = 0; i < 4; ++i) {
    p.os[i] = out_strides[i];
    p.dos[i] = dout_strides[i];
    p.dqs[i] = dq_strides[i];
    p.dks[i] = dk_strides[i];
    p.dvs[i] = dv_strides[i];
  }
  p.lse = const_cast<float*>(lse);
  p.dbias = d_soft_bias;
  if (Z * H * N == 0) return SA_OK;
  if (!q || !k || !v || !out || !dout || !lse || !lists || !counts || !dq || !dk || !dv)
    return fail(SA_EINVAL, "null pointer argument");
  const int64_t need = sa_block_list_attention_bwd_workspace_bytes(Z, H, Hkv, N, D, route_block);
  if (!workspace || workspace_bytes < need)
    return fail(SA_EWORKSPACE, "backward workspace too small (" + std::to_string(workspace_bytes) +
                                   " < " + std::to_string(need) + ")");
  if (reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(SA_EINVAL, "workspace must be 256-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  char* w = static_cast<char*>(workspace);
  const int64_t NB = p.NB;
  p.delta = reinterpret_cast<float*>(w);
  w += align256((size_t)Z * H * N * sizeof(float));
  int32_t* k_lists = reinterpret_cast<int32_t*>(w);
  w += align256((size_t)Z * H * NB * NB * sizeof(int32_t));
  int32_t* k_slots = reinterpret_cast<int32_t*>(w);
  w += align256((size_t)Z * H * NB * NB * sizeof(int32_t));
  int32_t* q_counts = reinterpret_cast<int32_t*>(w);
  w += align256((size_t)Z * H * NB * sizeof(int32_t));
  p.stats = reinterpret_cast<float*>(w);
  w += align256((size_t)Z * H * ((N + 63) / 64) * 128 * sizeof(float));
  p.plan_dq = w;
  w += align256((size_t)bwd_plan_bytes(kPlanDq, Z, H, Hkv, N, D));
  p.plan_dkdv = w;
  w += align256((size_t)bwd_plan_bytes(kPlanDkdv, Z, H, Hkv, N, D));
  p.k_lists = k_lists;
  p.k_slots = k_slots;
  p.q_counts = q_counts;

  if (phase < 0 || phase > 5) return fail(SA_EINVAL, "backward phase must be 0..5");
  // phase 0 = the whole backward, fused when the shape allows; 1-3 = the two-kernel path
  // (prep, dQ, dK/dV: reproducible dQ sums); 4-5 = the fused path (prep, fused kernel)
  const bool fused = (phase == 0 || phase >= 4) && fused_shape(D, route_block) && bwd_fused_eligible(p);
  if (fused) p.dq_acc = reinterpret_cast<float*>(w);
  if (phase == 4 && !fused) phase = 1;  // shapes without the fused kernel: two-kernel path
  if (phase == 5 && !fused) {
    rc = launch_bwd_sm100(p, s, kBwdDq | kBwdDkDv);
    if (rc != SA_EUNSUPPORTED) return rc;
    return launch_bwd_simt(p, s, kBwdDq | kBwdDkDv);
  }
  if (phase == 0 || phase == 1 || phase == 4) {
    // Delta (HBM-bound, a wide grid) runs on the caller's stream; the transposition and the
    // dK/dV planner (small, latency-bound, independent of Delta) on a high-priority second
    // stream beside it.  The caller's stream waits for both.  (The dQ planner runs with the
    // dQ kernel, under its first wave.)
    cudaStream_t side;
    cudaEvent_t fork, join;
    rc = side_stream(&side, &fork, &join);
    if (rc) return rc;
    if (cudaEventRecord(fork, s) != cudaSuccess || cudaStreamWaitEvent(side, fork, 0) != cudaSuccess)
      return check_launch("backward fork");
    rc = launch_transpose_lists(lists, list_stride, counts, Z * H, NB, NB, k_lists, NB,
                                q_counts, k_slots, 0, side);
    if (!rc) rc = plan_bwd_sm100(p, side, kBwdDkDv);
    if (cudaEventRecord(join, side) != cudaSuccess) return check_launch("backward join");
    if (!rc) rc = launch_delta(p, s);
    // join before any return, so the side stream never runs past this call
    if (cudaStreamWaitEvent(s, join, 0) != cudaSuccess) return check_launch("backward join");
    if (rc) return rc;
    if (d_soft_bias) {
      if (cudaMemsetAsync(d_soft_bias, 0, (size_t)Z * H * NB * list_stride * sizeof(float), s) !=
          cudaSuccess)
        return check_launch("memset d_soft_bias");
    }
  }
  int parts = phase == 0 ? (kBwdDq | kBwdDkDv) : phase == 2 ? kBwdDq : phase == 3 ? kBwdDkDv : 0;
  if (fused && (phase == 0 || phase == 5)) parts = kBwdFused;
  if (!parts) return SA_OK;
  rc = launch_bwd_sm100(p, s, parts);
  if (rc != SA_EUNSUPPORTED) return rc;
  return launch_bwd_simt(p, s, parts);
}

int sa_block_list_attention_bwd(int dtype, int64_t Z, int64_t H, int64_t Hkv, int64_t N,
                                int64_t D, int64_t route_block, const void* q,
                                const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                const void* v, const int64_t* v_strides, const void* out,
                                const int64_t* out_strides, const void* dout,
                                const int64_t* dout_strides, const float* lse,
                                const int32_t* lists, int64_t list_stride, const int32_t* counts,
                                const void* soft_bias, int sb_dtype, const int64_t* sb_strides,
                                int is_causal, float sm_scale, void* dq,
                                const int64_t* dq_strides, void* dk, const int64_t* dk_strides,
                                void* dv, const int64_t* dv_strides, float* d_soft_bias,
                                void* workspace, int64_t workspace_bytes, void* stream) {
  return sa_block_list_attention_bwd_phase(
      0, dtype, Z, H, Hkv, N, D, route_block, q, q_strides, k, k_strides, v, v_strides, out,
      out_strides, dout, dout_strides, lse, lists, list_stride, counts, soft_bias, sb_dtype,
      sb_strides, is_causal, sm_scale, dq, dq_strides, dk, dk_strides, dv, dv_strides,
      d_soft_bias, workspace, workspace_bytes, stream);
}

}  // extern "C"

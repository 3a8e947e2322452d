// Log-sum-exp merge of partial attention results: the combine step of the sequence-sharded
// ring (each hop attends this rank's queries to one visiting K/V chunk and yields a partial
// output O_j, already normalised, and its natural-log LSE_j):
//
//   lse = log(exp(lse_acc) + exp(lse_j)),  O = O_acc * exp(lse_acc - lse) + O_j * exp(lse_j - lse)
//
// Rows that saw no key in a hop carry lse_j = -inf and contribute nothing; a row with no
// key in any hop keeps O = 0 and lse = -inf (the forward's empty-row convention,
// src/ultrametric/block_list.py:455-470 of sparse-ai).  The accumulator is fp32.
#include "common.cuh"

namespace sa {
namespace {

struct MergeArgs {
  int64_t Z, H, N, D;
  const void* o;  // (Z, H, N, D) partial, dtype
  int64_t os[4];
  const float* lse;  // (Z, H, N) partial
  float* acc;        // (Z, H, N, D) fp32 contiguous
  float* lse_acc;    // (Z, H, N) fp32
  void* out;         // optional (Z, H, N, D) dtype: the merged result after this hop
  int64_t outs[4];
  int init;
};

// One warp per row; lanes stride the head dim.
template <typename T>
__global__ void __launch_bounds__(256) lse_merge_kernel(const MergeArgs a) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= a.Z * a.H * a.N) return;
  const int64_t n = row % a.N, zh = row / a.N, z = zh / a.H, h = zh % a.H;
  const float lj = a.lse[row];
  const float la = a.init ? -INFINITY : a.lse_acc[row];
  const float m = fmaxf(la, lj);
  float wa = 0.f, wj = 0.f, lnew = -INFINITY;
  if (m != -INFINITY) {
    const float ea = expf(la - m), ej = expf(lj - m);
    lnew = m + logf(ea + ej);
    wa = expf(la - lnew);
    wj = expf(lj - lnew);
  }
  const T* o = static_cast<const T*>(a.o) + z * a.os[0] + h * a.os[1] + n * a.os[2];
  float* acc = a.acc + row * a.D;
  T* out = a.out ? static_cast<T*>(a.out) + z * a.outs[0] + h * a.outs[1] + n * a.outs[2] : nullptr;
  for (int64_t d = lane; d < a.D; d += 32) {
    const float prev = a.init ? 0.f : acc[d];
    const float v = (wa > 0.f ? prev * wa : 0.f) + (wj > 0.f ? to_f32<T>(o[d]) * wj : 0.f);
    acc[d] = v;
    if (out) out[d] = from_f32<T>(v);
  }
  if (lane == 0) a.lse_acc[row] = lnew;
}

}  // namespace
}  // namespace sa

extern "C" {

int sa_attention_lse_merge(int dtype, int64_t Z, int64_t H, int64_t N, int64_t D, const void* o_part,
                           const int64_t* o_part_strides, const float* lse_part, float* o_acc,
                           float* lse_acc, int init, void* out, const int64_t* out_strides,
                           void* stream) {
  using namespace sa;
  if (Z < 0 || H < 0 || N < 0 || D <= 0) return fail(SA_EINVAL, "merge: bad sizes");
  if (Z * H * N == 0) return SA_OK;
  if (!o_part || !o_part_strides || !lse_part || !o_acc || !lse_acc)
    return fail(SA_EINVAL, "merge: null pointer argument");
  if (out && !out_strides) return fail(SA_EINVAL, "merge: out needs out_strides");
  if (o_part_strides[3] != 1 || (out && out_strides[3] != 1))
    return fail(SA_EUNSUPPORTED, "merge: head_dim must be the contiguous dimension");
  MergeArgs a{};
  a.Z = Z;
  a.H = H;
  a.N = N;
  a.D = D;
  a.o = o_part;
  a.lse = lse_part;
  a.acc = o_acc;
  a.lse_acc = lse_acc;
  a.out = out;
  a.init = init;
  for (int i = 0; i < 4; ++i) {
    a.os[i] = o_part_strides[i];
    a.outs[i] = out ? out_strides[i] : 0;
  }
  const int64_t rows = Z * H * N;
  const unsigned blocks = (unsigned)((rows * 32 + 255) / 256);
  cudaStream_t s = (cudaStream_t)stream;
  switch (dtype) {
    case SA_F32: lse_merge_kernel<float><<<blocks, 256, 0, s>>>(a); break;
    case SA_F16: lse_merge_kernel<__half><<<blocks, 256, 0, s>>>(a); break;
    case SA_BF16: lse_merge_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(a); break;
    default: return fail(SA_EUNSUPPORTED, "merge: dtype must be fp32, fp16 or bf16");
  }
  return check_launch("lse_merge_kernel");
}

}  // extern "C"

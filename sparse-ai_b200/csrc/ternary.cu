// Ternary (2-bit) K/V: quantise + pack, and unpack + dequantise, for the ternary prefill of
// sparse-ai's LLaMA surgery (src/llama_surgery/surgery.py:15-75, kernel.py:147-249 there).
//
// Quantisation (TernaryQuantize.forward, surgery.py:15-28): per row of D values,
// gamma = mean |x|, x_t = +1 where x > gamma / 2, -1 where x < -gamma / 2, else 0.
// Packing (pack_ternary, surgery.py:35-55): 16 values per int32, value i of a group in bits
// [2i, 2i + 2) with code 1 = +1, 2 = -1, 0 = 0.  The ternary attention kernel of the
// reference dequantises each row as x_t * scale with scale = gamma (per token), rounded to
// fp16 before its dot products (kernel.py:203-205, 230-232).
// One warp per row: lane j owns 16 consecutive values (one packed word) when D = 512, fewer
// lanes otherwise; HBM-bound byte work.
#include <string>

#include "common.cuh"

namespace sa {
namespace {

// quantise + pack: rows of D values (any float type) -> packed (rows, D / 16) int32, scale (rows,)
template <typename T>
__global__ void __launch_bounds__(256) ternary_pack_kernel(const T* __restrict__ x, int64_t xs,
                                                           int64_t rows, int D, int32_t* packed,
                                                           float* scale) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;  // uniform over the warp
  const T* xr = x + row * xs;
  float s = 0.f;
  for (int d = lane; d < D; d += 32) s += fabsf(to_f32<T>(xr[d]));
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float gamma = s / (float)D, thr = 0.5f * gamma;
  for (int w = lane; w < D / 16; w += 32) {
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float v = to_f32<T>(xr[w * 16 + i]);
      const uint32_t code = v > thr ? 1u : (v < -thr ? 2u : 0u);
      word |= code << (2 * i);
    }
    packed[row * (D / 16) + w] = (int32_t)word;
  }
  if (lane == 0) scale[row] = gamma;
}

// unpack + dequantise: packed (rows, D / 16), scale (rows,) -> out rows (x_t * scale in T)
template <typename T>
__global__ void __launch_bounds__(256) ternary_unpack_kernel(const int32_t* __restrict__ packed,
                                                             const float* __restrict__ scale,
                                                             int64_t rows, int D, T* out, int64_t os) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one packed word
  const int64_t words = (int64_t)D / 16;
  if (i >= rows * words) return;
  const int64_t row = i / words, w = i % words;
  const uint32_t word = (uint32_t)packed[i];
  const float sc = scale[row];
  T* dst = out + row * os + w * 16;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const uint32_t code = (word >> (2 * k)) & 3u;
    const float v = code == 1u ? sc : (code == 2u ? -sc : 0.f);
    dst[k] = from_f32<T>(v);
  }
}

}  // namespace
}  // namespace sa

extern "C" {

int sa_ternary_quantize_pack(int dtype, int64_t rows, int64_t D, const void* x, int64_t x_row_stride,
                             int32_t* packed, float* scale, void* stream) {
  using namespace sa;
  if (rows < 0 || D <= 0 || D % 16) return fail(SA_EINVAL, "ternary pack: D must be a positive multiple of 16");
  if (rows == 0) return SA_OK;
  if (!x || !packed || !scale) return fail(SA_EINVAL, "ternary pack: null pointer argument");
  const unsigned grid = (unsigned)((rows * 32 + 255) / 256);
  cudaStream_t s = (cudaStream_t)stream;
  switch (dtype) {
    case SA_F32:
      ternary_pack_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(x), x_row_stride, rows,
                                                       (int)D, packed, scale);
      break;
    case SA_F16:
      ternary_pack_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(x), x_row_stride, rows,
                                                        (int)D, packed, scale);
      break;
    case SA_BF16:
      ternary_pack_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                               x_row_stride, rows, (int)D, packed, scale);
      break;
    default: return fail(SA_EUNSUPPORTED, "ternary pack: dtype");
  }
  return check_launch("ternary_pack_kernel");
}

int sa_ternary_dequantize(int dtype, int64_t rows, int64_t D, const int32_t* packed, const float* scale,
                          void* out, int64_t out_row_stride, void* stream) {
  using namespace sa;
  if (rows < 0 || D <= 0 || D % 16) return fail(SA_EINVAL, "ternary dequantize: D must be a positive multiple of 16");
  if (rows == 0) return SA_OK;
  if (!packed || !scale || !out) return fail(SA_EINVAL, "ternary dequantize: null pointer argument");
  const int64_t words = rows * (D / 16);
  const unsigned grid = (unsigned)((words + 255) / 256);
  cudaStream_t s = (cudaStream_t)stream;
  switch (dtype) {
    case SA_F32:
      ternary_unpack_kernel<float><<<grid, 256, 0, s>>>(packed, scale, rows, (int)D, static_cast<float*>(out),
                                                         out_row_stride);
      break;
    case SA_F16:
      ternary_unpack_kernel<__half><<<grid, 256, 0, s>>>(packed, scale, rows, (int)D, static_cast<__half*>(out),
                                                          out_row_stride);
      break;
    case SA_BF16:
      ternary_unpack_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(packed, scale, rows, (int)D,
                                                                 static_cast<__nv_bfloat16*>(out), out_row_stride);
      break;
    default: return fail(SA_EUNSUPPORTED, "ternary dequantize: dtype");
  }
  return check_launch("ternary_unpack_kernel");
}

}  // extern "C"

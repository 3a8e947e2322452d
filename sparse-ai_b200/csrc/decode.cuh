// Shared declarations of the routed paged decode (general split-K path in decode.cu, the
// tensor-core fast path in decode_sm100.cu).
#pragma once

#include "common.cuh"

namespace sa {

struct DecodeParams {
  int64_t B, H, Hkv, G, D, page, num_pages, maxL, TD, r, local_blocks;
  int sink;
  const void* q;
  int64_t qs[3];
  const void* kc;
  int64_t ks[4];
  const void* vc;
  int64_t vs[4];
  const int32_t* bt;
  int64_t bts[2];
  const int32_t* ctx;
  const void* router;
  int router_dtype;
  int64_t rs[3];
  const void* qrouter;
  int qrouter_dtype;
  int64_t qrs[3];
  void* out;
  int64_t os[3];
  float* part;  // [B][Hkv][S][G][D + 2]: m (log2 units), l, acc[D]
  int S;
  int stages;
};

// Tensor-core fast path: bf16/fp16, head_dim 64 or 128, <= 16 query heads per KV head, page
// size 16, 32 or a multiple of 64, 16-byte aligned query rows.  Returns false (and leaves
// no error) when the shape needs the general path.
bool decode_fast_eligible(const DecodeParams& p, int dtype);
int64_t decode_fast_workspace_bytes(int64_t B, int64_t H, int64_t Hkv, int64_t D, int64_t maxL);
int launch_decode_fast(const DecodeParams& p, int dtype, void* workspace, int64_t workspace_bytes,
                       cudaStream_t stream);

}  // namespace sa

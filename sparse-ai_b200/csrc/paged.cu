// Paged K/V cache maintenance for the routed decode: append one token per request and keep
// the routing vector of each request's tail page current.
//
// sparse-ai decodes from a dense per-layer cache with an eager token mask
// (src/llama_surgery/surgery.py:883-891); its paged decode kernel
// (src/ultrametric/kernel_decode.py:188-247) has no caller that fills a paged cache.  This is
// that missing writer: the per-step scatter of the new token's K and V rows into the page
// that holds position context_lens[b] (the page itself is assigned by the host's page
// allocator), and the refresh of that page's routing vector, which the reference recomputes
// for its tail block at every decode step (surgery.py:350-374).  Byte work, HBM-bound: one
// CTA per request, 16-byte copies.
#include <string>

#include "common.cuh"

namespace sa {
namespace {

struct AppendParams {
  const void* kn;
  int64_t kns[2];  // (B, Hkv, D): request, head strides (D contiguous)
  const void* vn;
  int64_t vns[2];
  const int32_t* bt;
  int64_t bts[2];
  int32_t* ctx;
  void* kc;
  int64_t ks[3];  // (P, Hkv, page, D): page, head, row strides
  void* vc;
  int64_t vs[3];
  const void* routes;  // (B, H, TD) or null
  int routes_dtype;
  int64_t rts[3];
  void* router;  // (P, H, TD)
  int router_dtype;
  int64_t rrs[3];
  int64_t Hkv, D, page, num_pages, maxL, H, TD;
  int esz;  // element bytes of K / V
  unsigned* status;
};

__global__ void __launch_bounds__(256) paged_append_kernel(AppendParams p) {
  const int64_t b = blockIdx.x;
  const int32_t pos = p.ctx[b];
  const int64_t lp = pos / p.page, slot = pos % p.page;
  const int32_t phys = lp < p.maxL ? p.bt[b * p.bts[0] + lp * p.bts[1]] : -1;
  if (phys < 0 || phys >= p.num_pages) {  // no page assigned for this position: skip the row
    if (threadIdx.x == 0) raise_status(p.status, kStatusBadIndex);
    return;
  }
  // K and V rows: Hkv x D elements each, copied in 16-byte units
  const int64_t units = p.Hkv * p.D * p.esz / 16, per_head = p.D * p.esz / 16;
  for (int64_t u = threadIdx.x; u < 2 * units; u += blockDim.x) {
    const bool is_v = u >= units;
    const int64_t uu = is_v ? u - units : u, h = uu / per_head, c = uu % per_head;
    const char* src = static_cast<const char*>(is_v ? p.vn : p.kn) +
                      (b * (is_v ? p.vns[0] : p.kns[0]) + h * (is_v ? p.vns[1] : p.kns[1])) * p.esz + c * 16;
    const int64_t* cs = is_v ? p.vs : p.ks;
    char* dst = static_cast<char*>(is_v ? p.vc : p.kc) + (phys * cs[0] + h * cs[1] + slot * cs[2]) * p.esz + c * 16;
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
  }
  if (p.routes) {
    for (int64_t i = threadIdx.x; i < p.H * p.TD; i += blockDim.x) {
      const int64_t h = i / p.TD, l = i % p.TD;
      const int64_t v = load_any_i64(p.routes, p.routes_dtype, b * p.rts[0] + h * p.rts[1] + l * p.rts[2]);
      const int64_t o = (int64_t)phys * p.rrs[0] + h * p.rrs[1] + l * p.rrs[2];
      if (p.router_dtype == SA_I64)
        static_cast<int64_t*>(p.router)[o] = v;
      else
        static_cast<int32_t*>(p.router)[o] = (int32_t)v;
    }
  }
  __syncthreads();  // every thread has read ctx[b] before it moves on
  if (threadIdx.x == 0) p.ctx[b] = pos + 1;
}

}  // namespace
}  // namespace sa

extern "C" {

int sa_paged_kv_append(int dtype, int64_t B, int64_t Hkv, int64_t D, int64_t page_size,
                       int64_t num_pages, const void* k_new, const int64_t* k_new_strides,
                       const void* v_new, const int64_t* v_new_strides,
                       const int32_t* block_tables, const int64_t* bt_strides,
                       int64_t max_logical_pages, int32_t* context_lens, void* k_cache,
                       const int64_t* k_strides, void* v_cache, const int64_t* v_strides,
                       const void* routes, int routes_dtype, const int64_t* routes_strides,
                       int64_t H, int64_t TD, void* router, int router_dtype,
                       const int64_t* router_strides, void* stream) {
  using namespace sa;
  if (B < 0 || Hkv <= 0 || D <= 0 || page_size <= 0 || num_pages < 0 || max_logical_pages < 0)
    return fail(SA_EINVAL, "paged append: bad sizes");
  if (B == 0) return SA_OK;
  if (dtype != SA_F32 && dtype != SA_F16 && dtype != SA_BF16)
    return fail(SA_EUNSUPPORTED, "paged append: dtype must be fp32, fp16 or bf16");
  if (!k_new || !v_new || !block_tables || !context_lens || !k_cache || !v_cache ||
      !k_new_strides || !v_new_strides || !bt_strides || !k_strides || !v_strides)
    return fail(SA_EINVAL, "paged append: null pointer argument");
  const int esz = dtype == SA_F32 ? 4 : 2;
  if (k_new_strides[2] != 1 || v_new_strides[2] != 1 || k_strides[3] != 1 || v_strides[3] != 1)
    return fail(SA_EUNSUPPORTED, "paged append: head_dim must be contiguous");
  if ((D * esz) % 16) return fail(SA_EUNSUPPORTED, "paged append: rows must be multiples of 16 bytes");
  const void* ptrs[4] = {k_new, v_new, k_cache, v_cache};
  for (auto q : ptrs)
    if (reinterpret_cast<uintptr_t>(q) % 16) return fail(SA_EUNSUPPORTED, "paged append: 16-byte alignment");
  for (int i = 0; i < 2; ++i)
    if ((k_new_strides[i] * esz) % 16 || (v_new_strides[i] * esz) % 16)
      return fail(SA_EUNSUPPORTED, "paged append: strides must be multiples of 16 bytes");
  for (int i = 0; i < 3; ++i)
    if ((k_strides[i] * esz) % 16 || (v_strides[i] * esz) % 16)
      return fail(SA_EUNSUPPORTED, "paged append: strides must be multiples of 16 bytes");
  if (routes) {
    if (!router || !routes_strides || !router_strides || H <= 0 || TD <= 0)
      return fail(SA_EINVAL, "paged append: routes need the router table, strides, H and TD");
    if ((routes_dtype != SA_I32 && routes_dtype != SA_I64) ||
        (router_dtype != SA_I32 && router_dtype != SA_I64))
      return fail(SA_EUNSUPPORTED, "paged append: routes must be int32 or int64");
  }
  if (B > 2147483647) return fail(SA_EUNSUPPORTED, "paged append: too many requests");
  if (int rc = check_stream_device(stream, "paged append")) return rc;
  AppendParams p{};
  p.kn = k_new;
  p.vn = v_new;
  for (int i = 0; i < 2; ++i) {
    p.kns[i] = k_new_strides[i];
    p.vns[i] = v_new_strides[i];
    p.bts[i] = bt_strides[i];
  }
  p.bt = block_tables;
  p.ctx = context_lens;
  p.kc = k_cache;
  p.vc = v_cache;
  for (int i = 0; i < 3; ++i) {
    p.ks[i] = k_strides[i];
    p.vs[i] = v_strides[i];
    p.rts[i] = routes ? routes_strides[i] : 0;
    p.rrs[i] = routes ? router_strides[i] : 0;
  }
  p.routes = routes;
  p.routes_dtype = routes_dtype;
  p.router = router;
  p.router_dtype = router_dtype;
  p.Hkv = Hkv;
  p.D = D;
  p.page = page_size;
  p.num_pages = num_pages;
  p.maxL = max_logical_pages;
  p.H = H;
  p.TD = TD;
  p.esz = esz;
  p.status = device_status_ptr();
  if (!p.status) return fail(SA_ELAUNCH, std::string("paged append: ") + sa_last_error());
  paged_append_kernel<<<(unsigned)B, 256, 0, (cudaStream_t)stream>>>(p);
  return check_launch("paged_append_kernel");
}

}  // extern "C"

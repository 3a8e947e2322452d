/*
 * sparse_ai_b200.h -- C ABI of the B200 (sm_100a) block-sparse attention library.
 *
 * The library re-implements the block-sparse attention hot path of sparse-ai's
 * src/ultrametric (routing -> block lists, block-list prefill forward/backward, routed
 * paged decode).  Each entry point below replaces one launch site of the reference's
 * Triton code; the comment above it names that site (path:line inside sparse-ai).
 *
 * Conventions
 *   - Every tensor argument is a raw DEVICE pointer; shapes are int64 element counts and
 *     strides are int64 ELEMENT strides given as host arrays (outermost dim first).
 *   - The caller allocates every input, output and workspace.  The library never
 *     allocates or frees device memory.
 *   - All work is enqueued on `stream` (a cudaStream_t passed as void*; NULL = legacy
 *     default stream).  Entries return without synchronising.
 *   - Return value: SA_OK (0) or a negative SA_E* code; sa_last_error() gives the message
 *     of the calling thread's last failure.
 */
#ifndef SPARSE_AI_B200_H
#define SPARSE_AI_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SA_API __attribute__((visibility("default")))
#else
#define SA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define SA_OK 0
#define SA_EINVAL (-1)      /* bad shape, stride, pointer or flag */
#define SA_EUNSUPPORTED (-2) /* dtype / head_dim / alignment this build does not handle */
#define SA_ELAUNCH (-3)     /* CUDA launch or runtime failure */
#define SA_EWORKSPACE (-4)  /* workspace smaller than sa_*_workspace_bytes() */

/* element types */
#define SA_F32 0
#define SA_F16 1
#define SA_BF16 2
#define SA_I32 3
#define SA_I64 4

/* Message of the calling thread's last failed call ("" if none). */
SA_API const char* sa_last_error(void);

/* ABI version of this library (bumped on any signature change; 3: the accumulating
 * forward takes the forward's optional workspace). */
SA_API int sa_abi_version(void);

/* Read the current device's status word (synchronises the device).  Kernels OR in
 * 1 when a bounded wait gave up, 2 on an out-of-range index, 4 when a kernel found its
 * dynamic shared memory too small for its aligned layout (it then does nothing);
 * reset != 0 clears it. */
SA_API int sa_read_device_status(int reset, unsigned* value);

/* Destroy the calling thread's side streams and events.  The backward's preparation phase
 * runs its small kernels on a second, high-priority stream per host thread and device,
 * created on first use and joined back into the caller's stream before each call returns;
 * this releases them (e.g. before a worker thread exits).  Synchronises those streams.
 * No counterpart in the reference (Triton keeps no such state). */
SA_API int sa_release_thread_resources(void);

/*
 * Routing vectors -> ascending active key-block lists.
 * Replaces: src/ultrametric/block_list.py:219-253 (mixed-radix prefix codes + launch of
 * _build_block_lists_kernel, kernel :127-167) and the torch fallback :255-278.
 *
 * router        (Z, H, NB, TD) integers (SA_I32 or SA_I64), any strides.
 * req_depth     device int32 (H,): levels that must agree per head, 0..TD.
 * base          radix of the prefix code (block_list.py:211-214: max(2, arity) on the
 *               sync-free path, max(2, max id + 1) otherwise).
 * use_codes     1: blocks match iff their wrapping int64 codes sum_{l<d} r_l*base^l are
 *               equal (block_list.py:224-229); 0: per-level equality (:256-258), used
 *               when TD*log2(base) >= 62.
 * lists         (Z, H, NB, list_stride) int32 out; row i gets its matches ascending in
 *               slots [0, counts[i]) and ZERO in slots [counts[i], list_stride).
 *               list_stride >= 1; matches beyond list_stride are counted, not stored.
 * counts        (Z, H, NB) int32 out.
 */
SA_API int sa_build_block_lists(const void* router, int router_dtype, const int64_t* router_strides,
                         int64_t Z, int64_t H, int64_t NB, int64_t TD,
                         const int32_t* req_depth, int64_t base, int use_codes,
                         int is_causal, int sink_block, int64_t local_blocks,
                         int32_t* lists, int64_t list_stride, int32_t* counts, void* stream);

/*
 * Key block -> ascending query blocks that list it (transposed lists for dK/dV).
 * Replaces: src/ultrametric/block_list.py:281-327 (build_transposed_block_lists).
 *
 * lists/counts  forward lists (ZH, NBQ, list_stride) / (ZH, NBQ); entries outside
 *               [0, NBK) are ignored.
 * k_lists       (ZH, NBK, k_list_stride) int32 out, zero padded; k_list_stride >= 1.
 * q_counts      (ZH, NBK) int32 out.
 * k_slots       optional (ZH, NBK, k_list_stride) int32 out: for entry (kb, j) = qb, the
 *               slot t with lists[qb][t] == kb (replaces the O(count) search of
 *               block_list.py:640-650); NULL to skip.
 */
SA_API int sa_build_transposed_block_lists(const int32_t* lists, int64_t list_stride,
                                    const int32_t* counts, int64_t ZH, int64_t NBQ, int64_t NBK,
                                    int32_t* k_lists, int64_t k_list_stride, int32_t* q_counts,
                                    int32_t* k_slots, void* stream);

/*
 * Router outputs -> block routes -> ascending block lists, all on the device.
 * Replaces: src/llama_surgery/surgery.py:533-547 (token argmax, per-block majority vote by
 * one-hot sums and argmax, or the argmax of block-level assignments) followed by the
 * build_block_lists(block_route, r, ..., arity=p) call of :562-564.
 *
 * assignments       (Z, H, S, levels, num_branches) of dtype (SA_F32/F16/BF16), any strides.
 * tokens_per_block  route block length in rows of `assignments`: route_block for
 *                   token-level outputs, 1 for block-level ones.  NB = ceil(S / it).
 * r                 levels that vote (0..min(levels, 32)); num_branches <= 16.
 *                   A block's branch per level is the majority of its rows' argmax branches
 *                   (first maximum wins within a row; vote ties go to the lowest branch id;
 *                   rows at or past S do not vote).
 * req_depth         device int32 (H,): levels that must agree per head (<= r).
 * arity             branch count; prefix codes use base max(2, arity) (the sync-free path).
 * block_route       (Z, H, NB, r) int32 out, contiguous (written only when r > 0).
 * lists/counts      as sa_build_block_lists.
 * Two launches on `stream` (vote, then compaction as its programmatic dependent); no
 * host synchronisation.
 */
SA_API int sa_build_block_lists_from_assignments(const void* assignments, int dtype,
                                          const int64_t* strides, int64_t Z, int64_t H,
                                          int64_t S, int64_t levels, int64_t num_branches,
                                          int64_t tokens_per_block, int64_t r,
                                          const int32_t* req_depth, int64_t arity,
                                          int is_causal, int sink_block, int64_t local_blocks,
                                          int32_t* block_route, int32_t* lists,
                                          int64_t list_stride, int32_t* counts, void* stream);

/*
 * Block-list attention forward.
 * Replaces: src/ultrametric/block_list.py:688-757 (_block_list_attention_fwd, kernel
 * :387-470).  Semantics: for each query row, online softmax over the keys of the route
 * blocks lists[z,h,qb,0:counts] (qb = row / route_block), scores q.k*sm_scale
 * (+ soft_bias[z,h,qb,t]), keys >= N masked, keys > row masked when is_causal; rows with
 * no visible key get out = 0 and lse = -inf.
 *
 * dtype         SA_BF16, SA_F16 (tcgen05 path) or SA_F32 (CUDA-core path); q/k/v/out share it.
 * q, out        (Z, H, N, D); k, v (Z, Hkv, N, D), H % Hkv == 0 (GQA: head h reads
 *               KV head h / (H/Hkv)).  Innermost stride must be 1.
 * lists/counts  int32 (Z, H, NB, list_stride) contiguous / (Z, H, NB), NB = ceil(N/route_block).
 * soft_bias     optional (Z, H, NB, list_stride) of sb_dtype with sb_strides, or NULL.
 * lse           optional fp32 (Z, H, N) contiguous, or NULL.
 * workspace     optional, >= sa_block_list_attention_fwd_workspace_bytes() bytes, 256-aligned:
 *               the tcgen05 kernel then schedules its work items heaviest-first from a queue
 *               (NULL: static round-robin; same results either way).
 */
SA_API int sa_block_list_attention_fwd(int dtype, int64_t Z, int64_t H, int64_t Hkv, int64_t N,
                                int64_t D, int64_t route_block,
                                const void* q, const int64_t* q_strides,
                                const void* k, const int64_t* k_strides,
                                const void* v, const int64_t* v_strides,
                                void* out, const int64_t* out_strides, float* lse,
                                const int32_t* lists, int64_t list_stride, const int32_t* counts,
                                const void* soft_bias, int sb_dtype, const int64_t* sb_strides,
                                int is_causal, float sm_scale,
                                void* workspace, int64_t workspace_bytes, void* stream);

/*
 * sa_block_list_attention_fwd that continues from a previous result instead of starting
 * from zero: out and lse hold the normalised output and natural-log LSE of the same rows
 * over an earlier, disjoint set of keys (e.g. the previous hop of the sequence-sharded
 * ring), and are updated in place to the result over both key sets -- the online softmax
 * resumes from that state, so no separate merge pass runs.  Rows with no listed block keep
 * their values.  No soft bias; tensor-core path only (bf16/fp16, head_dim 64/128,
 * route_block a multiple of 128, 16-byte aligned rows), else SA_EUNSUPPORTED.  The
 * optional workspace is the forward's (sa_block_list_attention_fwd_workspace_bytes; NULL:
 * static round-robin schedule).  No counterpart in the reference (it has no sequence parallelism; block_list.py:467-470 is
 * the LSE this consumes).
 */
SA_API int sa_block_list_attention_fwd_accumulate(int dtype, int64_t Z, int64_t H, int64_t Hkv,
                                                  int64_t N, int64_t D, int64_t route_block,
                                                  const void* q, const int64_t* q_strides,
                                                  const void* k, const int64_t* k_strides,
                                                  const void* v, const int64_t* v_strides,
                                                  void* out, const int64_t* out_strides, float* lse,
                                                  const int32_t* lists, int64_t list_stride,
                                                  const int32_t* counts, int is_causal,
                                                  float sm_scale, void* workspace,
                                                  int64_t workspace_bytes, void* stream);

/* Bytes of (optional) workspace for sa_block_list_attention_fwd, on the current device. */
SA_API int64_t sa_block_list_attention_fwd_workspace_bytes(int64_t Z, int64_t H, int64_t N,
                                                    int64_t D, int64_t route_block);

/* Bytes of workspace sa_block_list_attention_bwd needs for these sizes, on the current device. */
SA_API int64_t sa_block_list_attention_bwd_workspace_bytes(int64_t Z, int64_t H, int64_t Hkv,
                                                    int64_t N, int64_t D, int64_t route_block);

/*
 * Block-list attention backward.
 * Replaces: src/ultrametric/block_list.py:760-880 (_block_list_attention_bwd: Delta
 * :785, dQ kernel :494-584, transposed lists :844-846, dK/dV kernel :586-681).
 *
 * dout, out     (Z, H, N, D) like q; lse fp32 (Z, H, N) from the forward.
 * dq            (Z, H, N, D); dk, dv (Z, Hkv, N, D) -- overwritten (GQA groups summed).
 * d_soft_bias   optional fp32 (Z, H, NB, list_stride) contiguous, overwritten; needs
 *               soft_bias.  d_soft_bias[z,h,qb,t] = sum over the (row, key) pairs of the
 *               block pair of P*(dP - Delta) (unscaled dS).
 * workspace     >= sa_block_list_attention_bwd_workspace_bytes() bytes, 256-aligned.
 */
SA_API int sa_block_list_attention_bwd(int dtype, int64_t Z, int64_t H, int64_t Hkv, int64_t N,
                                int64_t D, int64_t route_block,
                                const void* q, const int64_t* q_strides,
                                const void* k, const int64_t* k_strides,
                                const void* v, const int64_t* v_strides,
                                const void* out, const int64_t* out_strides,
                                const void* dout, const int64_t* dout_strides,
                                const float* lse,
                                const int32_t* lists, int64_t list_stride, const int32_t* counts,
                                const void* soft_bias, int sb_dtype, const int64_t* sb_strides,
                                int is_causal, float sm_scale,
                                void* dq, const int64_t* dq_strides,
                                void* dk, const int64_t* dk_strides,
                                void* dv, const int64_t* dv_strides,
                                float* d_soft_bias,
                                void* workspace, int64_t workspace_bytes, void* stream);

/*
 * The backward split at the reference's own launch boundaries, for callers that schedule
 * or time the pieces separately (same arguments as sa_block_list_attention_bwd; the
 * workspace must persist from phase 1 to phases 2 and 3):
 *   phase 0  everything (== sa_block_list_attention_bwd)
 *   phase 1  Delta = rowsum(dO * O) and the transposed lists with slots
 *            (block_list.py:785 and :844-846), zeroes d_soft_bias
 *   phase 2  dQ and d_soft_bias (the _block_list_bwd_dq_kernel launch, block_list.py:811-842)
 *   phase 3  dK and dV (the _block_list_bwd_dkdv_kernel launch, block_list.py:844-876)
 */
SA_API int sa_block_list_attention_bwd_phase(int phase, int dtype, int64_t Z, int64_t H,
                                      int64_t Hkv, int64_t N, int64_t D, int64_t route_block,
                                      const void* q, const int64_t* q_strides,
                                      const void* k, const int64_t* k_strides,
                                      const void* v, const int64_t* v_strides,
                                      const void* out, const int64_t* out_strides,
                                      const void* dout, const int64_t* dout_strides,
                                      const float* lse,
                                      const int32_t* lists, int64_t list_stride,
                                      const int32_t* counts,
                                      const void* soft_bias, int sb_dtype, const int64_t* sb_strides,
                                      int is_causal, float sm_scale,
                                      void* dq, const int64_t* dq_strides,
                                      void* dk, const int64_t* dk_strides,
                                      void* dv, const int64_t* dv_strides,
                                      float* d_soft_bias,
                                      void* workspace, int64_t workspace_bytes, void* stream);

/* Bytes of workspace sa_ultrametric_decode needs for these sizes. */
SA_API int64_t sa_ultrametric_decode_workspace_bytes(int64_t B, int64_t H, int64_t Hkv, int64_t D,
                                              int64_t max_logical_pages);

/*
 * Routed sparse paged decode (one query token per request).
 * Replaces: src/ultrametric/kernel_decode.py:188-247 (ultrametric_decode launch, kernel
 * :23-124).  For request b and head h the logical pages l < ceil(ctx/page) whose routing
 * vector router[block_tables[b,l], h, 0:req_depth] equals q_router[b, h, 0:req_depth],
 * plus l == 0 when sink_block and the last local_blocks pages, are attended (tokens
 * >= context_lens[b] masked) at scale 1/sqrt(D).  context_lens[b] == 0 gives zeros.
 *
 * dtype         SA_BF16, SA_F16 or SA_F32 for q / caches / out.
 * q, out        (B, H, D); k_cache, v_cache (P, Hkv, page_size, D), innermost stride 1.
 * block_tables  int32 (B, max_logical_pages) with bt_strides; context_lens int32 (B,).
 * router        (P, H, TD) and q_router (B, H, TD) integers (SA_I32/SA_I64) with strides.
 * workspace     >= sa_ultrametric_decode_workspace_bytes() bytes, 256-aligned.
 */
SA_API int sa_ultrametric_decode(int dtype, int64_t B, int64_t H, int64_t Hkv, int64_t D,
                          int64_t page_size, int64_t num_pages,
                          const void* q, const int64_t* q_strides,
                          const void* k_cache, const int64_t* k_strides,
                          const void* v_cache, const int64_t* v_strides,
                          const int32_t* block_tables, const int64_t* bt_strides,
                          int64_t max_logical_pages, const int32_t* context_lens,
                          const void* router, int router_dtype, const int64_t* router_strides,
                          const void* q_router, int q_router_dtype, const int64_t* q_router_strides,
                          int64_t TD, int64_t req_depth, int64_t local_blocks, int sink_block,
                          void* out, const int64_t* out_strides,
                          void* workspace, int64_t workspace_bytes, void* stream);

/*
 * sa_ultrametric_decode without a caller workspace.  No counterpart in the reference: it is
 * for callers that cannot allocate device memory when they decode (a serving loop whose
 * memory is carved up front by its own pool and that binds only this C ABI, or a host that
 * must not trigger cudaMalloc's implicit synchronisation mid-step).  Same arguments and
 * results as sa_ultrametric_decode minus the workspace pair; the workspace (page lists,
 * chunk table, partials) comes from a fixed 16 MiB device array inside the library (held by every GPU that loads it
 * until exit).  Requests needing more than 16 MiB of workspace return SA_EWORKSPACE.  The
 * first call on a device looks the array up (make it before any stream capture).  All
 * calls share the array: calls that overlap on the GPU race.  `stream` must belong to the
 * current device, whose array is used (another device's stream: SA_EINVAL).  Allocates
 * nothing.
 */
SA_API int sa_ultrametric_decode_noalloc(int dtype, int64_t B, int64_t H, int64_t Hkv, int64_t D,
                          int64_t page_size, int64_t num_pages,
                          const void* q, const int64_t* q_strides,
                          const void* k_cache, const int64_t* k_strides,
                          const void* v_cache, const int64_t* v_strides,
                          const int32_t* block_tables, const int64_t* bt_strides,
                          int64_t max_logical_pages, const int32_t* context_lens,
                          const void* router, int router_dtype, const int64_t* router_strides,
                          const void* q_router, int q_router_dtype, const int64_t* q_router_strides,
                          int64_t TD, int64_t req_depth, int64_t local_blocks, int sink_block,
                          void* out, const int64_t* out_strides, void* stream);

/*
 * Append one token per request to a paged K/V cache (and refresh its page's route).
 * No counterpart in the reference kernels: sparse-ai's paged decode
 * (src/ultrametric/kernel_decode.py:188-247) reads such a cache but nothing there writes one
 * (its surgery layer decodes from a dense cache, src/llama_surgery/surgery.py:883-891); this
 * is the writer, with the tail-page route refresh of surgery.py:350-374.
 *
 * For request b: position pos = context_lens[b], page = block_tables[b][pos / page_size]
 * (assigned beforehand by the caller's allocator; an unassigned or out-of-range page sets
 * status bit 2 and skips the request), row pos % page_size of k_cache / v_cache
 * (P, Hkv, page_size, D) <- k_new / v_new (B, Hkv, D); when routes (B, H, TD) is given,
 * router (P, H, TD) of that page <- routes[b]; then context_lens[b] = pos + 1.
 * dtype SA_F32 / SA_F16 / SA_BF16 for K/V, rows 16-byte aligned; routes/router int32 or int64.
 */
SA_API int sa_paged_kv_append(int dtype, int64_t B, int64_t Hkv, int64_t D, int64_t page_size,
                              int64_t num_pages, const void* k_new, const int64_t* k_new_strides,
                              const void* v_new, const int64_t* v_new_strides,
                              const int32_t* block_tables, const int64_t* bt_strides,
                              int64_t max_logical_pages, int32_t* context_lens, void* k_cache,
                              const int64_t* k_strides, void* v_cache, const int64_t* v_strides,
                              const void* routes, int routes_dtype, const int64_t* routes_strides,
                              int64_t H, int64_t TD, void* router, int router_dtype,
                              const int64_t* router_strides, void* stream);

/*
 * Ternary K/V rows: quantise + pack, and unpack + dequantise.
 * Replaces: src/llama_surgery/surgery.py:15-75 (TernaryQuantize.forward, pack_ternary,
 * unpack_ternary) and the in-kernel unpacking of kernel.py:198-205, 226-232.
 *
 * quantize_pack: x (rows, D) of dtype (row stride x_row_stride, D contiguous, D % 16 == 0) ->
 *   scale[row] = mean |x[row]| (fp32), and packed (rows, D / 16) int32 contiguous: value i of
 *   16-value group w in bits [2i, 2i + 2) of word w, code 1 where x > scale / 2, 2 where
 *   x < -scale / 2, 0 otherwise.
 * dequantize: packed, scale -> out (rows, D) of dtype: code 1 -> +scale, 2 -> -scale, 0 -> 0.
 */
SA_API int sa_ternary_quantize_pack(int dtype, int64_t rows, int64_t D, const void* x,
                                    int64_t x_row_stride, int32_t* packed, float* scale,
                                    void* stream);
SA_API int sa_ternary_dequantize(int dtype, int64_t rows, int64_t D, const int32_t* packed,
                                 const float* scale, void* out, int64_t out_row_stride,
                                 void* stream);

/*
 * Log-sum-exp merge of partial attention outputs (the combine step of the sequence-sharded
 * ring for very long prefill; the reference has no ring -- its forward LSE output,
 * src/ultrametric/block_list.py:467-470, is the hook this uses).  Per row:
 *   lse_acc' = log(exp(lse_acc) + exp(lse_part))
 *   o_acc'   = o_acc * exp(lse_acc - lse_acc') + o_part * exp(lse_part - lse_acc')
 * o_part (Z, H, N, D) of dtype with strides (innermost 1) and lse_part fp32 (Z, H, N): one
 * partial (normalised output + natural-log LSE, as sa_block_list_attention_fwd writes
 * them); o_acc fp32 (Z, H, N, D) contiguous and lse_acc fp32 (Z, H, N) accumulate in place
 * (init != 0: start from this partial).  Rows with -inf LSE contribute nothing.  out
 * (optional, dtype, strides) receives the merged output after this partial.
 */
SA_API int sa_attention_lse_merge(int dtype, int64_t Z, int64_t H, int64_t N, int64_t D,
                                  const void* o_part, const int64_t* o_part_strides,
                                  const float* lse_part, float* o_acc, float* lse_acc, int init,
                                  void* out, const int64_t* out_strides, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPARSE_AI_B200_H */

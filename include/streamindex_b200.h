/* StreamIndex-B200 C ABI.
 *
 * Plain pointers, sizes and a cudaStream_t; no framework types.  Every call
 * only enqueues work on `stream` (no host synchronisation) and returns 0 on
 * success or -1 with a message available from si_last_error().
 *
 * Each entry point replaces one function of the reference's Python API
 * (tsukimia-hoshi/StreamIndex); the replaced function is cited beside it.
 * Tensors are contiguous, row-major, device-resident.
 *
 * Workspaces are caller-allocated device buffers; their first 256 bytes hold
 * a device status word (0 = ok, non-zero = a bounded wait inside a kernel
 * timed out), readable with si_read_status().
 */
#ifndef STREAMINDEX_B200_H
#define STREAMINDEX_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SI_ABI_VERSION 1

#if defined(__GNUC__)
#define SI_API __attribute__((visibility("default")))
#else
#define SI_API
#endif

SI_API int si_abi_version(void);
SI_API const char* si_last_error(void);
/* Synchronises `stream` and copies the workspace's status word to *status_out. */
SI_API int si_read_status(const void* ws, int* status_out, cudaStream_t stream);

/* Self-test of the kernels' bounded waits: launches one CTA that waits on a
 * barrier nothing arrives on; after limit_ns (<= 2 s) the wait gives up,
 * writes status 1 (the "data never arrived" code) to the workspace status
 * word and the kernel returns normally.  No counterpart in the reference. */
SI_API int si_selftest_wait_timeout(void* ws, unsigned long long limit_ns, cudaStream_t stream);

/* Workspace bytes for si_indexer_topk on the current device. */
SI_API size_t si_indexer_topk_ws_bytes(int B, int S, int T, int H, int D, int top_k);

/* Fused lightning-indexer score + streaming top-k.
 * Replaces chunked_indexer_topk (flash_sparse/triton/chunked_indexer.py:47-160)
 * and indexer_score_topk (flash_sparse/triton/indexer_score.py:182-205).
 *   q        [B,S,H,D]  bf16 (fp16 if ab_fp16)     H in {16,32,64,128}, D % 8 == 0, D <= 128
 *   k        [B,T,D]    same dtype as q
 *   w        [B,S,H]    fp32, or bf16 if w_is_bf16
 *   causal_ratio > 0: key t is legal for query s iff t < (s+1)/causal_ratio;
 *   causal_mask (nullable, [B,S,T] bytes, nonzero = legal) used when causal_ratio <= 0;
 *   neither: all keys legal.
 *   out_idx    [B,S,top_k] int64, sorted by score desc then index asc; -1 pads
 *   out_scores [B,S,top_k] fp32; -inf pads
 * Results do not depend on any chunking: the selection is exact. */
SI_API int si_indexer_topk(const void* q, const void* k, const void* w, int w_is_bf16, int ab_fp16, int B, int S, int T,
                    int H, int D, int top_k, int causal_ratio, const uint8_t* causal_mask, int64_t* out_idx,
                    float* out_scores, void* ws, size_t ws_bytes, cudaStream_t stream);

/* si_indexer_topk with two extensions used by S-sharding and profiling.
 *   s_offset: global position of local query 0; the causal limit of local
 *             query s is (s_offset + s + 1) / causal_ratio.  q, w and the
 *             outputs cover only the local queries.
 *   flags:    SI_FLAG_SKIP_SORT leaves out_idx holding the unsorted 64-bit
 *             selection keys (score order-key << 32 | 0xFFFFFFFF - index,
 *             0 = empty) for a later si_topk_row_sort; out_scores untouched. */
#define SI_FLAG_SKIP_SORT 1u
SI_API int si_indexer_topk_ex(const void* q, const void* k, const void* w, int w_is_bf16, int ab_fp16, int B, int S,
                              int T, int H, int D, int top_k, int causal_ratio, const uint8_t* causal_mask,
                              long long s_offset, unsigned flags, int64_t* out_idx, float* out_scores, void* ws,
                              size_t ws_bytes, cudaStream_t stream);

/* si_indexer_topk_ex over strided inputs (the reference passes arbitrary
 * strides to its kernels, flash_sparse/triton/indexer_score.py:162-170; here
 * the last dimension must be contiguous):
 *   q_strides {b, s, h} and k_strides {b, t}: element strides, multiples of 8;
 *   w_strides {b, s, h}: element strides of w;
 *   a null stride array means that tensor is contiguous.
 * q and k are read in place through 4-D / 3-D tensor maps (no copy). */
SI_API int si_indexer_topk_strided(const void* q, const long long* q_strides, const void* k,
                                   const long long* k_strides, const void* w, const long long* w_strides,
                                   int w_is_bf16, int ab_fp16, int B, int S, int T, int H, int D, int top_k,
                                   int causal_ratio, const uint8_t* causal_mask, long long s_offset, unsigned flags,
                                   int64_t* out_idx, float* out_scores, void* ws, size_t ws_bytes,
                                   cudaStream_t stream);

/* Sorts `rows` rows of top_k selection keys (as left by SI_FLAG_SKIP_SORT)
 * descending and decodes them in place into int64 indices (-1 pads) and
 * fp32 scores (-inf pads). */
SI_API int si_topk_row_sort(int64_t* idx_keys, float* out_scores, long long rows, int top_k, cudaStream_t stream);

/* Allocation-free si_indexer_topk.  No counterpart in the reference.
 * For callers that cannot allocate device memory (a host runtime that owns
 * the allocator and forbids plugins from calling cudaMalloc, or a caller that
 * must not allocate while other work is in flight): the workspace is a
 * file-scope device array of si_indexer_topk_noalloc_max_ws_bytes() bytes
 * (16 MiB) held by every GPU that loads the library until process exit.
 * Same arguments and results as si_indexer_topk without ws / ws_bytes.
 *   - Rejects shapes whose workspace exceeds the maximum (-1, message in
 *     si_last_error()); si_indexer_topk_ws_bytes() tells the need.
 *   - The first call on a device resolves the array's device address
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *   - All calls share the one array: calls that overlap on the GPU (other
 *     streams, other host threads) race and corrupt each other's results.
 *     Serialise them on one stream.
 *   - Calls no cudaMalloc / cudaFree; enqueues a 4-byte status memset and the
 *     kernels on `stream`.  The status word is the first int of the array. */
SI_API size_t si_indexer_topk_noalloc_max_ws_bytes(void);
SI_API int si_indexer_topk_noalloc(const void* q, const void* k, const void* w, int w_is_bf16, int ab_fp16, int B,
                                   int S, int T, int H, int D, int top_k, int causal_ratio,
                                   const uint8_t* causal_mask, int64_t* out_idx, float* out_scores,
                                   cudaStream_t stream);
/* Status word of the allocation-free path (0 = ok, non-zero = a bounded wait
 * inside the last si_indexer_topk_noalloc kernel on this device timed out and
 * its results are incomplete).  Synchronises `stream`; allocates nothing. */
SI_API int si_indexer_topk_noalloc_read_status(int* status_out, cudaStream_t stream);

/* Materialised indexer scores, no mask.
 * Replaces indexer_score (flash_sparse/triton/indexer_score.py:123-179).
 *   out [B,S,T] fp32.  ws: at least 256 bytes (status word). */
SI_API int si_indexer_score(const void* q, const void* k, const void* w, int w_is_bf16, int ab_fp16, int B, int S, int T,
                     int H, int D, float* out, void* ws, size_t ws_bytes, cudaStream_t stream);

/* Sparse MQA attention forward with attention sink.
 * Replaces sparse_attn_fwd (flash_sparse/triton/sparse_attn_fwd.py:180-292) and
 * the math of reference_sparse_attn (flash_sparse/reference.py:44-130).
 *   q          [B,S,H,D]   bf16        D % 8 == 0, D <= 896
 *   kv         [B,Nkv,D]   bf16        one shared KV head
 *   attn_sink  [H]         fp32        enters the softmax denominator only
 *   topk_idxs  [B,S,K]     int32       row of kv per slot; -1 (or >= Nkv) = masked
 *   o          [B,S,H,Dv]  bf16        o = softmax(scale * q.kv^T) . kv[..., :Dv]
 *   lse        [B,S,H]     fp32 (nullable)  log(sum exp + exp(sink)); -1e30 if empty
 *   Dv: value width, a multiple of 64 and <= D (512 for the 576/512 MLA layout,
 *       D for the reference's full-width output).  ws: >= 256 bytes. */
SI_API int si_sparse_attn_fwd(const void* q, const void* kv, const float* attn_sink, const int32_t* topk_idxs, int B,
                              int S, int H, int D, int Nkv, int K, int Dv, float softmax_scale, void* o, float* lse,
                              void* ws, size_t ws_bytes, cudaStream_t stream);

/* si_sparse_attn_fwd over a kv split in two tensors, as the CSA layer reads
 * cat[kv; kv_compressed] (flash_sparse/csa.py:199) without building it:
 * index v < Nkv reads kv[b, v], index v >= Nkv reads kv2[b, v - Nkv]. */
SI_API int si_sparse_attn_fwd_kv2(const void* q, const void* kv, int Nkv, const void* kv2, int Nkv2,
                                  const float* attn_sink, const int32_t* topk_idxs, int B, int S, int H, int D, int K,
                                  int Dv, float softmax_scale, void* o, float* lse, void* ws, size_t ws_bytes,
                                  cudaStream_t stream);

/* FP8 KV row format (the V4 production KV row, described in the reference's
 * docs/ir_analysis.md:45-55; its quantisation is the reference's
 * act_quant_simulate, flash_sparse/utils/quantization.py:19-36, at block 64):
 *   [n_nope e4m3 | n_nope/64 fp32 block scales | pad to 16 B | D-n_nope bf16 | pad to 16 B]
 * n_nope a multiple of 64 in [64,512], 0 < D - n_nope <= 64.  672 bytes per
 * row at D=576/n_nope=512 (vs 1152 in bf16); 608 at the V4-Pro 512/448 split.
 * si_fp8_kv_row_bytes returns the row size (-1 for an unsupported split). */
SI_API int si_fp8_kv_row_bytes(int D, int n_nope);
/* bf16 kv [rows, D] -> FP8 rows [rows, row_bytes].  Per 64-dim block:
 * amax = max(max|x|, 1e-4), scale = bf16(amax/448), e = e4m3(clamp(bf16(x/scale), +-448)),
 * evaluated in bf16 like the simulation, so bf16(float(e) * scale) equals
 * act_quant_simulate(kv[..., :n_nope], 64) exactly. */
SI_API int si_kv_quant_fp8(const void* kv, long long rows, int D, int n_nope, void* out, cudaStream_t stream);
/* si_sparse_attn_fwd_kv2 over FP8 KV rows (kv2_rows / Nkv2 optional, same
 * format): the gather dequantises each selected row, value = bf16(float(e) *
 * scale), into the bf16 tile the tensor cores read, so the result equals
 * sparse attention over the dequantised kv (the reference's FP8 simulation
 * path, flash_sparse/reference.py:44-130 on act_quant_simulate(kv)) while each
 * gathered row moves row_bytes instead of 2*D bytes.  q and o stay bf16. */
SI_API int si_sparse_attn_fwd_fp8kv(const void* q, const void* kv_rows, int Nkv, const void* kv2_rows, int Nkv2,
                                    int n_nope, const float* attn_sink, const int32_t* topk_idxs, int B, int S, int H,
                                    int D, int K, int Dv, float softmax_scale, void* o, float* lse, void* ws,
                                    size_t ws_bytes, cudaStream_t stream);

/* CSA sparse attention with the index list built inside the kernel.
 * Replaces the index concatenation of flash_csa_forward
 * (flash_sparse/csa.py:176-179, window of flash_sparse/reference.py:460-475)
 * followed by its sparse_attn call (flash_sparse/csa.py:199-205), without
 * materialising the [B,S,n_win+top_k] int32 list or cat[kv; kv_comp]:
 *   q        [B,S,H,D]   bf16   the query slice [s_offset, s_offset+S) of a
 *                               sequence of S_total tokens (S_total = S and
 *                               s_offset = 0 for a whole sequence)
 *   kv       [B,S_total,D]  bf16     window rows
 *   kv_comp  [B,T,D]        bf16     compressed rows
 *   comp_idx [B,S,top_k]    int64    compressed top-k picks (-1 = empty), as
 *                                    returned by si_indexer_topk_ex(s_offset)
 * Slot j < n_win reads kv[p - n_win + 1 + j] for global position p (masked
 * if negative); slot n_win + j reads kv_comp[comp_idx[.., j]] (masked if -1).
 * Everything else as si_sparse_attn_fwd. */
SI_API int si_csa_sparse_attn_fwd(const void* q, const void* kv, int S_total, const void* kv_comp, int T,
                                  const float* attn_sink, const int64_t* comp_idx, int top_k, int n_win,
                                  long long s_offset, int B, int S, int H, int D, int Dv, float softmax_scale, void* o,
                                  float* lse, void* ws, size_t ws_bytes, cudaStream_t stream);

/* si_sparse_attn_fwd_kv2 with the element type of q / kv / o chosen by dtype:
 * 0 = bf16, 1 = fp16 (the reference accepts either,
 * flash_sparse/triton/sparse_attn_fwd.py:207).  In fp16 the probabilities P
 * enter the P.V product as fp16 (both tensor-core operands share one type). */
SI_API int si_sparse_attn_fwd_ex(const void* q, const void* kv, int Nkv, const void* kv2, int Nkv2,
                                 const float* attn_sink, const int32_t* topk_idxs, int B, int S, int H, int D, int K,
                                 int Dv, float softmax_scale, int dtype, void* o, float* lse, void* ws,
                                 size_t ws_bytes, cudaStream_t stream);

/* si_sparse_attn_fwd_ex with a strided q (element strides {b, s, h}, multiples
 * of 8, last dimension contiguous; null = contiguous), read in place through a
 * 4-D tensor map (sparse_attn_fwd.py:267-270 of the reference passes q's
 * strides to its kernel).  kv, indices and outputs are contiguous. */
SI_API int si_sparse_attn_fwd_strided(const void* q, const long long* q_strides, const void* kv, int Nkv,
                                      const void* kv2, int Nkv2, const float* attn_sink, const int32_t* topk_idxs,
                                      int B, int S, int H, int D, int K, int Dv, float softmax_scale, int dtype,
                                      void* o, float* lse, void* ws, size_t ws_bytes, cudaStream_t stream);

/* Sparse MQA attention backward with attention sink.
 * Replaces sparse_attn_bwd (flash_sparse/triton/sparse_attn_bwd.py:286-416):
 *   inputs as si_sparse_attn_fwd plus o [B,S,H,Dv] bf16 and lse [B,S,H] fp32
 *   from the forward and dout [B,S,H,Dv] bf16;
 *   dq      [B,S,H,D]  bf16   (written; zero it first when K == 0)
 *   dkv_f32 [B,Nkv,D]  fp32   accumulated with atomic adds: zero it first
 *   dsink   [H]        fp32   accumulated with atomic adds: zero it first
 * D in {64,128,256,512,576}; Dv a multiple of 32, <= D (value = first Dv dims).
 * bf16 only. */
SI_API int si_sparse_attn_bwd(const void* q, const void* kv, const float* attn_sink, const int32_t* topk_idxs,
                              const void* o, const float* lse, const void* dout, int B, int S, int H, int D, int Nkv,
                              int K, int Dv, float softmax_scale, void* dq, float* dkv_f32, float* dsink,
                              cudaStream_t stream);

/* Top-k of a materialised score matrix [B,S,T] fp32 with the causal limit
 * t < (s+1)/causal_ratio (<= 0: none); same output contract as si_indexer_topk.
 * Replaces the masked_fill + topk + post-mask of build_csa_topk_idxs
 * (flash_sparse/csa.py:55-69) and of indexer_score_topk with a causal mask
 * (flash_sparse/triton/indexer_score.py:200-205). */
SI_API size_t si_scores_topk_ws_bytes(int B, int S, int top_k);
SI_API int si_scores_topk(const float* scores, int B, int S, int T, int top_k, int causal_ratio, int64_t* out_idx,
                          float* out_scores, void* ws, size_t ws_bytes, cudaStream_t stream);

/* si_scores_topk with an optional explicit [B,S,T] byte mask (nonzero = legal),
 * applied together with the causal ratio (<= 0: none).  Replaces the
 * masked_fill + topk of reference_csa_forward's causal_mask_for_compressed
 * (flash_sparse/reference.py:389-397). */
SI_API int si_scores_topk_mask(const float* scores, int B, int S, int T, int top_k, int causal_ratio,
                               const uint8_t* causal_mask, int64_t* out_idx, float* out_scores, void* ws,
                               size_t ws_bytes, cudaStream_t stream);

/* CSA attention index list [B,S,n_win+top_k] int32: sliding window then
 * compressed picks offset by S (-1 kept).  Replaces _build_sliding_window_idxs
 * (flash_sparse/reference.py:460-475) + the concatenation of
 * flash_sparse/csa.py:76-83 / :176-179.  comp_idx: [B,S,top_k] int64. */
SI_API int si_csa_build_idx(const int64_t* comp_idx, int B, int S, int top_k, int n_win, int32_t* out,
                            cudaStream_t stream);

/* si_csa_build_idx for a query slice: local rows [0,S) are global positions
 * s_offset + s of a sequence of S_total tokens (window and causality use the
 * global position; compressed picks are offset by S_total).  Used by the
 * S-sharded CSA forward. */
SI_API int si_csa_build_idx_ex(const int64_t* comp_idx, int B, int S, long long s_offset, int S_total, int top_k,
                               int n_win, int32_t* out, cudaStream_t stream);

/* HCA attention index list [B,S,n_win+n_comp] int32: sliding window, then all
 * compressed blocks legal for the query ((i+1)*m_prime - 1 <= s) offset by S,
 * else -1.  Replaces build_hca_topk_idxs (flash_sparse/hca.py:24-51). */
SI_API int si_hca_build_idx(int B, int S, int n_win, int n_comp, int m_prime, int32_t* out, cudaStream_t stream);

/* Softmax-gated token compressor [B,S,C] -> [B,S/m,C] (fp32 math; bf16 or fp32
 * tensors).  Replaces reference_token_compressor (flash_sparse/reference.py:176-272):
 * overlap = 0: weights softmax_m(z_a + b_a), b_a [m,C];
 * overlap = 1: joint 2m-way softmax over the block's a-stream and the previous
 *              block's b-stream (c_b, z_b, b_b [m,C]); block 0 has no b-stream. */
SI_API int si_token_compressor(const void* c_a, const void* z_a, const void* b_a, const void* c_b, const void* z_b,
                               const void* b_b, int B, int S, int C, int m, int overlap, int is_bf16, void* out,
                               cudaStream_t stream);

/* Mean-pool compressor [B,S,C] bf16 -> [B,S/m,C] bf16 (trailing S % m tokens
 * dropped).  Equals reference_token_compressor(overlap=False) with zero scores
 * and bias (flash_sparse/reference.py:234-240). */
SI_API int si_mean_pool(const void* x, int B, int S, int C, int m, void* out, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif

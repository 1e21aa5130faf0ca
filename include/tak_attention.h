/*
 * tak_attention.h -- C ABI of the B200 (sm_100a) attention hot path.
 *
 * Drop-in native backend for suluner/triton-ascend-kernels' attention/*.py.
 * Each entry point below replaces one Triton launch (or host-side loop) of the
 * reference; the file:line of the interface it replaces is cited with it.
 * The Python modules of this package (attention/*.py, same names and call
 * signatures as the reference's) bind these symbols with ctypes.
 *
 * Conventions
 *   - Every pointer is a device pointer (CUDA global memory) unless stated.
 *   - Strides are in elements, int64, one per tensor dimension, passed as a
 *     pointer to a small host array (e.g. q_strides[3] for q[T, H, D]).
 *   - dtype: TAK_F16, TAK_BF16 or TAK_F32; q, k, v and out share it.
 *   - Index tensors (cu_seqlens, block tables, top-k rows, offsets) are int32.
 *   - cu_seqlens is cumulative: cu_seqlens[0] = 0, non-decreasing, last entry
 *     <= the row count of the tensors it indexes.  Kernels read it on the
 *     device and do not check this (nor does the reference).
 *   - lse (optional, may be NULL) is float32 [rows, H] contiguous: the natural
 *     log of the softmax denominator, sink term included; -inf for a row with
 *     no key.  The reference has no LSE output; it is an addition.
 *   - stream is a cudaStream_t (NULL = legacy default stream).  Calls are
 *     asynchronous; no entry point synchronises the device.
 *   - Return value: 0 on success, nonzero on error (1 = invalid argument,
 *     2 = unsupported shape, 3 = CUDA error); tak_last_error() describes the
 *     last error of the calling thread.  No entry point aborts the process.
 */
#ifndef TAK_ATTENTION_H_
#define TAK_ATTENTION_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { TAK_F16 = 0, TAK_BF16 = 1, TAK_F32 = 2 };

/* Library version, e.g. "tak-b200 0.1". */
const char* tak_version(void);

/* Message of the last error returned on the calling thread ("" if none). */
const char* tak_last_error(void);

/* Synchronises `stream`, returns the device-side error word (0 = none,
 * 1 = a bounded wait inside a kernel timed out, 2 = TMEM allocation failed)
 * and clears it.  For tests and diagnostics, not for the hot path. */
int tak_read_device_error(void* stream);

/* Kernel selection for cross-checking: 0 = automatic (tensor-core kernels
 * where the shape allows), 1 = always the generic CUDA-core kernels.
 * Process-wide; returns the previous value. */
int tak_set_kernel_path(int path);

/* Name of the main kernel that the calling thread's last attention or
 * pooling call launched: "prefill_tc", "prefill_generic", "sparse_tc",
 * "sparse_generic", "paged_decode_tc", "paged_decode_generic",
 * "compress_bulk", "compress_dual", "compress_csa_hca", "compress_stream",
 * "compress_split" or "compress_rows"; "" when the call launched nothing (an
 * empty problem, an error).  Lets a caller see whether a shape took the
 * tensor-core kernels or fell back to the CUDA-core ones. */
const char* tak_last_kernel(void);

/*
 * Varlen flash prefill.  Replaces flash_attention_prefill(q, k, v, cu_seqlens,
 * causal) of attention/flash_attention_prefill.py:108-171 (Triton launch at
 * :158).  q [T,H,D], k/v [T,H_kv,D], out [T,H,D]; cu_seqlens [num_seqs+1].
 * scale is the softmax scale (the reference uses 1/sqrt(D), :136).
 * No host synchronisation: the (sequence, row-block) schedule the reference
 * builds on the host (:144-153) is derived on the device.
 */
int tak_flash_attention_prefill(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                const void* v, const int64_t* v_strides, const int32_t* cu_seqlens,
                                int64_t num_seqs, void* out, const int64_t* out_strides, float* lse,
                                int64_t total_tokens, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                                float scale, int causal, int dtype, void* stream);

/*
 * Paged decode.  Replaces paged_attention_decode(q, k_cache, v_cache,
 * block_tables, context_lens, block_size, block_n) of
 * attention/paged_attention_decode.py:104-151 (Triton launch at :138).
 * q [B,H,D], k_cache/v_cache [num_blocks,H_kv,cache_rows,D],
 * block_tables [B,max_blocks], context_lens [B], out [B,H,D].
 * workspace: device scratch of at least tak_paged_attention_decode_workspace_size()
 * bytes for the split-KV partials (may be NULL if that size is 0); no
 * initialisation needed.  Calls that share a workspace must not overlap on the
 * GPU (issue them on one stream).  Context rows past the block table
 * (ctx > max_blocks * block_size) are ignored; a block-table entry outside
 * [0, num_blocks) is never read: its rows count as zero keys and values
 * (score 0, value 0).
 * split_pages: pages per split-KV work unit, 0 = automatic.
 */
size_t tak_paged_attention_decode_workspace_size(int64_t num_seqs, int64_t num_q_heads, int64_t num_kv_heads,
                                                 int64_t head_dim, int64_t block_size, int64_t max_blocks,
                                                 int split_pages);
int tak_paged_attention_decode(const void* q, const int64_t* q_strides, const void* k_cache,
                               const int64_t* k_strides, const void* v_cache, const int64_t* v_strides,
                               const int32_t* block_tables, const int64_t* bt_strides, const int32_t* context_lens,
                               void* out, const int64_t* out_strides, float* lse, int64_t num_seqs,
                               int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, int64_t block_size,
                               int64_t max_blocks, int64_t num_blocks, int64_t cache_rows, float scale, int dtype,
                               void* workspace, size_t workspace_bytes, int split_pages, void* stream);

/*
 * Paged decode that allocates nothing.  No counterpart in the reference: it
 * exists for callers that cannot provide the workspace above -- code where a
 * cudaMalloc is not allowed or would stall the device, hosts whose device
 * memory is owned by a framework allocator, bindings without a device
 * allocator.  Same arguments and results as tak_paged_attention_decode minus
 * the workspace: the split-KV scratch is a 32 MiB array inside the library
 * (held by every GPU that loads the library until exit).  Sizes whose scratch
 * would exceed 32 MiB are rejected with status 2 (a larger split_pages lowers
 * the need; fp32 caches, unaligned strides and single-split sizes run
 * kernels that need no scratch and are never rejected for size).  Arguments
 * are validated as for tak_paged_attention_decode.  All calls on a GPU share
 * the array: calls that overlap on the GPU race; nothing in it needs clearing
 * between calls.  The first call with a given GPU current, and the first after
 * that GPU's context was recreated (cudaDeviceReset), looks up the array's
 * device address; make those calls before any stream capture.
 */
int tak_paged_attention_decode_static_scratch(const void* q, const int64_t* q_strides, const void* k_cache,
                                              const int64_t* k_strides, const void* v_cache,
                                              const int64_t* v_strides, const int32_t* block_tables,
                                              const int64_t* bt_strides, const int32_t* context_lens, void* out,
                                              const int64_t* out_strides, float* lse, int64_t num_seqs,
                                              int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                                              int64_t block_size, int64_t max_blocks, int64_t num_blocks,
                                              int64_t cache_rows, float scale, int dtype, int split_pages,
                                              void* stream);

/*
 * Top-k sparse prefill with per-head sink logits.  Replaces
 * sparse_attn_prefill(q, k, v, topk_idxs, cu_seqlens, attn_sink) of
 * attention/sparse_attn_fwd.py:263-314 (Triton launch at :298).
 * q [T,H,Dqk], k [rows,H_kv,Dqk], v [rows,H_kv,Dv] (Dv may differ from Dqk:
 * the reference requires equal shapes, :279), topk_idxs [T,k_topk] (< 0 =
 * masked; >= rows is treated as masked too), attn_sink [H] float32 or NULL,
 * out [T,H,Dv].  cu_seqlens does not enter the math (as in the reference
 * kernel, whose grid covers every token, :296) and is not an argument.
 */
int tak_sparse_attn_prefill(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                            const void* v, const int64_t* v_strides, const int32_t* topk_idxs,
                            const int64_t* topk_strides, const float* attn_sink, void* out,
                            const int64_t* out_strides, float* lse, int64_t total_tokens, int64_t num_q_heads,
                            int64_t num_kv_heads, int64_t head_dim, int64_t head_dim_v, int64_t kv_rows,
                            int64_t k_topk, float scale, int dtype, void* stream);

/*
 * Sparse prefill over two row sources without concatenating them: index j <
 * kv_rows addresses row j of k/v [kv_rows, H_kv, D(v)], index j >= kv_rows
 * row j - kv_rows of k2/v2 [kv2_rows, H_kv, D(v)] (same head dims and
 * head-dim strides); every other argument as tak_sparse_attn_prefill.
 * Replaces the torch.cat([k, compressed_k]) / torch.cat([v, compressed_v])
 * and the sparse_attn_prefill call of csa_prefill_forward
 * (attention/csa.py:191-194) and hca_prefill_forward (attention/hca.py:173-176),
 * whose index rows address the concatenation (entries total_tokens +
 * comp_offsets[s] + i).  v/v2 being prefix views of k/k2 (one latent tensor
 * as K and V) lets each gathered row serve both.
 */
int tak_sparse_attn_prefill_2src(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                 const void* v, const int64_t* v_strides, int64_t kv_rows, const void* k2,
                                 const int64_t* k2_strides, const void* v2, const int64_t* v2_strides,
                                 int64_t kv2_rows, const int32_t* topk_idxs, const int64_t* topk_strides,
                                 const float* attn_sink, void* out, const int64_t* out_strides, float* lse,
                                 int64_t total_tokens, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                                 int64_t head_dim_v, int64_t k_topk, float scale, int dtype, void* stream);

/*
 * Top-k sparse decode over a paged window plus compressed rows.  Replaces
 * sparse_attn_decode(q, k_cache, v_cache, compressed_k, compressed_v,
 * block_tables, topk_idxs, context_lens, num_win, block_size, attn_sink) of
 * attention/sparse_attn_fwd.py:317-382 (Triton launch at :359), with its
 * slot-position rule (:151-210): slots < num_win address the paged cache and
 * need 0 <= idx < ctx; later slots address compressed rows idx - ctx.
 * block_tables is [num_seqs, max_blocks] and the caches have num_blocks pages.
 * A window slot is masked unless it also lies inside its block-table row
 * (idx < max_blocks * block_size) and that row's entry is a page of the cache
 * (0 <= page < num_blocks); the reference's kernel reads past both unchecked
 * (:159-170).
 */
int tak_sparse_attn_decode(const void* q, const int64_t* q_strides, const void* k_cache, const int64_t* k_strides,
                           const void* v_cache, const int64_t* v_strides, const void* compressed_k,
                           const int64_t* ck_strides, const void* compressed_v, const int64_t* cv_strides,
                           const int32_t* block_tables, const int64_t* bt_strides, const int32_t* topk_idxs,
                           const int64_t* topk_strides, const int32_t* context_lens, const float* attn_sink,
                           void* out, const int64_t* out_strides, float* lse, int64_t num_seqs,
                           int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, int64_t head_dim_v,
                           int64_t num_compressed, int64_t k_topk, int64_t num_win, int64_t block_size,
                           int64_t max_blocks, int64_t num_blocks, float scale, int dtype, void* stream);

/* token -> sequence map (0 for tokens outside every sequence).  Replaces
 * build_token_to_seq of attention/sparse_attn_fwd.py:253-260. */
int tak_build_token_to_seq(const int32_t* cu_seqlens, int64_t num_seqs, int64_t total_tokens, int32_t* out,
                           void* stream);

/*
 * Window pooling of K and V into compressed slots.  Replaces
 * compress_kv_overlap (attention/csa.py:9-69; window = 2m, stride = m) and
 * compress_kv_simple (attention/hca.py:9-69; window = stride = m').
 * k [T,H_kv,D], v [T,H_kv,Dv], comp_offsets [num_seqs+1] (computed by the
 * caller: max(1, ceil(L/stride)) slots per non-empty sequence), compressed
 * outputs [num_compressed,H_kv,D(v)].  gate: NULL = plain mean (the
 * reference); else float32 [T] logits and each slot is the softmax(gate)-
 * weighted sum of its window (an addition, no counterpart in the reference).
 * v = NULL (with compressed_v = NULL and head_dim_v = 0; v_strides and
 * cv_strides are then ignored) pools K alone: for callers whose V is a view
 * of K, whose compressed V is then the same view of compressed K (an
 * addition; the reference always pools both).
 */
int tak_compress_kv(const void* k, const int64_t* k_strides, const void* v, const int64_t* v_strides,
                    const float* gate, int64_t gate_stride, const int32_t* cu_seqlens, const int32_t* comp_offsets,
                    int64_t num_seqs, int64_t num_compressed, void* compressed_k, const int64_t* ck_strides,
                    void* compressed_v, const int64_t* cv_strides, int64_t num_kv_heads, int64_t head_dim,
                    int64_t head_dim_v, int64_t stride, int64_t window, int dtype, void* stream);

/*
 * Same pooling, reading each sequence's first context_lens[s] rows straight
 * from a paged cache [num_blocks,H_kv,P,D] through block_tables
 * [num_seqs, max_blocks].  Replaces the page gather + compress of
 * csa_decode_forward (attention/csa.py:225-256) and hca_decode_forward
 * (attention/hca.py:204-232).  gate (optional) is float32 [num_blocks, P]
 * with strides gate_strides[2].  v_cache = NULL pools K alone, as for
 * tak_compress_kv.  A context row past its block-table row (row >=
 * max_blocks * P), or on a page id outside [0, num_blocks), is never read: it
 * pools as a zero row with gate logit 0 (the reference's gather raises an
 * IndexError past the row, attention/csa.py:229-245, and reads any page id).
 */
int tak_compress_kv_paged(const void* k_cache, const int64_t* k_strides, const void* v_cache,
                          const int64_t* v_strides, const float* gate, const int64_t* gate_strides,
                          const int32_t* block_tables, const int64_t* bt_strides, const int32_t* context_lens,
                          int64_t block_size, int64_t max_blocks, int64_t num_blocks, const int32_t* comp_offsets,
                          int64_t num_seqs, int64_t num_compressed, void* compressed_k, const int64_t* ck_strides,
                          void* compressed_v, const int64_t* cv_strides, int64_t num_kv_heads, int64_t head_dim,
                          int64_t head_dim_v, int64_t stride, int64_t window, int dtype, void* stream);

/* CSA and HCA pooling of the same TND K/V (and gate) in one pass: the CSA
 * outputs of compress_kv_overlap (attention/csa.py:9-69, window 2m, stride m,
 * offsets csa_offsets) and the HCA outputs of compress_kv_simple
 * (attention/hca.py:9-69, window = stride = m_prime, offsets hca_offsets),
 * which the reference computes with two separate passes over K/V.  One pass
 * runs on the bulk-copy kernel when the inputs are 16-bit with strides in
 * multiples of 8 elements, m_prime is a multiple of m, m <= 64, m_prime + m
 * <= 2048 and head_dim + head_dim_v <= 2048; else on the TMA-box kernel when
 * m_prime + m <= 256 and the head dims are multiples of 128; other shapes
 * (fp32 among them) run as two tak_compress_kv passes with the same results.
 * total_tokens = rows of K/V/gate.  The bulk-copy kernel is launched with
 * programmatic stream serialization: it waits in-kernel for the grid before it
 * on the stream (whose outputs may be its inputs) and lets the grid after it be
 * scheduled while it drains; a following launch without that attribute waits
 * for it as usual. */
int tak_compress_kv_csa_hca(const void* k, const int64_t* k_strides, const void* v, const int64_t* v_strides,
                            const float* gate, int64_t gate_stride, const int32_t* cu_seqlens, int64_t num_seqs,
                            int64_t total_tokens, const int32_t* csa_offsets, int64_t num_csa, void* csa_k,
                            const int64_t* csa_k_strides, void* csa_v, const int64_t* csa_v_strides,
                            const int32_t* hca_offsets, int64_t num_hca, void* hca_k, const int64_t* hca_k_strides,
                            void* hca_v, const int64_t* hca_v_strides, int64_t num_kv_heads, int64_t head_dim,
                            int64_t head_dim_v, int64_t m, int64_t m_prime, int dtype, void* stream);

/* Sliding-window columns [0, n_win) of prefill index rows (row stride ld).
 * Replaces attention/csa.py:108-117 (same rule at hca.py:133-137). */
int tak_build_window_idxs(const int32_t* cu_seqlens, int64_t num_seqs, int64_t total_tokens, int64_t n_win,
                          int32_t* out, int64_t ld, void* stream);

/* Full HCA prefill index rows [T, n_win + max_n_comp].  Replaces
 * build_hca_topk_idxs of attention/hca.py:76-146 (max_n_comp from :103-115,
 * computed by the caller). */
int tak_build_hca_topk_idxs(const int32_t* cu_seqlens, const int32_t* comp_offsets, int64_t num_seqs,
                            int64_t total_tokens, int64_t n_win, int64_t max_n_comp, int64_t m_prime,
                            int32_t* out, int64_t ld, void* stream);

/* Decode index rows [B, n_win + n_comp_cols]: window ctx - n_win + wi, and
 * with m_prime > 0 the HCA compressed part (attention/hca.py:245-259); with
 * m_prime == 0 the compressed columns are -1 for tak_csa_indexer_topk to fill
 * (attention/csa.py:263-276). */
int tak_build_decode_topk_idxs(const int32_t* context_lens, const int32_t* comp_offsets, int64_t num_seqs,
                               int64_t n_win, int64_t n_comp_cols, int64_t m_prime, int32_t* out, int64_t ld,
                               void* stream);

/*
 * comp_offsets [num_seqs + 1] (int32, device) computed on the device from
 * per-sequence lengths (is_cu = 0: lens[num_seqs], e.g. context_lens) or from
 * cu_seqlens (is_cu = 1: lens[num_seqs + 1]): max(1, ceil(L / stride)) slots
 * per non-empty sequence, cumulative -- the comp_offsets of
 * compress_kv_overlap / compress_kv_simple (attention/csa.py:38-59,
 * attention/hca.py:38-59), which the reference builds on the host.  With
 * capacity >= 0 the offsets are clamped to it and a larger total records
 * device error 3 (tak_read_device_error); the pooling, index and attention
 * entry points then touch no slot beyond the capacity.  Lets the decode
 * wrappers run without reading lengths on the host (an addition).
 */
int tak_comp_offsets(const int32_t* lens, int64_t num_seqs, int is_cu, int64_t stride, int64_t capacity,
                     int32_t* comp_offsets, void* stream);

/*
 * CSA Lightning indexer: columns [n_win, n_win + top_k) of the index rows.
 * Replaces the indexer of build_csa_topk_idxs (attention/csa.py:119-164) and
 * of csa_decode_forward (:278-302).  Prefill (cu_seqlens != NULL): one row per
 * token, entry = total_tokens + comp_offsets[s] + slot.  Decode (cu_seqlens ==
 * NULL, context_lens given): one row per sequence, entry = ctx +
 * comp_offsets[s] + slot.  Scores are unscaled q.k~ of the last query head
 * against the last KV head (the head whose choice survives in the reference),
 * rounded to dtype; slot causal iff slot*m < position; descending score, ties
 * to the lower slot; masked slots appended in ascending order when fewer than
 * min(top_k, n_c) are causal.  max_comp_per_seq bounds n_c (<= 51200).
 * workspace (may be NULL) of at least tak_csa_indexer_workspace_size bytes
 * (for the rows: total_tokens in prefill, num_seqs in decode) holds the
 * scores before the selection: prefill rows compute them as tensor-core GEMM
 * tiles (the reference's matmul, CSA:144), decode rows split each row's dot
 * products over many CTAs; without it one CTA per row scores on CUDA cores.
 * compressed_rows = rows of compressed_k.
 */
int tak_csa_indexer_topk(const void* q, const int64_t* q_strides, const void* compressed_k,
                         const int64_t* ck_strides, const int32_t* cu_seqlens, const int32_t* context_lens,
                         const int32_t* comp_offsets, int64_t num_seqs, int64_t total_tokens, int64_t num_q_heads,
                         int64_t num_kv_heads, int64_t head_dim, int64_t n_win, int64_t top_k, int64_t m,
                         int64_t max_comp_per_seq, int32_t* out, int64_t ld, int dtype, void* workspace,
                         int64_t workspace_bytes, int64_t compressed_rows, void* stream);

/* Bytes of the score scratch of tak_csa_indexer_topk for `total_tokens` rows
 * (prefill tokens, or decode sequences): rows x max_comp_per_seq rounded up
 * to 128 x the element size. */
int64_t tak_csa_indexer_workspace_size(int64_t total_tokens, int64_t max_comp_per_seq, int dtype);

#ifdef __cplusplus
}
#endif

#endif /* TAK_ATTENTION_H_ */

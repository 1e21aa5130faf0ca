// Internal host-side interface between the C-ABI layer (capi.cu) and the
// kernel files.  Argument structs carry raw device pointers, sizes and element
// strides exactly as the extern "C" entry points receive them.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace tak {

// error reporting (capi.cu): stores a message for tak_last_error(), returns code
int set_error(int code, const char* msg);
// records, for tak_last_kernel(), the main kernel the calling thread's current
// entry point launched (a string literal)
void note_kernel(const char* name);
// cudaGetLastError after a launch: 0, or status 3 with the CUDA error as message
int check_launch(const char* what);
int num_sms();
// cudaFuncAttributeMaxDynamicSharedMemorySize of `func` on the current device,
// raised to at least `bytes` (set once per device and kernel, cached)
int ensure_smem_attr(const void* func, int bytes);
// cuTensorMapEncodeTiled through the runtime's driver entry point
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, const uint32_t* elem_strides,
                 CUtensorMapSwizzle swizzle);

struct PagedDecodeArgs {
  const void* q; int64_t sq[3];
  const void* k_cache; int64_t sk[4];
  const void* v_cache; int64_t sv[4];
  const int32_t* block_tables; int64_t sbt[2];
  const int32_t* context_lens;
  void* out; int64_t so[3];
  float* lse;
  int num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, max_blocks;
  int64_t num_blocks, cache_rows;
  float scale;
  int dtype;
  void* workspace; size_t workspace_bytes;
  int split_pages;    // 0 = automatic
  int force_generic;  // 1 = use the generic kernel (tests)
};
size_t paged_decode_workspace_bytes(const PagedDecodeArgs& a);
// Workspace bytes paged_decode_launch will use for these arguments: 0 when
// the generic kernel runs or every sequence fits one split.
size_t paged_decode_required_workspace(const PagedDecodeArgs& a);
int paged_decode_launch(const PagedDecodeArgs& a, cudaStream_t st);
// Argument validation and filling shared by the decode entry points (capi.cu).
int make_paged_decode_args(PagedDecodeArgs* out_args, const void* q, const int64_t* q_strides, const void* k_cache,
                           const int64_t* k_strides, const void* v_cache, const int64_t* v_strides,
                           const int32_t* block_tables, const int64_t* bt_strides, const int32_t* context_lens,
                           void* out, const int64_t* out_strides, float* lse, int64_t num_seqs,
                           int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, int64_t block_size,
                           int64_t max_blocks, int64_t num_blocks, int64_t cache_rows, float scale, int dtype,
                           int split_pages);

struct PrefillArgs {
  const void* q; int64_t sq[3];
  const void* k; int64_t sk[3];
  const void* v; int64_t sv[3];
  const int32_t* cu_seqlens;
  void* out; int64_t so[3];
  float* lse;
  int num_seqs, total_tokens, num_q_heads, num_kv_heads, head_dim, head_dim_v;
  float scale;
  int causal;
  int dtype;
  int force_generic;
};
int prefill_launch(const PrefillArgs& a, cudaStream_t st);

// Sparse attention, prefill (flat K/V rows) and decode (paged window + flat
// compressed rows) forms share one argument struct.
struct SparseArgs {
  const void* q; int64_t sq[3];
  // prefill: k/v rows [rows, H_kv, D]; decode: the paged caches
  const void* k; int64_t sk[4];
  const void* v; int64_t sv[4];
  // decode: the compressed rows; prefill: the second row source (see rows1)
  const void* ck; int64_t sck[3];
  const void* cv; int64_t scv[3];
  const int32_t* block_tables; int64_t sbt[2];
  const int32_t* context_lens;
  int64_t num_compressed;
  int num_win, block_size;
  int max_blocks;      // block-table width: window rows past max_blocks * block_size are masked
  int64_t num_blocks;  // pages of the cache: a window row on a page id outside [0, num_blocks) is masked
  // both
  const int32_t* topk; int64_t stk[2];
  const float* sink;
  void* out; int64_t so[3];
  float* lse;
  int num_tokens, num_q_heads, num_kv_heads, head_dim, head_dim_v, k_topk;
  int64_t kv_rows;
  // prefill with two row sources: rows [0, rows1) of k/v, then rows
  // [rows1, kv_rows) as rows 0.. of ck/cv (the compressed rows); rows1 ==
  // kv_rows when there is one source
  int64_t rows1;
  float scale;
  int dtype;
  int decode;
  int force_generic;
};
int sparse_launch(const SparseArgs& a, cudaStream_t st);

struct CompressArgs {
  const void* k; int64_t sk[4];
  const void* v; int64_t sv[4];
  const float* gate; int64_t sg[2];   // [T] (TND) or [num_blocks, P] (paged); may be null
  // TND rows: row r of sequence s is token cu_seqlens[s] + r.
  const int32_t* cu_seqlens;
  // paged rows (cu_seqlens == null): page block_tables[s, r / P], offset r % P
  const int32_t* block_tables; int64_t sbt[2];
  const int32_t* context_lens;
  int block_size;
  int max_blocks;      // block-table width (paged)
  int64_t num_blocks;  // pages of the cache (paged); rows past the table or on pages outside it read as zeros
  const int32_t* comp_offsets;
  int num_seqs;
  int64_t num_compressed;
  void* ck; int64_t sck[3];
  void* cv; int64_t scv[3];
  int num_kv_heads, head_dim, head_dim_v;
  int stride, window;
  int dtype;
  int64_t total_rows;  // TND token count (only the fused CSA + HCA launch reads it)
};
// Page holding row r of paged sequence s, or -1 when the row lies past the
// sequence's block-table row or the table names a page outside the cache
// (such rows pool as zero rows with gate logit 0).
__device__ __forceinline__ int64_t paged_row_page(const CompressArgs& a, int s, int r) {
  const int pg = r / a.block_size;
  if (pg >= a.max_blocks) return -1;
  const int64_t page = a.block_tables[s * a.sbt[0] + static_cast<int64_t>(pg) * a.sbt[1]];
  return (page >= 0 && page < a.num_blocks) ? page : -1;
}

int compress_launch(const CompressArgs& a, cudaStream_t st);
// Plain-mean pooling streamed through shared memory by bulk copies (16-bit
// rows, strides in multiples of 8 elements, window = stride or 2 * stride, no
// gate).  Returns false, launching nothing, for other shapes; *err is the
// launch status when it returns true.
bool compress_bulk_launch(const CompressArgs& a, cudaStream_t st, int* err);
// CSA + HCA pooling of the same TND rows in one pass on the bulk-copy
// pipeline (one CTA per HCA slot); false (nothing launched) when it does not apply.
bool compress_dual_launch(const CompressArgs& csa, const CompressArgs& hca, cudaStream_t st, int* err);
// CSA (window 2m, stride m) and HCA (window = stride = m') pooling of the same
// K/V/gate in one pass; falls back to two compress_launch calls for shapes the
// fused kernel does not take.
int compress_csa_hca_launch(const CompressArgs& csa, const CompressArgs& hca, cudaStream_t st);

int token_to_seq_launch(const int32_t* cu, int num_seqs, int total_tokens, int32_t* out, cudaStream_t st);
int window_idxs_launch(const int32_t* cu, int num_seqs, int total_tokens, int n_win, int32_t* out, int64_t ld,
                       cudaStream_t st);
int hca_idxs_launch(const int32_t* cu, const int32_t* offs, int num_seqs, int total_tokens, int n_win,
                    int max_n_comp, int m_prime, int32_t* out, int64_t ld, cudaStream_t st);
int comp_offsets_launch(const int32_t* lens, int num_seqs, int is_cu, int stride, int64_t capacity, int32_t* offs,
                        cudaStream_t st);
int decode_idxs_launch(const int32_t* context_lens, const int32_t* offs, int num_seqs, int n_win, int n_comp_cols,
                       int m_prime, int32_t* out, int64_t ld, cudaStream_t st);

struct IndexerArgs {
  const void* q; int64_t sq[3];
  const void* ck; int64_t sck[3];
  const int32_t* cu_seqlens;    // prefill: query rows per sequence
  const int32_t* context_lens;  // decode (cu_seqlens == null): one query per sequence
  const int32_t* comp_offsets;
  int num_seqs, total_tokens, num_q_heads, num_kv_heads, head_dim;
  int n_win, top_k, m;
  int max_comp_per_seq;  // largest comp_offsets[s+1] - comp_offsets[s]
  int32_t* out; int64_t ld;
  int dtype;
  int64_t comp_rows;     // rows of compressed_k
  void* ws; int64_t ws_bytes;      // scratch for tensor-core scores (prefill), may be null
  const void* scores; int64_t sld;  // scores provided: [rows, sld] in the input dtype
};
int csa_indexer_launch(const IndexerArgs& a, cudaStream_t st);
// Scratch bytes for the tensor-core scores of total_tokens prefill rows.
int64_t csa_scores_ws_bytes(int64_t total_tokens, int max_comp_per_seq, int dtype);
// Scores of prefill rows on the tensor cores into a.ws ([total_tokens, *ld]);
// false when the shapes or the scratch do not allow it (nothing launched).
bool csa_scores_tc_launch(const IndexerArgs& a, cudaStream_t st, int64_t* ld, int* err);
// Top-k selection of prefill rows from provided scores, one warp per row
// (at most 1024 slots per sequence); false when it does not apply.
bool csa_select_warp_launch(const IndexerArgs& a, cudaStream_t st);
// Top-k selection of decode rows (one per sequence) from provided scores, one
// 512-thread CTA per row (at most 2048 slots); false when it does not apply.
bool csa_select_block_launch(const IndexerArgs& a, int rows, cudaStream_t st);

}  // namespace tak

// extern "C" entry points declared in include/tak_attention.h: argument
// validation, error strings, tensor-map encoding, dispatch to the kernels.
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "../../include/tak_attention.h"
#include "common.cuh"
#include "kernels.h"

namespace tak {

__device__ int g_tak_device_error = 0;

static thread_local char t_err[512] = "";
static thread_local const char* t_kernel = "";
static int g_kernel_path = 0;

int set_error(int code, const char* msg) {
  std::snprintf(t_err, sizeof(t_err), "%s", msg);
  return code;
}

void note_kernel(const char* name) { t_kernel = name; }

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char buf[400];
    std::snprintf(buf, sizeof(buf), "%s: CUDA error %s", what, cudaGetErrorString(e));
    return set_error(3, buf);
  }
  return 0;
}

int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

int ensure_smem_attr(const void* func, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  int& have = done[{func, dev}];
  if (have >= bytes) return 0;
  const cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    char buf[160];
    std::snprintf(buf, sizeof(buf), "cudaFuncSetAttribute(max dynamic shared memory = %d) failed: %s", bytes,
                  cudaGetErrorString(e));
    return set_error(3, buf);
  }
  have = bytes;
  return 0;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, const uint32_t* elem_strides,
                 CUtensorMapSwizzle swizzle) {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (!fn) return set_error(3, "cuTensorMapEncodeTiled is not available");
  const CUresult r = fn(map, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(base), dims, strides_bytes, box,
                        elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[128];
    std::snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return set_error(3, buf);
  }
  return 0;
}

int prefill_generic_launch(const PrefillArgs& a, cudaStream_t st);
int sparse_generic_launch(const SparseArgs& a, cudaStream_t st);
int prefill_tc_launch(const PrefillArgs& a, cudaStream_t st, bool* handled);
int sparse_tc_launch(const SparseArgs& a, cudaStream_t st, bool* handled);

int prefill_launch(const PrefillArgs& a, cudaStream_t st) {
  if (!a.force_generic) {
    bool handled = false;
    const int r = prefill_tc_launch(a, st, &handled);
    if (r || handled) return r;
  }
  return prefill_generic_launch(a, st);
}

int sparse_launch(const SparseArgs& a, cudaStream_t st) {
  if (!a.force_generic) {
    bool handled = false;
    const int r = sparse_tc_launch(a, st, &handled);
    if (r || handled) return r;
  }
  return sparse_generic_launch(a, st);
}

}  // namespace tak

using namespace tak;

#define TAK_REQUIRE(cond, msg) \
  do {                         \
    if (!(cond)) return set_error(1, msg); \
  } while (0)

// every entry point that launches attention or pooling kernels starts with no
// kernel recorded for tak_last_kernel()
#define TAK_ENTRY() (t_kernel = "")

static void copy_strides(int64_t* dst, const int64_t* src, int n) {
  for (int i = 0; i < n; ++i) dst[i] = src ? src[i] : 0;
}

extern "C" {

const char* tak_version(void) { return "tak-b200 0.1"; }

const char* tak_last_error(void) { return t_err; }

const char* tak_last_kernel(void) { return t_kernel; }

int tak_set_kernel_path(int path) {
  const int old = g_kernel_path;
  g_kernel_path = path;
  return old;
}

int tak_read_device_error(void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(st) != cudaSuccess) return set_error(3, "tak_read_device_error: sync failed"), -1;
  int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_tak_device_error, sizeof(int)) != cudaSuccess) return -1;
  cudaMemcpyToSymbol(g_tak_device_error, &zero, sizeof(int));
  return v;
}

int tak_flash_attention_prefill(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                const void* v, const int64_t* v_strides, const int32_t* cu_seqlens,
                                int64_t num_seqs, void* out, const int64_t* out_strides, float* lse,
                                int64_t total_tokens, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                                float scale, int causal, int dtype, void* stream) {
  TAK_ENTRY();
  TAK_REQUIRE(dtype >= 0 && dtype <= 2, "prefill: unknown dtype");
  TAK_REQUIRE(num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
              "prefill: num_q_heads must be a multiple of num_kv_heads");
  TAK_REQUIRE(head_dim > 0 && head_dim <= 640, "prefill: head_dim must be in [1, 640]");
  TAK_REQUIRE(num_seqs >= 0 && total_tokens >= 0, "prefill: negative sizes");
  if (total_tokens == 0) return 0;
  TAK_REQUIRE(q && k && v && out && cu_seqlens && q_strides && k_strides && v_strides && out_strides,
              "prefill: null pointer");
  PrefillArgs a{};
  a.q = q; copy_strides(a.sq, q_strides, 3);
  a.k = k; copy_strides(a.sk, k_strides, 3);
  a.v = v; copy_strides(a.sv, v_strides, 3);
  a.cu_seqlens = cu_seqlens;
  a.out = out; copy_strides(a.so, out_strides, 3);
  a.lse = lse;
  a.num_seqs = static_cast<int>(num_seqs);
  a.total_tokens = static_cast<int>(total_tokens);
  a.num_q_heads = static_cast<int>(num_q_heads);
  a.num_kv_heads = static_cast<int>(num_kv_heads);
  a.head_dim = a.head_dim_v = static_cast<int>(head_dim);
  a.scale = scale;
  a.causal = causal;
  a.dtype = dtype;
  a.force_generic = g_kernel_path == 1;
  const int r = prefill_launch(a, static_cast<cudaStream_t>(stream));
  return r ? r : check_launch("prefill");
}

size_t tak_paged_attention_decode_workspace_size(int64_t num_seqs, int64_t num_q_heads, int64_t num_kv_heads,
                                                 int64_t head_dim, int64_t block_size, int64_t max_blocks,
                                                 int split_pages) {
  if (num_kv_heads <= 0 || num_q_heads <= 0 || block_size <= 0) return 0;
  PagedDecodeArgs a{};
  a.num_seqs = static_cast<int>(num_seqs);
  a.num_q_heads = static_cast<int>(num_q_heads);
  a.num_kv_heads = static_cast<int>(num_kv_heads);
  a.head_dim = static_cast<int>(head_dim);
  a.block_size = static_cast<int>(block_size);
  a.max_blocks = static_cast<int>(max_blocks);
  a.split_pages = split_pages;
  return paged_decode_workspace_bytes(a);
}

}  // extern "C"

namespace tak {

int make_paged_decode_args(PagedDecodeArgs* out_args, const void* q, const int64_t* q_strides, const void* k_cache,
                           const int64_t* k_strides, const void* v_cache, const int64_t* v_strides,
                           const int32_t* block_tables, const int64_t* bt_strides, const int32_t* context_lens,
                           void* out, const int64_t* out_strides, float* lse, int64_t num_seqs,
                           int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, int64_t block_size,
                           int64_t max_blocks, int64_t num_blocks, int64_t cache_rows, float scale, int dtype,
                           int split_pages) {
  TAK_REQUIRE(dtype >= 0 && dtype <= 2, "paged decode: unknown dtype");
  TAK_REQUIRE(num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
              "paged decode: num_q_heads must be a multiple of num_kv_heads");
  TAK_REQUIRE(head_dim > 0 && head_dim <= 640, "paged decode: head_dim must be in [1, 640]");
  TAK_REQUIRE(block_size > 0 && block_size <= cache_rows, "paged decode: block_size must be in [1, cache_rows]");
  TAK_REQUIRE(num_seqs >= 0 && max_blocks >= 0 && num_blocks >= 0, "paged decode: negative sizes");
  PagedDecodeArgs a{};
  a.num_seqs = static_cast<int>(num_seqs);
  if (num_seqs == 0) {
    *out_args = a;
    return 0;
  }
  TAK_REQUIRE(q && k_cache && v_cache && block_tables && context_lens && out, "paged decode: null pointer");
  TAK_REQUIRE(q_strides && k_strides && v_strides && bt_strides && out_strides, "paged decode: null strides");
  a.q = q; copy_strides(a.sq, q_strides, 3);
  a.k_cache = k_cache; copy_strides(a.sk, k_strides, 4);
  a.v_cache = v_cache; copy_strides(a.sv, v_strides, 4);
  a.block_tables = block_tables; copy_strides(a.sbt, bt_strides, 2);
  a.context_lens = context_lens;
  a.out = out; copy_strides(a.so, out_strides, 3);
  a.lse = lse;
  a.num_q_heads = static_cast<int>(num_q_heads);
  a.num_kv_heads = static_cast<int>(num_kv_heads);
  a.head_dim = static_cast<int>(head_dim);
  a.block_size = static_cast<int>(block_size);
  a.max_blocks = static_cast<int>(max_blocks);
  a.num_blocks = num_blocks;
  a.cache_rows = cache_rows;
  a.scale = scale;
  a.dtype = dtype;
  a.split_pages = split_pages;
  a.force_generic = g_kernel_path == 1;
  *out_args = a;
  return 0;
}

}  // namespace tak

extern "C" {

int tak_paged_attention_decode(const void* q, const int64_t* q_strides, const void* k_cache,
                               const int64_t* k_strides, const void* v_cache, const int64_t* v_strides,
                               const int32_t* block_tables, const int64_t* bt_strides, const int32_t* context_lens,
                               void* out, const int64_t* out_strides, float* lse, int64_t num_seqs,
                               int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, int64_t block_size,
                               int64_t max_blocks, int64_t num_blocks, int64_t cache_rows, float scale, int dtype,
                               void* workspace, size_t workspace_bytes, int split_pages, void* stream) {
  TAK_ENTRY();
  PagedDecodeArgs a{};
  int r = make_paged_decode_args(&a, q, q_strides, k_cache, k_strides, v_cache, v_strides, block_tables, bt_strides,
                                 context_lens, out, out_strides, lse, num_seqs, num_q_heads, num_kv_heads, head_dim,
                                 block_size, max_blocks, num_blocks, cache_rows, scale, dtype, split_pages);
  if (r || num_seqs == 0) return r;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  r = paged_decode_launch(a, static_cast<cudaStream_t>(stream));
  return r ? r : check_launch("paged decode");
}

static int fill_sparse_common(SparseArgs& a, const void* q, const int64_t* q_strides, const int32_t* topk_idxs,
                              const int64_t* topk_strides, const float* attn_sink, void* out,
                              const int64_t* out_strides, float* lse, int64_t rows, int64_t num_q_heads,
                              int64_t num_kv_heads, int64_t head_dim, int64_t head_dim_v, int64_t k_topk,
                              float scale, int dtype) {
  TAK_REQUIRE(dtype >= 0 && dtype <= 2, "sparse attention: unknown dtype");
  TAK_REQUIRE(num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
              "sparse attention: num_q_heads must be a multiple of num_kv_heads");
  TAK_REQUIRE(head_dim > 0 && head_dim <= 640 && head_dim_v > 0 && head_dim_v <= 640,
              "sparse attention: head dims must be in [1, 640]");
  TAK_REQUIRE(k_topk >= 0, "sparse attention: negative k_topk");
  TAK_REQUIRE(q && out && q_strides && out_strides && (k_topk == 0 || (topk_idxs && topk_strides)),
              "sparse attention: null pointer");
  a.q = q; copy_strides(a.sq, q_strides, 3);
  a.topk = topk_idxs; copy_strides(a.stk, topk_strides, 2);
  a.sink = attn_sink;
  a.out = out; copy_strides(a.so, out_strides, 3);
  a.lse = lse;
  a.num_tokens = static_cast<int>(rows);
  a.num_q_heads = static_cast<int>(num_q_heads);
  a.num_kv_heads = static_cast<int>(num_kv_heads);
  a.head_dim = static_cast<int>(head_dim);
  a.head_dim_v = static_cast<int>(head_dim_v);
  a.k_topk = static_cast<int>(k_topk);
  a.scale = scale;
  a.dtype = dtype;
  a.force_generic = g_kernel_path == 1;
  return 0;
}

int tak_sparse_attn_prefill(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                            const void* v, const int64_t* v_strides, const int32_t* topk_idxs,
                            const int64_t* topk_strides, const float* attn_sink, void* out,
                            const int64_t* out_strides, float* lse, int64_t total_tokens, int64_t num_q_heads,
                            int64_t num_kv_heads, int64_t head_dim, int64_t head_dim_v, int64_t kv_rows,
                            int64_t k_topk, float scale, int dtype, void* stream) {
  TAK_ENTRY();
  if (total_tokens == 0) return 0;
  SparseArgs a{};
  int r = fill_sparse_common(a, q, q_strides, topk_idxs, topk_strides, attn_sink, out, out_strides, lse,
                             total_tokens, num_q_heads, num_kv_heads, head_dim, head_dim_v, k_topk, scale, dtype);
  if (r) return r;
  TAK_REQUIRE(k && v && k_strides && v_strides, "sparse prefill: null k/v");
  a.k = k; copy_strides(a.sk, k_strides, 3);
  a.v = v; copy_strides(a.sv, v_strides, 3);
  a.kv_rows = kv_rows;
  a.rows1 = kv_rows;
  a.decode = 0;
  r = sparse_launch(a, static_cast<cudaStream_t>(stream));
  return r ? r : check_launch("sparse prefill");
}

int tak_sparse_attn_prefill_2src(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                 const void* v, const int64_t* v_strides, int64_t kv_rows, const void* k2,
                                 const int64_t* k2_strides, const void* v2, const int64_t* v2_strides,
                                 int64_t kv2_rows, const int32_t* topk_idxs, const int64_t* topk_strides,
                                 const float* attn_sink, void* out, const int64_t* out_strides, float* lse,
                                 int64_t total_tokens, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                                 int64_t head_dim_v, int64_t k_topk, float scale, int dtype, void* stream) {
  TAK_ENTRY();
  if (total_tokens == 0) return 0;
  SparseArgs a{};
  int r = fill_sparse_common(a, q, q_strides, topk_idxs, topk_strides, attn_sink, out, out_strides, lse,
                             total_tokens, num_q_heads, num_kv_heads, head_dim, head_dim_v, k_topk, scale, dtype);
  if (r) return r;
  TAK_REQUIRE(kv_rows >= 0 && kv2_rows >= 0, "sparse prefill (two sources): negative row counts");
  TAK_REQUIRE(k && v && k_strides && v_strides, "sparse prefill (two sources): null k/v");
  TAK_REQUIRE(kv2_rows == 0 || (k2 && v2 && k2_strides && v2_strides),
              "sparse prefill (two sources): null second k/v");
  a.k = k; copy_strides(a.sk, k_strides, 3);
  a.v = v; copy_strides(a.sv, v_strides, 3);
  if (kv2_rows > 0) {
    a.ck = k2; copy_strides(a.sck, k2_strides, 3);
    a.cv = v2; copy_strides(a.scv, v2_strides, 3);
    if (a.sck[2] != a.sk[2] || a.scv[2] != a.sv[2])
      return set_error(2, "sparse prefill (two sources): the two sources need the same head-dim stride");
  }
  a.kv_rows = kv_rows + kv2_rows;
  a.rows1 = kv_rows;
  a.decode = 0;
  r = sparse_launch(a, static_cast<cudaStream_t>(stream));
  return r ? r : check_launch("sparse prefill (two sources)");
}

int tak_sparse_attn_decode(const void* q, const int64_t* q_strides, const void* k_cache, const int64_t* k_strides,
                           const void* v_cache, const int64_t* v_strides, const void* compressed_k,
                           const int64_t* ck_strides, const void* compressed_v, const int64_t* cv_strides,
                           const int32_t* block_tables, const int64_t* bt_strides, const int32_t* topk_idxs,
                           const int64_t* topk_strides, const int32_t* context_lens, const float* attn_sink,
                           void* out, const int64_t* out_strides, float* lse, int64_t num_seqs,
                           int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, int64_t head_dim_v,
                           int64_t num_compressed, int64_t k_topk, int64_t num_win, int64_t block_size,
                           int64_t max_blocks, int64_t num_blocks, float scale, int dtype, void* stream) {
  TAK_ENTRY();
  if (num_seqs == 0) return 0;
  SparseArgs a{};
  int r = fill_sparse_common(a, q, q_strides, topk_idxs, topk_strides, attn_sink, out, out_strides, lse, num_seqs,
                             num_q_heads, num_kv_heads, head_dim, head_dim_v, k_topk, scale, dtype);
  if (r) return r;
  TAK_REQUIRE(k_cache && v_cache && k_strides && v_strides && block_tables && bt_strides && context_lens,
              "sparse decode: null pointer");
  TAK_REQUIRE(num_compressed == 0 || (compressed_k && compressed_v && ck_strides && cv_strides),
              "sparse decode: null compressed k/v");
  TAK_REQUIRE(block_size > 0 && num_win >= 0, "sparse decode: bad block_size / num_win");
  TAK_REQUIRE(max_blocks >= 0 && max_blocks <= 2147483647 && num_blocks >= 0,
              "sparse decode: bad max_blocks / num_blocks");
  a.k = k_cache; copy_strides(a.sk, k_strides, 4);
  a.v = v_cache; copy_strides(a.sv, v_strides, 4);
  a.ck = compressed_k; copy_strides(a.sck, ck_strides, 3);
  a.cv = compressed_v; copy_strides(a.scv, cv_strides, 3);
  a.block_tables = block_tables; copy_strides(a.sbt, bt_strides, 2);
  a.context_lens = context_lens;
  a.num_compressed = num_compressed;
  a.num_win = static_cast<int>(num_win);
  a.block_size = static_cast<int>(block_size);
  a.max_blocks = static_cast<int>(max_blocks);
  a.num_blocks = num_blocks;
  a.decode = 1;
  r = sparse_launch(a, static_cast<cudaStream_t>(stream));
  return r ? r : check_launch("sparse decode");
}

int tak_build_token_to_seq(const int32_t* cu_seqlens, int64_t num_seqs, int64_t total_tokens, int32_t* out,
                           void* stream) {
  if (total_tokens == 0) return 0;
  TAK_REQUIRE(cu_seqlens && out && num_seqs >= 0, "token_to_seq: bad arguments");
  const int r = token_to_seq_launch(cu_seqlens, static_cast<int>(num_seqs), static_cast<int>(total_tokens), out,
                                    static_cast<cudaStream_t>(stream));
  return r ? r : check_launch("token_to_seq");
}

static int compress_common(CompressArgs& a, const void* k, const int64_t* k_strides, int nk, const void* v,
                           const int64_t* v_strides, const int32_t* comp_offsets, int64_t num_seqs,
                           int64_t num_compressed, void* compressed_k, const int64_t* ck_strides,
                           void* compressed_v, const int64_t* cv_strides, int64_t num_kv_heads, int64_t head_dim,
                           int64_t head_dim_v, int64_t stride, int64_t window, int dtype) {
  TAK_REQUIRE(dtype >= 0 && dtype <= 2, "compress: unknown dtype");
  TAK_REQUIRE(stride > 0 && window > 0, "compress: stride and window must be positive");
  // v == null: K only (no V rows, no compressed V, head_dim_v 0), for callers whose V is a view of K
  const bool k_only = v == nullptr;
  TAK_REQUIRE(num_kv_heads > 0 && head_dim > 0 && (k_only ? head_dim_v == 0 : head_dim_v > 0),
              "compress: bad head sizes");
  TAK_REQUIRE(k_only == (compressed_v == nullptr), "compress: v and compressed_v must both be given or both null");
  TAK_REQUIRE(k && k_strides && (k_only || v_strides) && comp_offsets && compressed_k && ck_strides &&
                  (k_only || cv_strides),
              "compress: null pointer");
  a.k = k; copy_strides(a.sk, k_strides, nk);
  a.v = v; copy_strides(a.sv, v_strides, nk);
  a.comp_offsets = comp_offsets;
  a.num_seqs = static_cast<int>(num_seqs);
  a.num_compressed = num_compressed;
  a.ck = compressed_k; copy_strides(a.sck, ck_strides, 3);
  a.cv = compressed_v; copy_strides(a.scv, cv_strides, 3);
  a.num_kv_heads = static_cast<int>(num_kv_heads);
  a.head_dim = static_cast<int>(head_dim);
  a.head_dim_v = static_cast<int>(head_dim_v);
  a.stride = static_cast<int>(stride);
  a.window = static_cast<int>(window);
  a.dtype = dtype;
  return 0;
}

int tak_compress_kv(const void* k, const int64_t* k_strides, const void* v, const int64_t* v_strides,
                    const float* gate, int64_t gate_stride, const int32_t* cu_seqlens, const int32_t* comp_offsets,
                    int64_t num_seqs, int64_t num_compressed, void* compressed_k, const int64_t* ck_strides,
                    void* compressed_v, const int64_t* cv_strides, int64_t num_kv_heads, int64_t head_dim,
                    int64_t head_dim_v, int64_t stride, int64_t window, int dtype, void* stream) {
  TAK_ENTRY();
  if (num_compressed == 0) return 0;
  CompressArgs a{};
  int r = compress_common(a, k, k_strides, 3, v, v_strides, comp_offsets, num_seqs, num_compressed, compressed_k,
                          ck_strides, compressed_v, cv_strides, num_kv_heads, head_dim, head_dim_v, stride, window,
                          dtype);
  if (r) return r;
  TAK_REQUIRE(cu_seqlens, "compress: null cu_seqlens");
  a.cu_seqlens = cu_seqlens;
  a.gate = gate;
  a.sg[0] = gate_stride;
  r = compress_launch(a, static_cast<cudaStream_t>(stream));
  return r ? r : check_launch("compress");
}

int tak_compress_kv_paged(const void* k_cache, const int64_t* k_strides, const void* v_cache,
                          const int64_t* v_strides, const float* gate, const int64_t* gate_strides,
                          const int32_t* block_tables, const int64_t* bt_strides, const int32_t* context_lens,
                          int64_t block_size, int64_t max_blocks, int64_t num_blocks, const int32_t* comp_offsets,
                          int64_t num_seqs, int64_t num_compressed, void* compressed_k, const int64_t* ck_strides,
                          void* compressed_v, const int64_t* cv_strides, int64_t num_kv_heads, int64_t head_dim,
                          int64_t head_dim_v, int64_t stride, int64_t window, int dtype, void* stream) {
  TAK_ENTRY();
  if (num_compressed == 0) return 0;
  CompressArgs a{};
  int r = compress_common(a, k_cache, k_strides, 4, v_cache, v_strides, comp_offsets, num_seqs, num_compressed,
                          compressed_k, ck_strides, compressed_v, cv_strides, num_kv_heads, head_dim, head_dim_v,
                          stride, window, dtype);
  if (r) return r;
  TAK_REQUIRE(block_tables && bt_strides && context_lens && block_size > 0, "compress paged: bad page table");
  TAK_REQUIRE(max_blocks >= 0 && max_blocks <= 2147483647 && num_blocks >= 0,
              "compress paged: bad max_blocks / num_blocks");
  TAK_REQUIRE(!gate || gate_strides, "compress paged: gate needs strides");
  a.cu_seqlens = nullptr;
  a.block_tables = block_tables; copy_strides(a.sbt, bt_strides, 2);
  a.context_lens = context_lens;
  a.block_size = static_cast<int>(block_size);
  a.max_blocks = static_cast<int>(max_blocks);
  a.num_blocks = num_blocks;
  a.gate = gate;
  if (gate) copy_strides(a.sg, gate_strides, 2);
  r = compress_launch(a, static_cast<cudaStream_t>(stream));
  return r ? r : check_launch("compress paged");
}

int tak_compress_kv_csa_hca(const void* k, const int64_t* k_strides, const void* v, const int64_t* v_strides,
                            const float* gate, int64_t gate_stride, const int32_t* cu_seqlens, int64_t num_seqs,
                            int64_t total_tokens, const int32_t* csa_offsets, int64_t num_csa, void* csa_k,
                            const int64_t* csa_k_strides, void* csa_v, const int64_t* csa_v_strides,
                            const int32_t* hca_offsets, int64_t num_hca, void* hca_k, const int64_t* hca_k_strides,
                            void* hca_v, const int64_t* hca_v_strides, int64_t num_kv_heads, int64_t head_dim,
                            int64_t head_dim_v, int64_t m, int64_t m_prime, int dtype, void* stream) {
  TAK_ENTRY();
  if (num_csa == 0 && num_hca == 0) return 0;
  TAK_REQUIRE(v && csa_v && hca_v, "compress csa+hca: null v");
  TAK_REQUIRE(m > 0 && m_prime > 0, "compress csa+hca: m and m_prime must be positive");
  TAK_REQUIRE(total_tokens > 0, "compress csa+hca: total_tokens must be positive when slots exist");
  CompressArgs csa{}, hca{};
  int r = compress_common(csa, k, k_strides, 3, v, v_strides, csa_offsets, num_seqs, num_csa, csa_k, csa_k_strides,
                          csa_v, csa_v_strides, num_kv_heads, head_dim, head_dim_v, m, 2 * m, dtype);
  if (r) return r;
  r = compress_common(hca, k, k_strides, 3, v, v_strides, hca_offsets, num_seqs, num_hca, hca_k, hca_k_strides,
                      hca_v, hca_v_strides, num_kv_heads, head_dim, head_dim_v, m_prime, m_prime, dtype);
  if (r) return r;
  TAK_REQUIRE(cu_seqlens, "compress csa+hca: null cu_seqlens");
  for (CompressArgs* a : {&csa, &hca}) {
    a->cu_seqlens = cu_seqlens;
    a->gate = gate;
    a->sg[0] = gate_stride;
    a->total_rows = total_tokens;
  }
  r = compress_csa_hca_launch(csa, hca, static_cast<cudaStream_t>(stream));
  return r ? r : check_launch("compress csa+hca");
}

int tak_build_window_idxs(const int32_t* cu_seqlens, int64_t num_seqs, int64_t total_tokens, int64_t n_win,
                          int32_t* out, int64_t ld, void* stream) {
  if (total_tokens == 0 || n_win == 0) return 0;
  TAK_REQUIRE(cu_seqlens && out && n_win > 0 && ld >= n_win, "window idxs: bad arguments");
  const int r = window_idxs_launch(cu_seqlens, static_cast<int>(num_seqs), static_cast<int>(total_tokens),
                                   static_cast<int>(n_win), out, ld, static_cast<cudaStream_t>(stream));
  return r ? r : check_launch("window idxs");
}

int tak_build_hca_topk_idxs(const int32_t* cu_seqlens, const int32_t* comp_offsets, int64_t num_seqs,
                            int64_t total_tokens, int64_t n_win, int64_t max_n_comp, int64_t m_prime,
                            int32_t* out, int64_t ld, void* stream) {
  if (total_tokens == 0) return 0;
  TAK_REQUIRE(cu_seqlens && comp_offsets && out && m_prime > 0 && n_win >= 0 && max_n_comp >= 0 &&
                  ld >= n_win + max_n_comp,
              "hca idxs: bad arguments");
  const int r = hca_idxs_launch(cu_seqlens, comp_offsets, static_cast<int>(num_seqs), static_cast<int>(total_tokens),
                                static_cast<int>(n_win), static_cast<int>(max_n_comp), static_cast<int>(m_prime), out,
                                ld, static_cast<cudaStream_t>(stream));
  return r ? r : check_launch("hca idxs");
}

int tak_comp_offsets(const int32_t* lens, int64_t num_seqs, int is_cu, int64_t stride, int64_t capacity,
                     int32_t* comp_offsets, void* stream) {
  TAK_REQUIRE(num_seqs >= 0 && num_seqs <= 2147483647 && stride > 0 && stride <= 2147483647,
              "comp offsets: bad num_seqs / stride");
  TAK_REQUIRE(comp_offsets && (num_seqs == 0 || lens), "comp offsets: null pointer");
  const int r = comp_offsets_launch(lens, static_cast<int>(num_seqs), is_cu ? 1 : 0, static_cast<int>(stride),
                                    capacity, comp_offsets, static_cast<cudaStream_t>(stream));
  return r ? r : check_launch("comp offsets");
}

int tak_build_decode_topk_idxs(const int32_t* context_lens, const int32_t* comp_offsets, int64_t num_seqs,
                               int64_t n_win, int64_t n_comp_cols, int64_t m_prime, int32_t* out, int64_t ld,
                               void* stream) {
  if (num_seqs == 0) return 0;
  TAK_REQUIRE(context_lens && out && n_win >= 0 && n_comp_cols >= 0 && m_prime >= 0 && ld >= n_win + n_comp_cols,
              "decode idxs: bad arguments");
  TAK_REQUIRE(m_prime == 0 || comp_offsets, "decode idxs: null comp_offsets");
  const int r = decode_idxs_launch(context_lens, comp_offsets, static_cast<int>(num_seqs), static_cast<int>(n_win),
                                   static_cast<int>(n_comp_cols), static_cast<int>(m_prime), out, ld,
                                   static_cast<cudaStream_t>(stream));
  return r ? r : check_launch("decode idxs");
}

int tak_csa_indexer_topk(const void* q, const int64_t* q_strides, const void* compressed_k,
                         const int64_t* ck_strides, const int32_t* cu_seqlens, const int32_t* context_lens,
                         const int32_t* comp_offsets, int64_t num_seqs, int64_t total_tokens, int64_t num_q_heads,
                         int64_t num_kv_heads, int64_t head_dim, int64_t n_win, int64_t top_k, int64_t m,
                         int64_t max_comp_per_seq, int32_t* out, int64_t ld, int dtype, void* workspace,
                         int64_t workspace_bytes, int64_t compressed_rows, void* stream) {
  TAK_REQUIRE(dtype >= 0 && dtype <= 2, "csa indexer: unknown dtype");
  TAK_REQUIRE(q && q_strides && comp_offsets && out && (cu_seqlens || context_lens), "csa indexer: null pointer");
  TAK_REQUIRE(max_comp_per_seq == 0 || (compressed_k && ck_strides), "csa indexer: null compressed_k");
  TAK_REQUIRE(m > 0 && top_k >= 0 && n_win >= 0 && ld >= n_win + top_k, "csa indexer: bad sizes");
  TAK_REQUIRE(num_kv_heads > 0 && num_q_heads > 0 && head_dim > 0, "csa indexer: bad head sizes");
  if (top_k == 0 || max_comp_per_seq == 0) return 0;
  IndexerArgs a{};
  a.q = q; copy_strides(a.sq, q_strides, 3);
  a.ck = compressed_k; copy_strides(a.sck, ck_strides, 3);
  a.cu_seqlens = cu_seqlens;
  a.context_lens = context_lens;
  a.comp_offsets = comp_offsets;
  a.num_seqs = static_cast<int>(num_seqs);
  a.total_tokens = static_cast<int>(total_tokens);
  a.num_q_heads = static_cast<int>(num_q_heads);
  a.num_kv_heads = static_cast<int>(num_kv_heads);
  a.head_dim = static_cast<int>(head_dim);
  a.n_win = static_cast<int>(n_win);
  a.top_k = static_cast<int>(top_k);
  a.m = static_cast<int>(m);
  a.max_comp_per_seq = static_cast<int>(max_comp_per_seq);
  a.out = out;
  a.ld = ld;
  a.dtype = dtype;
  a.ws = workspace;
  a.ws_bytes = workspace ? workspace_bytes : 0;
  a.comp_rows = compressed_rows;
  const int r = csa_indexer_launch(a, static_cast<cudaStream_t>(stream));
  return r ? r : check_launch("csa indexer");
}

int64_t tak_csa_indexer_workspace_size(int64_t total_tokens, int64_t max_comp_per_seq, int dtype) {
  if (total_tokens <= 0 || max_comp_per_seq <= 0) return 0;
  return csa_scores_ws_bytes(total_tokens, static_cast<int>(max_comp_per_seq), dtype);
}

}  // extern "C"

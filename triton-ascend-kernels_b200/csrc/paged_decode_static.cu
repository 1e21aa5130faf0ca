// Paged decode for callers that cannot allocate device memory.
//
// tak_paged_attention_decode() needs a caller-provided workspace for its
// split-KV partials.  Some callers cannot obtain one: code that runs where a
// cudaMalloc is not allowed or not affordable (cudaMalloc may synchronise the
// device and stall a serving loop), hosts whose device memory belongs to a
// framework's caching allocator that must not be bypassed, and bindings from
// languages without any device-allocation API.  This entry point takes the
// scratch from a fixed array compiled into the library instead, so a call
// allocates nothing: no cudaMalloc, no cudaFree, no allocating library routine.
//
// Limits and rules:
//   * the array is kStaticScratchBytes (32 MiB) per GPU; every GPU that loads
//     the library holds it until the process exits;
//   * a call whose split-KV partials would need more than that is rejected
//     with status 2 and a message (a larger split_pages shrinks the need);
//   * all calls on a GPU share the one array, which keeps the last call's
//     contents: calls that overlap on the GPU (different streams, different
//     host threads) race and corrupt each other's partials -- serialise them;
//   * nothing in the array needs to start at zero (every partial a call reads
//     was written earlier in the same call);
//   * the array's device address is looked up on the first call made with a
//     GPU current and again whenever that GPU's context has changed since
//     (after cudaDeviceReset, for one); make the first call on each GPU, and
//     the first after a reset, before any stream capture begins;
//   * the arguments are validated as for tak_paged_attention_decode, and the
//     size limit applies only when the split-KV kernels run (fp32 caches,
//     unaligned strides and single-split sizes need no scratch).
#include <cstdio>
#include <mutex>

#include "../../include/tak_attention.h"
#include "common.cuh"
#include "kernels.h"

namespace tak {

constexpr size_t kStaticScratchBytes = size_t(32) << 20;

// Device-side split-KV scratch.  In host code this name is only a stand-in
// for the symbol: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_decode_static_scratch[kStaticScratchBytes];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
struct ScratchAddr {
  void* ptr;
  unsigned long long ctx_id;  // context the address belongs to (0: unknown)
};
ScratchAddr g_scratch[kMaxDevices] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current CUDA context (0 when the driver
// cannot tell); a new primary context after a device reset gets a new id.
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current && get_id && get_current(&ctx) == CUDA_SUCCESS && ctx && get_id(ctx, &id) == CUDA_SUCCESS)
    return id;
  return 0;
}

// Device address of the scratch array on the current GPU: resolved on the
// first call with that GPU current, and again when its context has changed.
int static_scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return set_error(3, "paged decode (static scratch): no usable current CUDA device");
  const unsigned long long ctx_id = current_context_id();
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchAddr& e = g_scratch[dev];
  if (e.ptr == nullptr || e.ctx_id != ctx_id) {
    void* p = nullptr;
    const cudaError_t r = cudaGetSymbolAddress(&p, g_decode_static_scratch);
    if (r != cudaSuccess || p == nullptr) {
      char buf[200];
      std::snprintf(buf, sizeof(buf), "paged decode (static scratch): cudaGetSymbolAddress failed: %s",
                    cudaGetErrorString(r));
      return set_error(3, buf);
    }
    e.ptr = p;
    e.ctx_id = current_context_id();  // the lookup made the device's context current
  }
  *out = e.ptr;
  return 0;
}
}  // namespace

}  // namespace tak

extern "C" int tak_paged_attention_decode_static_scratch(
    const void* q, const int64_t* q_strides, const void* k_cache, const int64_t* k_strides, const void* v_cache,
    const int64_t* v_strides, const int32_t* block_tables, const int64_t* bt_strides, const int32_t* context_lens,
    void* out, const int64_t* out_strides, float* lse, int64_t num_seqs, int64_t num_q_heads, int64_t num_kv_heads,
    int64_t head_dim, int64_t block_size, int64_t max_blocks, int64_t num_blocks, int64_t cache_rows, float scale,
    int dtype, int split_pages, void* stream) {
  using namespace tak;
  note_kernel("");
  PagedDecodeArgs a{};
  int r = make_paged_decode_args(&a, q, q_strides, k_cache, k_strides, v_cache, v_strides, block_tables, bt_strides,
                                 context_lens, out, out_strides, lse, num_seqs, num_q_heads, num_kv_heads, head_dim,
                                 block_size, max_blocks, num_blocks, cache_rows, scale, dtype, split_pages);
  if (r || num_seqs == 0) return r;
  const size_t need = paged_decode_required_workspace(a);
  if (need > kStaticScratchBytes) {
    char buf[300];
    std::snprintf(buf, sizeof(buf),
                  "paged decode (static scratch): these sizes need %zu bytes of split-KV scratch, the library's "
                  "static scratch holds %zu; use a larger split_pages or tak_paged_attention_decode with a workspace",
                  need, kStaticScratchBytes);
    return set_error(2, buf);
  }
  if (need > 0) {
    if ((r = static_scratch_address(&a.workspace))) return r;
    a.workspace_bytes = kStaticScratchBytes;
  }
  r = paged_decode_launch(a, static_cast<cudaStream_t>(stream));
  return r ? r : check_launch("paged decode (static scratch)");
}

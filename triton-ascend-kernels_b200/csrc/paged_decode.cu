// Paged decode attention (one query token per sequence against a paged KV
// cache), split-KV, bandwidth-bound.
//
// Semantics follow attention/paged_attention_decode.py of the reference
// (kernel PD:11-98, wrapper PD:104-151): for sequence s and query head h, the
// keys are logical rows [0, ctx_s) of the cache, row r living in page
// block_tables[s, r / block_size] at offset r % block_size, KV head
// h / (H / H_kv).  Output = softmax(scale * q.K^T) V, plus (an addition) the
// natural-log LSE of the softmax denominator.
//
// Fast path (16-bit types, head_dim 64/128/256, block_size a multiple of 16 up
// to 64 or of 64 above, 16-byte aligned strides):
//   grid  = (splits, H_kv * head_chunks, B); a CTA owns `pages_per_split`
//           pages of one (sequence, KV head) and all <=16 query heads of that
//           KV head's group (GQA: every K/V byte is read once per group).
//   warp 4 (one lane) streams K and V chunks of CH = min(block_size, 64) rows
//           into a 3-stage shared-memory ring with 4-D TMA loads (128-byte
//           swizzle, page id taken from the block table; an out-of-range page
//           id reads zeros instead of faulting).
//   warps 0-3 each take 16 rows of a chunk: S = Q K^T and O += P V with
//           mma.sync m16n8k16 (query heads padded to 16 rows), online softmax
//           in registers, base-2 exponentials.
//   epilogue: the 4 warps merge through shared memory; single-split sequences
//           write the output directly, others write (O, max, sum) partials
//           that paged_decode_combine_kernel merges (one CTA per sequence and
//           KV head; all splits' loads in flight at once).
// Generic path (any dtype incl. fp32, any strides / block size / head dim):
//   one CTA of 4 warps per (sequence, query head); each warp walks a strided
//   subset of the keys (lanes split the head dim), then the warps merge.
#include <cstdio>

#include "decode_unit.cuh"

namespace tak {

// ---------------------------------------------------------------------------
// fast path
// ---------------------------------------------------------------------------
// Two CTAs per SM for head dims up to 128; a 256-dim ring (192 KB of shared
// memory) fits one CTA per SM, which may then use the full register file.
template <typename T, int D, int CH, int NS>
__global__ void __launch_bounds__(160, D >= 256 ? 1 : 2)
    paged_decode_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                           const DecodeParams p) {
  // let the split-KV combine grid (launched with programmatic stream
  // serialization) be scheduled as this grid's last wave runs; it still waits
  // for this whole grid to complete before reading any partial
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  decode_unit<T, D, CH, NS>(&tmK, &tmV, p, blockIdx.x, blockIdx.y, blockIdx.z, smem, threadIdx.x, 0, 1);
}

// The split combine as its own launch: one CTA per (sequence, KV head chunk).
// When launched with programmatic stream serialization the grid may start
// while the partial-writing grid is still running; griddepcontrol.wait holds
// it until that grid has completed.
template <typename T>
__global__ void __launch_bounds__(128) paged_decode_combine_kernel(const DecodeParams p) {
  __shared__ float wts[16 * 64];
  __shared__ float inv_l[16];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  decode_combine<T>(p, blockIdx.x, blockIdx.y, threadIdx.x, wts, inv_l, 0);
}

// ---------------------------------------------------------------------------
// generic path
// ---------------------------------------------------------------------------
struct DecodeGenericParams {
  const void* q;
  int64_t sq_s, sq_h, sq_d;
  const void* kc;
  int64_t sk_b, sk_h, sk_s, sk_d;
  const void* vc;
  int64_t sv_b, sv_h, sv_s, sv_d;
  const int32_t* block_tables;
  int64_t sbt_s, sbt_b;
  const int32_t* context_lens;
  void* out;
  int64_t so_s, so_h, so_d;
  float* lse;
  int H, G, D, block_size, max_ctx;
  int64_t num_blocks;
  float scale_log2;
};

constexpr int kGenMaxDPerLane = 20;  // head_dim <= 640

template <typename T>
__global__ void __launch_bounds__(128) paged_decode_generic_kernel(const DecodeGenericParams p) {
  const int seq = blockIdx.y, h = blockIdx.x, kvh = h / p.G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ctx = min(p.context_lens[seq], p.max_ctx);
  const T* q = reinterpret_cast<const T*>(p.q) + seq * p.sq_s + h * p.sq_h;
  const T* kc = reinterpret_cast<const T*>(p.kc);
  const T* vc = reinterpret_cast<const T*>(p.vc);
  float qr[kGenMaxDPerLane], acc[kGenMaxDPerLane];
#pragma unroll
  for (int i = 0; i < kGenMaxDPerLane; ++i) {
    const int d = lane + 32 * i;
    qr[i] = d < p.D ? Elem<T>::to_f(q[d * p.sq_d]) : 0.f;
    acc[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int tok = warp; tok < ctx; tok += 4) {
    const int64_t page = p.block_tables[seq * p.sbt_s + (tok / p.block_size) * p.sbt_b];
    // a page id outside the cache reads as a zero row (score 0, value 0), as
    // the fast path's TMA loads zero-fill it
    const bool in_cache = page >= 0 && page < p.num_blocks;
    const int off = tok % p.block_size;
    const T* kr = kc + page * p.sk_b + kvh * p.sk_h + off * p.sk_s;
    const T* vr = vc + page * p.sv_b + kvh * p.sv_h + off * p.sv_s;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kGenMaxDPerLane; ++i) {
      const int d = lane + 32 * i;
      if (d < p.D && in_cache) s += qr[i] * Elem<T>::to_f(kr[d * p.sk_d]);
    }
    s = warp_sum(s) * p.scale_log2;
    const float mn = fmaxf(m, s);
    const float a = fast_exp2(m - mn), e = fast_exp2(s - mn);
    l = l * a + e;
#pragma unroll
    for (int i = 0; i < kGenMaxDPerLane; ++i) {
      const int d = lane + 32 * i;
      acc[i] = acc[i] * a + (d < p.D && in_cache ? e * Elem<T>::to_f(vr[d * p.sv_d]) : 0.f);
    }
    m = mn;
  }
  __shared__ float sm_m[4], sm_l[4];
  __shared__ float sm_o[4][32 * kGenMaxDPerLane];
  if (lane == 0) {
    sm_m[warp] = m;
    sm_l[warp] = l;
  }
#pragma unroll
  for (int i = 0; i < kGenMaxDPerLane; ++i) sm_o[warp][lane + 32 * i] = acc[i];
  __syncthreads();
  float M = fmaxf(fmaxf(sm_m[0], sm_m[1]), fmaxf(sm_m[2], sm_m[3]));
  const float Mu = (M == -INFINITY) ? 0.f : M;
  float L = 0.f, f[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    f[w] = fast_exp2(sm_m[w] - Mu);
    L += sm_l[w] * f[w];
  }
  T* out = reinterpret_cast<T*>(p.out) + seq * p.so_s + h * p.so_h;
  for (int d = threadIdx.x; d < p.D; d += 128) {
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) o += sm_o[w][d] * f[w];
    out[d * p.so_d] = Elem<T>::from_f(L > 0.f ? o / L : 0.f);
  }
  if (threadIdx.x == 0 && p.lse) p.lse[seq * p.H + h] = L > 0.f ? (M + __log2f(L)) * kLn2 : -INFINITY;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static int pick_pages_per_split(const PagedDecodeArgs& a, int units) {
  // at most 64 splits per sequence (the combine kernel's weight table)
  const int min_pps = a.max_blocks > 64 ? (a.max_blocks + 63) / 64 : 1;
  if (a.split_pages > 0) return a.split_pages > min_pps ? a.split_pages : min_pps;
  // Aim for ~4 waves of 2 CTAs/SM assuming contexts fill half the table on
  // average, with at most 2048 tokens per split.  Each CTA fills its TMA ring
  // before it streams at full rate, so splits much shorter than this lose
  // bandwidth (measured on batch 64, contexts up to 8192, page 128: 4-page
  // splits 5.5 TB/s, 12-16-page splits 6.3 TB/s).
  const int64_t target_ctas = static_cast<int64_t>(num_sms()) * 2 * 4;
  int64_t pps = (static_cast<int64_t>(units) * a.max_blocks / 2 + target_ctas - 1) / target_ctas;
  const int64_t cap = (2048 + a.block_size - 1) / a.block_size;
  if (pps < 1) pps = 1;
  if (pps > cap) pps = cap;
  if (pps > a.max_blocks) pps = a.max_blocks > 0 ? a.max_blocks : 1;
  if (pps < min_pps) pps = min_pps;
  return static_cast<int>(pps);
}

static bool decode_fast_path_ok(const PagedDecodeArgs& a, int* ch) {
  if (a.dtype == kF32) return false;
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return false;
  if (a.sk[3] != 1 || a.sv[3] != 1) return false;
  int c = a.block_size <= 64 ? a.block_size : 64;
  if (c % 16 != 0 || a.block_size % c != 0) return false;
  const int64_t bytes[] = {a.sk[0] * 2, a.sk[1] * 2, a.sk[2] * 2, a.sv[0] * 2, a.sv[1] * 2, a.sv[2] * 2};
  for (int64_t b : bytes)
    if (b % 16 != 0 || b <= 0) return false;
  if ((reinterpret_cast<uintptr_t>(a.k_cache) | reinterpret_cast<uintptr_t>(a.v_cache)) & 15) return false;
  if (a.block_size > a.cache_rows) return false;
  *ch = c;
  return true;
}

// Workspace layout (256-byte aligned): (max, sum) [B, H, splits, 2], then O
// partials [B, H, splits, D], fp32.  Nothing in it needs initialising.
size_t paged_decode_workspace_bytes(const PagedDecodeArgs& a) {
  const int units = a.num_seqs * a.num_kv_heads * ((a.num_q_heads / a.num_kv_heads + 15) / 16);
  const int pps = pick_pages_per_split(a, units);
  const int64_t max_splits = (a.max_blocks + pps - 1) / pps;
  if (max_splits <= 1) return 0;
  return static_cast<size_t>(static_cast<int64_t>(a.num_seqs) * a.num_q_heads * max_splits * (a.head_dim + 2) * 4 +
                             256);
}

size_t paged_decode_required_workspace(const PagedDecodeArgs& a) {
  if (a.num_seqs == 0 || a.num_q_heads == 0 || a.num_kv_heads == 0) return 0;
  int ch = 0;
  if (a.force_generic || !decode_fast_path_ok(a, &ch)) return 0;
  return paged_decode_workspace_bytes(a);
}

static int encode_cache_map(CUtensorMap* map, const void* base, const int64_t* st, int64_t num_blocks,
                            int64_t hkv, int64_t rows, int64_t d, int box_rows) {
  const uint64_t dims[4] = {static_cast<uint64_t>(d), static_cast<uint64_t>(rows), static_cast<uint64_t>(hkv),
                            static_cast<uint64_t>(num_blocks)};
  const uint64_t strides[3] = {static_cast<uint64_t>(st[2] * 2), static_cast<uint64_t>(st[1] * 2),
                               static_cast<uint64_t>(st[0] * 2)};
  const uint32_t box[4] = {64, static_cast<uint32_t>(box_rows), 1, 1};
  const uint32_t estr[4] = {1, 1, 1, 1};
  return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, base, dims, strides, box, estr,
                      CU_TENSOR_MAP_SWIZZLE_128B);
}

// Tensor maps and parameters of the split-KV fast path (its workspace
// pointers inside a.workspace).
static int decode_fast_setup(const PagedDecodeArgs& a, int D, int CH, int pps, int max_splits, int head_chunks,
                             CUtensorMap* mk, CUtensorMap* mv, DecodeParams* pp) {
  if (encode_cache_map(mk, a.k_cache, a.sk, a.num_blocks, a.num_kv_heads, a.cache_rows, D, CH)) return 3;
  if (encode_cache_map(mv, a.v_cache, a.sv, a.num_blocks, a.num_kv_heads, a.cache_rows, D, CH)) return 3;
  DecodeParams& p = *pp;
  p = DecodeParams{};
  p.q = a.q;
  p.sq_s = a.sq[0]; p.sq_h = a.sq[1]; p.sq_d = a.sq[2];
  p.block_tables = a.block_tables;
  p.sbt_s = a.sbt[0]; p.sbt_b = a.sbt[1];
  p.context_lens = a.context_lens;
  p.out = a.out;
  p.so_s = a.so[0]; p.so_h = a.so[1]; p.so_d = a.so[2];
  p.lse = a.lse;
  float* ws = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(a.workspace) + 255) & ~uintptr_t(255));
  p.ws_ml = ws;
  p.ws_o = ws + static_cast<int64_t>(a.num_seqs) * a.num_q_heads * max_splits * 2;
  p.B = a.num_seqs; p.H = a.num_q_heads; p.Hkv = a.num_kv_heads; p.G = a.num_q_heads / a.num_kv_heads;
  p.D = D; p.block_size = a.block_size; p.pages_per_split = pps; p.max_splits = max_splits;
  p.head_chunks = head_chunks;
  p.max_ctx = a.max_blocks * a.block_size;
  p.scale_log2 = a.scale * kLog2e;
  return 0;
}

int decode_fast_setup_d128(const PagedDecodeArgs& a, CUtensorMap* mk, CUtensorMap* mv, DecodeParams* p,
                           int* max_splits, int* groups) {
  int ch = 0;
  if (a.num_seqs == 0 || a.force_generic || a.head_dim != 128 || !decode_fast_path_ok(a, &ch) || ch != 64) return -1;
  const int G = a.num_q_heads / a.num_kv_heads;
  const int head_chunks = (G + 15) / 16;
  const int pps = pick_pages_per_split(a, a.num_seqs * a.num_kv_heads * head_chunks);
  *max_splits = (a.max_blocks + pps - 1) / pps;
  *groups = a.num_kv_heads * head_chunks;
  return decode_fast_setup(a, 128, 64, pps, *max_splits, head_chunks, mk, mv, p);
}

template <typename T, int D, int CH>
static int launch_fast(const PagedDecodeArgs& a, int pps, int max_splits, int head_chunks, cudaStream_t st) {
  constexpr int NS = 3;
  constexpr int SMEM = DecodeSmem<D, CH, NS>::BYTES + 1024;
  CUtensorMap mk, mv;
  DecodeParams p;
  if (int r = decode_fast_setup(a, D, CH, pps, max_splits, head_chunks, &mk, &mv, &p)) return r;
  p.q = a.q;
  p.sq_s = a.sq[0]; p.sq_h = a.sq[1]; p.sq_d = a.sq[2];
  p.block_tables = a.block_tables;
  p.sbt_s = a.sbt[0]; p.sbt_b = a.sbt[1];
  p.context_lens = a.context_lens;
  p.out = a.out;
  p.so_s = a.so[0]; p.so_h = a.so[1]; p.so_d = a.so[2];
  auto kern = paged_decode_tc_kernel<T, D, CH, NS>;
  if (const int r = ensure_smem_attr(reinterpret_cast<const void*>(kern), SMEM)) return r;
  dim3 grid(max_splits, a.num_kv_heads * head_chunks, a.num_seqs);
  kern<<<grid, 160, SMEM, st>>>(mk, mv, p);
  note_kernel("paged_decode_tc");
  if (max_splits > 1) {
    // programmatic dependent launch: the combine grid may be scheduled during
    // the main grid's last wave (it waits for the main grid in-kernel)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.num_seqs, a.num_kv_heads * head_chunks);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, paged_decode_combine_kernel<T>, p);
    if (e != cudaSuccess) {
      char buf[160];
      std::snprintf(buf, sizeof(buf), "paged decode: combine launch failed: %s", cudaGetErrorString(e));
      return set_error(3, buf);
    }
  }
  return 0;
}

template <typename T>
static int launch_generic(const PagedDecodeArgs& a, cudaStream_t st) {
  DecodeGenericParams p{};
  p.q = a.q; p.sq_s = a.sq[0]; p.sq_h = a.sq[1]; p.sq_d = a.sq[2];
  p.kc = a.k_cache; p.sk_b = a.sk[0]; p.sk_h = a.sk[1]; p.sk_s = a.sk[2]; p.sk_d = a.sk[3];
  p.vc = a.v_cache; p.sv_b = a.sv[0]; p.sv_h = a.sv[1]; p.sv_s = a.sv[2]; p.sv_d = a.sv[3];
  p.block_tables = a.block_tables; p.sbt_s = a.sbt[0]; p.sbt_b = a.sbt[1];
  p.context_lens = a.context_lens;
  p.out = a.out; p.so_s = a.so[0]; p.so_h = a.so[1]; p.so_d = a.so[2];
  p.lse = a.lse;
  p.H = a.num_q_heads; p.G = a.num_q_heads / a.num_kv_heads; p.D = a.head_dim; p.block_size = a.block_size;
  p.max_ctx = a.max_blocks * a.block_size;
  p.num_blocks = a.num_blocks;
  p.scale_log2 = a.scale * kLog2e;
  dim3 grid(a.num_q_heads, a.num_seqs);
  note_kernel("paged_decode_generic");
  paged_decode_generic_kernel<T><<<grid, 128, 0, st>>>(p);
  return 0;
}

int paged_decode_launch(const PagedDecodeArgs& a, cudaStream_t st) {
  if (a.num_seqs == 0 || a.num_q_heads == 0) return 0;
  if (a.head_dim > 32 * kGenMaxDPerLane) return set_error(2, "paged decode: head_dim > 640 is not supported");
  int ch = 0;
  const bool fast = !a.force_generic && decode_fast_path_ok(a, &ch);
  if (!fast) {
    if (a.dtype == kBF16) return launch_generic<__nv_bfloat16>(a, st);
    if (a.dtype == kF16) return launch_generic<__half>(a, st);
    return launch_generic<float>(a, st);
  }
  const int G = a.num_q_heads / a.num_kv_heads;
  const int head_chunks = (G + 15) / 16;
  const int pps = pick_pages_per_split(a, a.num_seqs * a.num_kv_heads * head_chunks);
  const int max_splits = (a.max_blocks + pps - 1) / pps;
  if (max_splits > 1 && (a.workspace == nullptr || a.workspace_bytes < paged_decode_workspace_bytes(a)))
    return set_error(2, "paged decode: workspace too small");
#define TAK_DEC(T, D, CH) return launch_fast<T, D, CH>(a, pps, max_splits, head_chunks, st)
#define TAK_DEC_CH(T, D)   \
  switch (ch) {            \
    case 16: TAK_DEC(T, D, 16); \
    case 32: TAK_DEC(T, D, 32); \
    case 48: TAK_DEC(T, D, 48); \
    default: TAK_DEC(T, D, 64); \
  }
#define TAK_DEC_D(T)                       \
  switch (a.head_dim) {                    \
    case 64: TAK_DEC_CH(T, 64);            \
    case 128: TAK_DEC_CH(T, 128);          \
    default: TAK_DEC_CH(T, 256);           \
  }
  if (a.dtype == kBF16) {
    TAK_DEC_D(__nv_bfloat16)
  } else {
    TAK_DEC_D(__half)
  }
#undef TAK_DEC_D
#undef TAK_DEC_CH
#undef TAK_DEC
}

}  // namespace tak

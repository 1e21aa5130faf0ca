// Generic (CUDA-core) attention kernels: any dtype (fp16 / bf16 / fp32), any
// strides, head dims up to 512.  They carry the cases the tensor-core kernels
// do not (fp32 inputs, odd head dims, unaligned strides) and serve as a
// second, independent implementation in the tests.
//
// One CTA of 4 warps per (query row, query head).  Each warp walks a strided
// subset of the key rows; the lanes split the head dim; online softmax in base
// 2; the 4 warps merge through shared memory.  Sink logits (SA:86-92) enter
// the max and the denominator only.
#include "common.cuh"
#include "kernels.h"

namespace tak {

constexpr int kMaxDPerLane = 20;  // head dims up to 640 (MLA: 576 + 64 spare)

template <typename T>
struct RowPair {
  const T* k;
  const T* v;
};

// Row source for dense prefill: keys [start, start + n) of the sequence.
template <typename T>
struct DenseRows {
  const T* k; int64_t sk_t;
  const T* v; int64_t sv_t;
  int start;
  __device__ bool get(int i, RowPair<T>& r) const {
    r.k = k + static_cast<int64_t>(start + i) * sk_t;
    r.v = v + static_cast<int64_t>(start + i) * sv_t;
    return true;
  }
};

// Row source for sparse prefill: rows topk[i] of flat K/V, -1 (or out of
// range) masked (SA:55-57); rows from rows1 on come from a second source
// (compressed rows appended after the K/V rows).
template <typename T>
struct TopkRows {
  const T* k; int64_t sk_t;
  const T* v; int64_t sv_t;
  const int32_t* idx; int64_t s_idx;
  int64_t rows;
  int64_t rows1;
  const T* k2; int64_t sk2_t;
  const T* v2; int64_t sv2_t;
  __device__ bool get(int i, RowPair<T>& r) const {
    const int64_t j = idx[i * s_idx];
    if (j < 0 || j >= rows) return false;
    if (j < rows1) {
      r.k = k + j * sk_t;
      r.v = v + j * sv_t;
    } else {
      r.k = k2 + (j - rows1) * sk2_t;
      r.v = v2 + (j - rows1) * sv2_t;
    }
    return true;
  }
};

// Row source for sparse decode, slot-position semantics of SA:151-210:
// slots < num_win address the paged cache and need 0 <= idx < ctx; later
// slots address compressed rows idx - ctx and need idx >= ctx.
template <typename T>
struct DecodeTopkRows {
  const T* kc; int64_t sk_b, sk_s;
  const T* vc; int64_t sv_b, sv_s;
  const T* ck; int64_t sck_t;
  const T* cv; int64_t scv_t;
  const int32_t* bt; int64_t sbt_b;
  const int32_t* idx; int64_t s_idx;
  int ctx, num_win, block_size;
  int64_t ncomp;
  int64_t wreach;      // block-table width x block_size
  int64_t num_blocks;  // pages of the cache
  __device__ bool get(int i, RowPair<T>& r) const {
    const int64_t j = idx[i * s_idx];
    if (i < num_win) {
      // inside the context, inside the block-table row, on a page of the cache
      if (j < 0 || j >= ctx || j >= wreach) return false;
      const int64_t page = bt[(j / block_size) * sbt_b];
      if (page < 0 || page >= num_blocks) return false;
      const int64_t off = j % block_size;
      r.k = kc + page * sk_b + off * sk_s;
      r.v = vc + page * sv_b + off * sv_s;
      return true;
    }
    if (j < ctx || j - ctx >= ncomp) return false;
    r.k = ck + (j - ctx) * sck_t;
    r.v = cv + (j - ctx) * scv_t;
    return true;
  }
};

template <typename T, class Rows>
__device__ __forceinline__ void generic_attend(const T* q, int64_t sq_d, int64_t sk_d, int64_t sv_d, int D, int Dv,
                                               int n, const Rows& rows, float scale_log2, bool has_sink,
                                               float sink_log2, T* out, int64_t so_d, float* lse_out,
                                               float out_eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float qr[kMaxDPerLane], acc[kMaxDPerLane];
#pragma unroll
  for (int i = 0; i < kMaxDPerLane; ++i) {
    const int d = lane + 32 * i;
    qr[i] = d < D ? Elem<T>::to_f(q[d * sq_d]) : 0.f;
    acc[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int i = warp; i < n; i += 4) {
    RowPair<T> r;
    if (!rows.get(i, r)) continue;
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxDPerLane; ++j) {
      const int d = lane + 32 * j;
      if (d < D) s += qr[j] * Elem<T>::to_f(r.k[d * sk_d]);
    }
    s = warp_sum(s) * scale_log2;
    const float mn = fmaxf(m, s);
    const float a = fast_exp2(m - mn), e = fast_exp2(s - mn);
    l = l * a + e;
#pragma unroll
    for (int j = 0; j < kMaxDPerLane; ++j) {
      const int d = lane + 32 * j;
      acc[j] = acc[j] * a + (d < Dv ? e * Elem<T>::to_f(r.v[d * sv_d]) : 0.f);
    }
    m = mn;
  }
  __shared__ float sm_m[4], sm_l[4];
  __shared__ float sm_o[4][32 * kMaxDPerLane];
  if (lane == 0) {
    sm_m[warp] = m;
    sm_l[warp] = l;
  }
#pragma unroll
  for (int j = 0; j < kMaxDPerLane; ++j) sm_o[warp][lane + 32 * j] = acc[j];
  __syncthreads();
  float M = fmaxf(fmaxf(sm_m[0], sm_m[1]), fmaxf(sm_m[2], sm_m[3]));
  if (has_sink) M = fmaxf(M, sink_log2);
  const float Mu = (M == -INFINITY) ? 0.f : M;
  float L = has_sink ? fast_exp2(sink_log2 - Mu) : 0.f, f[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    f[w] = fast_exp2(sm_m[w] - Mu);
    L += sm_l[w] * f[w];
  }
  const float inv = L > 0.f ? 1.f / (L + out_eps) : 0.f;
  for (int d = threadIdx.x; d < Dv; d += 128) {
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) o += sm_o[w][d] * f[w];
    out[d * so_d] = Elem<T>::from_f(o * inv);
  }
  if (threadIdx.x == 0 && lse_out) *lse_out = L > 0.f ? (M + __log2f(L)) * kLn2 : -INFINITY;
}

__device__ __forceinline__ int find_seq(const int32_t* cu, int num_seqs, int t) {
  // last s with cu[s] <= t (sequences may be empty); -1 if t is outside all
  int lo = 0, hi = num_seqs - 1, ans = -1;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    if (cu[mid] <= t) {
      ans = mid;
      lo = mid + 1;
    } else {
      hi = mid - 1;
    }
  }
  if (ans >= 0 && t >= cu[ans + 1]) ans = -1;
  return ans;
}

template <typename T>
__global__ void __launch_bounds__(128) prefill_generic_kernel(const PrefillArgs a, float scale_log2) {
  const int t = blockIdx.x, h = blockIdx.y;
  const int G = a.num_q_heads / a.num_kv_heads, kvh = h / G;
  const int s = find_seq(a.cu_seqlens, a.num_seqs, t);
  T* out = reinterpret_cast<T*>(a.out) + t * a.so[0] + h * a.so[1];
  float* lse = a.lse ? a.lse + static_cast<int64_t>(t) * a.num_q_heads + h : nullptr;
  if (s < 0) {  // token outside every sequence: zeros (FP:189)
    for (int d = threadIdx.x; d < a.head_dim_v; d += 128) out[d * a.so[2]] = Elem<T>::from_f(0.f);
    if (threadIdx.x == 0 && lse) *lse = -INFINITY;
    return;
  }
  const int start = a.cu_seqlens[s], end = a.cu_seqlens[s + 1];
  const int n = a.causal ? (t - start + 1) : (end - start);
  DenseRows<T> rows{reinterpret_cast<const T*>(a.k) + kvh * a.sk[1], a.sk[0],
                    reinterpret_cast<const T*>(a.v) + kvh * a.sv[1], a.sv[0], start};
  const T* q = reinterpret_cast<const T*>(a.q) + t * a.sq[0] + h * a.sq[1];
  // the reference normalises by (l + 1e-6) (FP:97); l is relative to the row max there
  generic_attend<T>(q, a.sq[2], a.sk[2], a.sv[2], a.head_dim, a.head_dim_v, n, rows, scale_log2, false, 0.f, out,
                    a.so[2], lse, 1e-6f);
}

template <typename T>
__global__ void __launch_bounds__(128) sparse_generic_kernel(const SparseArgs a, float scale_log2) {
  const int t = blockIdx.x, h = blockIdx.y;
  const int G = a.num_q_heads / a.num_kv_heads, kvh = h / G;
  T* out = reinterpret_cast<T*>(a.out) + t * a.so[0] + h * a.so[1];
  float* lse = a.lse ? a.lse + static_cast<int64_t>(t) * a.num_q_heads + h : nullptr;
  const T* q = reinterpret_cast<const T*>(a.q) + t * a.sq[0] + h * a.sq[1];
  const bool has_sink = a.sink != nullptr;
  const float sink_log2 = has_sink ? a.sink[h] * kLog2e : 0.f;
  if (!a.decode) {
    const bool two = a.rows1 < a.kv_rows;
    TopkRows<T> rows{reinterpret_cast<const T*>(a.k) + kvh * a.sk[1], a.sk[0],
                     reinterpret_cast<const T*>(a.v) + kvh * a.sv[1], a.sv[0],
                     a.topk + t * a.stk[0], a.stk[1], a.kv_rows, a.rows1,
                     two ? reinterpret_cast<const T*>(a.ck) + kvh * a.sck[1] : nullptr, a.sck[0],
                     two ? reinterpret_cast<const T*>(a.cv) + kvh * a.scv[1] : nullptr, a.scv[0]};
    generic_attend<T>(q, a.sq[2], a.sk[2], a.sv[2], a.head_dim, a.head_dim_v, a.k_topk, rows, scale_log2, has_sink,
                      sink_log2, out, a.so[2], lse, 0.f);
  } else {
    DecodeTopkRows<T> rows{reinterpret_cast<const T*>(a.k) + kvh * a.sk[1], a.sk[0], a.sk[2],
                           reinterpret_cast<const T*>(a.v) + kvh * a.sv[1], a.sv[0], a.sv[2],
                           reinterpret_cast<const T*>(a.ck) + kvh * a.sck[1], a.sck[0],
                           reinterpret_cast<const T*>(a.cv) + kvh * a.scv[1], a.scv[0],
                           a.block_tables + t * a.sbt[0], a.sbt[1],
                           a.topk + t * a.stk[0], a.stk[1],
                           a.context_lens[t], a.num_win, a.block_size, a.num_compressed,
                           static_cast<int64_t>(a.max_blocks) * a.block_size, a.num_blocks};
    generic_attend<T>(q, a.sq[2], a.sk[3], a.sv[3], a.head_dim, a.head_dim_v, a.k_topk, rows, scale_log2, has_sink,
                      sink_log2, out, a.so[2], lse, 0.f);
  }
}

int prefill_generic_launch(const PrefillArgs& a, cudaStream_t st) {
  if (a.total_tokens == 0 || a.num_q_heads == 0) return 0;
  const float sl2 = a.scale * kLog2e;
  dim3 grid(a.total_tokens, a.num_q_heads);
  note_kernel("prefill_generic");
  if (a.dtype == kBF16)
    prefill_generic_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(a, sl2);
  else if (a.dtype == kF16)
    prefill_generic_kernel<__half><<<grid, 128, 0, st>>>(a, sl2);
  else
    prefill_generic_kernel<float><<<grid, 128, 0, st>>>(a, sl2);
  return 0;
}

int sparse_generic_launch(const SparseArgs& a, cudaStream_t st) {
  if (a.num_tokens == 0 || a.num_q_heads == 0) return 0;
  const float sl2 = a.scale * kLog2e;
  dim3 grid(a.num_tokens, a.num_q_heads);
  note_kernel("sparse_generic");
  if (a.dtype == kBF16)
    sparse_generic_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(a, sl2);
  else if (a.dtype == kF16)
    sparse_generic_kernel<__half><<<grid, 128, 0, st>>>(a, sl2);
  else
    sparse_generic_kernel<float><<<grid, 128, 0, st>>>(a, sl2);
  return 0;
}

}  // namespace tak

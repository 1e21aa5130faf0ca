// KV compression (CSA overlapping / HCA non-overlapping window pooling) and the
// index-row builders of the CSA/HCA sparse paths.
//
// compress: slot i of sequence s pools rows [i*stride, min(i*stride + window,
//   L_s)) of K and V (CSA:49-55 with window = 2m, stride = m; HCA:49-55 with
//   window = stride = m').  Plain mean (the reference), or -- when a gate
//   vector is given -- the softmax(gate)-weighted sum over the window's rows.
//   Rows come from a TND tensor (cu_seqlens) or directly from a paged cache
//   (block tables), which fuses the reference decode wrappers' page gather
//   (CSA:225-253, HCA:204-230) into the pooling.  One CTA per (slot, KV head);
//   each thread owns one 16-byte vector (8 elements) of the [K | V] row and
//   accumulates in fp32.
// index builders: window part (CSA:108-117, decode CSA:270-273), HCA
//   compressed part (HCA:139-144, decode HCA:256-259), token -> sequence map
//   (SA:253-260).
// CSA indexer: Lightning-indexer scores q.k~ of the last query head against the
//   last KV head (the reference's per-head writes leave the last head's choice,
//   CSA:136-162), rounded to the input dtype like the reference's matmul
//   output, causal iff slot*m < position, top-k in descending score order with
//   ties to the lower slot, masked slots appended in ascending order when fewer
//   than k are causal.
#include "common.cuh"
#include "kernels.h"

namespace tak {

// Gate logit of paged row r of sequence s (0 for a row that paged_row_page rejects).
__device__ __forceinline__ float paged_gate(const CompressArgs& a, int s, int r) {
  const int64_t page = paged_row_page(a, s, r);
  return page < 0 ? 0.f : a.gate[page * a.sg[0] + (r % a.block_size) * a.sg[1]];
}

template <typename T, int VEC>
__global__ void compress_kernel(const CompressArgs a) {
  const int64_t slot = blockIdx.x;
  const int h = blockIdx.y;
  if (slot >= a.comp_offsets[a.num_seqs]) return;  // num_compressed may be a capacity
  const int s = find_slot_seq(a.comp_offsets, a.num_seqs, slot);
  const int i = static_cast<int>(slot - a.comp_offsets[s]);
  const bool paged = a.cu_seqlens == nullptr;
  const int L = paged ? a.context_lens[s] : (a.cu_seqlens[s + 1] - a.cu_seqlens[s]);
  const int r0 = i * a.stride;
  const int r1 = min(r0 + a.window, L);
  const int nk = a.head_dim / VEC, nv = a.head_dim_v / VEC;
  const int j = threadIdx.x;
  if (j >= nk + nv) return;
  const bool is_k = j < nk;
  const int d0 = (is_k ? j : j - nk) * VEC;
  const T* base = reinterpret_cast<const T*>(is_k ? a.k : a.v);
  const int64_t* st = is_k ? a.sk : a.sv;
  const int64_t sd = paged ? st[3] : st[2];

  // window weights: plain mean, or softmax of the gate logits of the window
  float gmax = 0.f, gsum = static_cast<float>(r1 - r0);
  if (a.gate) {
    gmax = -INFINITY;
    for (int r = r0; r < r1; ++r) {
      const float g = paged ? paged_gate(a, s, r) : a.gate[(a.cu_seqlens[s] + r) * a.sg[0]];
      gmax = fmaxf(gmax, g);
    }
    gsum = 0.f;
    // a window whose logits are all -inf (every row masked) pools to zeros
    if (gmax != -INFINITY) {
      for (int r = r0; r < r1; ++r) {
        const float g = paged ? paged_gate(a, s, r) : a.gate[(a.cu_seqlens[s] + r) * a.sg[0]];
        gsum += __expf(g - gmax);
      }
    }
  }
  const bool all_masked = a.gate && gmax == -INFINITY;
  float acc[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
  for (int r = r0; r < r1; ++r) {
    const T* row;
    float w = 1.f;
    if (paged) {
      const int64_t page = paged_row_page(a, s, r);
      if (a.gate) w = all_masked ? 0.f : __expf(paged_gate(a, s, r) - gmax);
      if (page < 0) continue;  // a zero row: adds nothing to the sum
      row = base + page * st[0] + h * st[1] + (r % a.block_size) * st[2];
    } else {
      const int64_t tok = a.cu_seqlens[s] + r;
      row = base + tok * st[0] + h * st[1];
      if (a.gate) w = all_masked ? 0.f : __expf(a.gate[tok * a.sg[0]] - gmax);
    }
    if constexpr (VEC == 8) {
      const uint4 u = *reinterpret_cast<const uint4*>(row + d0);
      const uint32_t* pw = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = Elem<T>::unpack2(pw[e]);
        acc[2 * e] += w * f.x;
        acc[2 * e + 1] += w * f.y;
      }
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[e] += w * Elem<T>::to_f(row[(d0 + e) * sd]);
    }
  }
  const float inv = gsum > 0.f ? 1.f / gsum : 0.f;
  T* dst = reinterpret_cast<T*>(is_k ? a.ck : a.cv);
  const int64_t* so = is_k ? a.sck : a.scv;
  T* orow = dst + slot * so[0] + h * so[1];
#pragma unroll
  for (int e = 0; e < VEC; ++e) orow[(d0 + e) * so[2]] = Elem<T>::from_f(acc[e] * inv);
}

// Streaming pooling for windows of one or two strides (the reference's CSA and
// HCA shapes): a CTA owns a run of consecutive slots, reads every row of that
// run exactly once (rows are summed into stride-sized blocks; a CSA slot is
// block i + block i+1), with 8 independent 16-byte loads in flight per thread.
// Thread j owns 8 consecutive elements of the [K | V] row.  With a gate the
// blocks carry (max logit, sum of weights, weighted sum) and slots merge them
// like an online softmax.
template <typename T, int WIN_BLOCKS>
__global__ void __launch_bounds__(128) compress_stream_kernel(const CompressArgs a, int slots_per_cta) {
  const int64_t g0 = static_cast<int64_t>(blockIdx.x) * slots_per_cta;
  const int64_t total = min(a.num_compressed, static_cast<int64_t>(a.comp_offsets[a.num_seqs]));
  const int h = blockIdx.y;
  const int nk = a.head_dim / 8, nv = a.head_dim_v / 8;
  const int j = threadIdx.x;
  const bool active = j < nk + nv;
  const bool is_k = j < nk;
  const int d0 = (is_k ? j : j - nk) * 8;
  const T* base = reinterpret_cast<const T*>(is_k ? a.k : a.v);
  const int64_t* st = is_k ? a.sk : a.sv;
  T* dst = reinterpret_cast<T*>(is_k ? a.ck : a.cv);
  const int64_t* so = is_k ? a.sck : a.scv;
  const bool paged = a.cu_seqlens == nullptr;
  const int m = a.stride;
  const int64_t gend = min(g0 + slots_per_cta, total);
  if (g0 >= gend) return;
  int64_t slot = g0;
  int s = find_slot_seq(a.comp_offsets, a.num_seqs, slot);
  while (slot < gend) {
    while (s + 1 < a.num_seqs && a.comp_offsets[s + 1] <= slot) ++s;
    const int64_t seg_end = min(gend, static_cast<int64_t>(a.comp_offsets[s + 1]));
    const int i0 = static_cast<int>(slot - a.comp_offsets[s]);
    const int i1 = static_cast<int>(seg_end - a.comp_offsets[s]);
    const int L = paged ? a.context_lens[s] : (a.cu_seqlens[s + 1] - a.cu_seqlens[s]);
    const int64_t tok0 = paged ? 0 : a.cu_seqlens[s];
    // blocks [i0, i1 + WIN_BLOCKS - 1) cover the segment's windows
    const int r_begin = i0 * m;
    const int r_end = min((i1 + WIN_BLOCKS - 1) * m, L);
    float prev[8], cur[8];
    float pm = -INFINITY, ps = 0.f, cm = -INFINITY, cs = 0.f;  // gate block (max, sum)
#pragma unroll
    for (int e = 0; e < 8; ++e) prev[e] = cur[e] = 0.f;
    int blk = i0;  // block being accumulated
    for (int r0 = r_begin; r0 < r_end; r0 += 8) {
      uint4 u[8];
      float gv[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int r = r0 + k;
        u[k] = make_uint4(0, 0, 0, 0);
        gv[k] = -INFINITY;
        if (r < r_end) {
          int64_t roff, goff;
          bool ok = true;
          if (paged) {
            const int64_t page = paged_row_page(a, s, r);
            ok = page >= 0;  // rows past the table or on pages outside the cache: zero row, logit 0
            roff = page * st[0] + h * st[1] + (r % a.block_size) * st[2];
            goff = page * a.sg[0] + (r % a.block_size) * a.sg[1];
          } else {
            roff = (tok0 + r) * st[0] + h * st[1];
            goff = (tok0 + r) * a.sg[0];
          }
          if (active && ok) u[k] = __ldg(reinterpret_cast<const uint4*>(base + roff + d0));
          if (a.gate) gv[k] = ok ? __ldg(a.gate + goff) : 0.f;
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int r = r0 + k;
        if (r >= r_end) break;
        float w = 1.f;
        if (a.gate) {
          if (gv[k] > cm) {  // new block max: rescale the block's running sums
            const float f = __expf(cm - gv[k]);
            cs *= f;
#pragma unroll
            for (int e = 0; e < 8; ++e) cur[e] *= f;
            cm = gv[k];
          }
          w = gv[k] == -INFINITY ? 0.f : __expf(gv[k] - cm);  // a -inf logit masks its row
          cs += w;
        }
        const uint32_t* pw = reinterpret_cast<const uint32_t*>(&u[k]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f2 = Elem<T>::unpack2(pw[e]);
          cur[2 * e] += w * f2.x;
          cur[2 * e + 1] += w * f2.y;
        }
        if (r + 1 == min((blk + 1) * m, r_end)) {
          // block `blk` is complete: emit the slot(s) it finishes
          const int emit = WIN_BLOCKS == 1 ? blk : blk - 1;
          if (emit >= i0 && emit < i1) {
            float o[8];
            if (a.gate) {
              float M = cm, S = cs;
              if (WIN_BLOCKS == 2) M = fmaxf(pm, cm);
              const float fc = cm == -INFINITY ? 0.f : __expf(cm - M);
              const float fp = (WIN_BLOCKS == 2 && pm != -INFINITY) ? __expf(pm - M) : 0.f;
              S = cs * fc + (WIN_BLOCKS == 2 ? ps * fp : 0.f);
              const float inv = S > 0.f ? 1.f / S : 0.f;
#pragma unroll
              for (int e = 0; e < 8; ++e) o[e] = (cur[e] * fc + (WIN_BLOCKS == 2 ? prev[e] * fp : 0.f)) * inv;
            } else {
              const int wr0 = emit * m;
              const int cnt = min(wr0 + WIN_BLOCKS * m, L) - wr0;
              const float inv = 1.f / static_cast<float>(cnt);
#pragma unroll
              for (int e = 0; e < 8; ++e) o[e] = (cur[e] + (WIN_BLOCKS == 2 ? prev[e] : 0.f)) * inv;
            }
            if (active) {
              uint4 q;
              q.x = Elem<T>::pack2(o[0], o[1]);
              q.y = Elem<T>::pack2(o[2], o[3]);
              q.z = Elem<T>::pack2(o[4], o[5]);
              q.w = Elem<T>::pack2(o[6], o[7]);
              *reinterpret_cast<uint4*>(dst + (a.comp_offsets[s] + emit) * so[0] + h * so[1] + d0) = q;
            }
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            prev[e] = cur[e];
            cur[e] = 0.f;
          }
          pm = cm;
          ps = cs;
          cm = -INFINITY;
          cs = 0.f;
          ++blk;
        }
      }
    }
    // CSA: the last slot's window ends at the sequence end (block i1 may not exist)
    if (WIN_BLOCKS == 2 && i1 * m >= L && i1 - 1 >= i0 && i1 - 1 == blk - 1) {
      const int emit = i1 - 1;
      float o[8];
      if (a.gate) {
        const float inv = ps > 0.f ? 1.f / ps : 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = prev[e] * inv;
      } else {
        const float inv = 1.f / static_cast<float>(L - emit * m);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = prev[e] * inv;
      }
      if (active) {
        uint4 q;
        q.x = Elem<T>::pack2(o[0], o[1]);
        q.y = Elem<T>::pack2(o[2], o[3]);
        q.z = Elem<T>::pack2(o[4], o[5]);
        q.w = Elem<T>::pack2(o[6], o[7]);
        *reinterpret_cast<uint4*>(dst + (a.comp_offsets[s] + emit) * so[0] + h * so[1] + d0) = q;
      }
    }
    slot = seg_end;
  }
}

// Non-overlapping windows of many rows (HCA, m' >= 64): one CTA per (slot,
// KV head), 4 row groups of 128 threads each streaming a quarter of the window
// with 8 independent 16-byte loads in flight per thread, merged through shared
// memory (with a gate: per-group max / weight-sum / weighted sum, merged like an
// online softmax).
template <typename T>
__global__ void __launch_bounds__(512) compress_split_kernel(const CompressArgs a) {
  constexpr int RG = 4;
  __shared__ float part[RG][128][8];
  __shared__ float gpart[RG][2];
  const int64_t slot = blockIdx.x;
  const int h = blockIdx.y;
  if (slot >= a.comp_offsets[a.num_seqs]) return;  // num_compressed may be a capacity
  const int s = find_slot_seq(a.comp_offsets, a.num_seqs, slot);
  const int i = static_cast<int>(slot - a.comp_offsets[s]);
  const bool paged = a.cu_seqlens == nullptr;
  const int L = paged ? a.context_lens[s] : (a.cu_seqlens[s + 1] - a.cu_seqlens[s]);
  const int64_t tok0 = paged ? 0 : a.cu_seqlens[s];
  const int r0 = i * a.stride, r1 = min(r0 + a.window, L);
  const int grp = threadIdx.x >> 7, j = threadIdx.x & 127;
  const int nk = a.head_dim / 8, nv = a.head_dim_v / 8;
  const bool active = j < nk + nv;
  const bool is_k = j < nk;
  const int d0 = (is_k ? j : j - nk) * 8;
  const T* base = reinterpret_cast<const T*>(is_k ? a.k : a.v);
  const int64_t* st = is_k ? a.sk : a.sv;
  const int rows = r1 - r0;
  const int per = (rows + RG - 1) / RG;
  const int ga = r0 + grp * per, gb = min(ga + per, r1);
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  float gm = -INFINITY, gs = 0.f;
  for (int rr = ga; rr < gb; rr += 8) {
    uint4 u[8];
    float gv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int r = rr + k;
      u[k] = make_uint4(0, 0, 0, 0);
      gv[k] = -INFINITY;
      if (r < gb) {
        int64_t roff, goff;
        bool ok = true;
        if (paged) {
          const int64_t page = paged_row_page(a, s, r);
          ok = page >= 0;  // rows past the table or on pages outside the cache: zero row, logit 0
          roff = page * st[0] + h * st[1] + (r % a.block_size) * st[2];
          goff = page * a.sg[0] + (r % a.block_size) * a.sg[1];
        } else {
          roff = (tok0 + r) * st[0] + h * st[1];
          goff = (tok0 + r) * a.sg[0];
        }
        if (active && ok) u[k] = __ldg(reinterpret_cast<const uint4*>(base + roff + d0));
        if (a.gate) gv[k] = ok ? __ldg(a.gate + goff) : 0.f;
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (rr + k >= gb) break;
      float w = 1.f;
      if (a.gate) {
        if (gv[k] > gm) {
          const float f = __expf(gm - gv[k]);
          gs *= f;
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] *= f;
          gm = gv[k];
        }
        w = gv[k] == -INFINITY ? 0.f : __expf(gv[k] - gm);  // a -inf logit masks its row
        gs += w;
      }
      const uint32_t* pw = reinterpret_cast<const uint32_t*>(&u[k]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f2 = Elem<T>::unpack2(pw[e]);
        acc[2 * e] += w * f2.x;
        acc[2 * e + 1] += w * f2.y;
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) part[grp][j][e] = acc[e];
  if (j == 0) {
    gpart[grp][0] = gm;
    gpart[grp][1] = gs;
  }
  __syncthreads();
  if (grp != 0 || !active) return;
  float o[8];
  if (a.gate) {
    float M = -INFINITY;
#pragma unroll
    for (int g = 0; g < RG; ++g) M = fmaxf(M, gpart[g][0]);
    float S = 0.f, f[RG];
#pragma unroll
    for (int g = 0; g < RG; ++g) {
      f[g] = gpart[g][0] == -INFINITY ? 0.f : __expf(gpart[g][0] - M);
      S += gpart[g][1] * f[g];
    }
    const float inv = S > 0.f ? 1.f / S : 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float v = 0.f;
#pragma unroll
      for (int g = 0; g < RG; ++g) v += part[g][j][e] * f[g];
      o[e] = v * inv;
    }
  } else {
    const float inv = rows > 0 ? 1.f / static_cast<float>(rows) : 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = (part[0][j][e] + part[1][j][e] + part[2][j][e] + part[3][j][e]) * inv;
  }
  T* dst = reinterpret_cast<T*>(is_k ? a.ck : a.cv);
  const int64_t* so = is_k ? a.sck : a.scv;
  uint4 q;
  q.x = Elem<T>::pack2(o[0], o[1]);
  q.y = Elem<T>::pack2(o[2], o[3]);
  q.z = Elem<T>::pack2(o[4], o[5]);
  q.w = Elem<T>::pack2(o[6], o[7]);
  *reinterpret_cast<uint4*>(dst + slot * so[0] + h * so[1] + d0) = q;
}

template <typename T>
static int compress_typed(const CompressArgs& a, cudaStream_t st) {
  const bool paged = a.cu_seqlens == nullptr;
  const int64_t kd = paged ? a.sk[3] : a.sk[2];
  const int64_t vd = paged ? a.sv[3] : a.sv[2];
  // no V (K-only pooling): its strides are all 0 and never used
  bool vec = sizeof(T) == 2 && kd == 1 && (vd == 1 || !a.v) && a.sck[2] == 1 && (a.scv[2] == 1 || !a.cv) &&
             a.head_dim % 8 == 0 && a.head_dim_v % 8 == 0;
  const int64_t* strides[] = {a.sk, a.sv};
  for (const int64_t* s4 : strides)
    for (int i = 0; i < (paged ? 3 : 2); ++i) vec = vec && (s4[i] % 8 == 0);
  vec = vec && ((reinterpret_cast<uintptr_t>(a.k) | reinterpret_cast<uintptr_t>(a.v)) & 15) == 0;
  vec = vec && a.sck[0] % 8 == 0 && a.sck[1] % 8 == 0 && a.scv[0] % 8 == 0 && a.scv[1] % 8 == 0 &&
        ((reinterpret_cast<uintptr_t>(a.ck) | reinterpret_cast<uintptr_t>(a.cv)) & 15) == 0;
  dim3 grid(static_cast<unsigned>(a.num_compressed), a.num_kv_heads);
  if constexpr (sizeof(T) == 2) {
    int err = 0;
    if (compress_bulk_launch(a, st, &err)) return err;
    const int threads = (a.head_dim + a.head_dim_v) / 8;
    if (vec && threads <= 128 && a.window == a.stride && a.stride >= 64) {
      compress_split_kernel<T><<<grid, 512, 0, st>>>(a);
      note_kernel("compress_split");
      return 0;
    }
    if (vec && threads <= 128 && (a.window == a.stride || a.window == 2 * a.stride)) {
      // ~32 rows per CTA: enough CTAs to fill the GPU, small halo for CSA
      const int spc = a.stride >= 32 ? 1 : 32 / a.stride;
      const unsigned ctas = static_cast<unsigned>((a.num_compressed + spc - 1) / spc);
      if (a.window == a.stride)
        compress_stream_kernel<T, 1><<<dim3(ctas, a.num_kv_heads), 128, 0, st>>>(a, spc);
      else
        compress_stream_kernel<T, 2><<<dim3(ctas, a.num_kv_heads), 128, 0, st>>>(a, spc);
      note_kernel("compress_stream");
      return 0;
    }
    if (vec) {
      const int threads = (a.head_dim + a.head_dim_v) / 8;
      if (threads > 1024) return set_error(2, "compress: head dim too large");
      compress_kernel<T, 8><<<grid, threads, 0, st>>>(a);
      note_kernel("compress_rows");
      return 0;
    }
  }
  {
    const int threads = a.head_dim + a.head_dim_v;
    if (threads > 1024) return set_error(2, "compress: head dim too large");
    compress_kernel<T, 1><<<grid, threads, 0, st>>>(a);
    note_kernel("compress_rows");
  }
  return 0;
}

int compress_launch(const CompressArgs& a, cudaStream_t st) {
  if (a.num_compressed == 0 || a.num_kv_heads == 0) return 0;
  if (a.dtype == kBF16) return compress_typed<__nv_bfloat16>(a, st);
  if (a.dtype == kF16) return compress_typed<__half>(a, st);
  return compress_typed<float>(a, st);
}

// ---------------------------------------------------------------------------
// index builders
// ---------------------------------------------------------------------------
__device__ __forceinline__ int seq_of_token(const int32_t* cu, int num_seqs, int t) {
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

__global__ void token_to_seq_kernel(const int32_t* cu, int num_seqs, int total_tokens, int32_t* out) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= total_tokens) return;
  const int s = seq_of_token(cu, num_seqs, t);
  out[t] = s < 0 ? 0 : s;
}

__global__ void window_idxs_kernel(const int32_t* cu, int num_seqs, int total_tokens, int n_win, int32_t* out,
                                   int64_t ld) {
  const int t = blockIdx.x;
  if (t >= total_tokens) return;
  const int s = seq_of_token(cu, num_seqs, t);
  for (int wi = threadIdx.x; wi < n_win; wi += blockDim.x) {
    int v = -1;
    if (s >= 0) {
      const int p = t - cu[s];
      const int src = p - n_win + 1 + wi;
      if (src >= 0) v = cu[s] + src;
    }
    out[t * ld + wi] = v;
  }
}

__global__ void hca_idxs_kernel(const int32_t* cu, const int32_t* offs, int num_seqs, int total_tokens, int n_win,
                                int max_n_comp, int m_prime, int32_t* out, int64_t ld) {
  const int t = blockIdx.x;
  const int s = seq_of_token(cu, num_seqs, t);
  const int p = s >= 0 ? t - cu[s] : 0;
  const int n_causal = s >= 0 ? min((p + m_prime - 1) / m_prime, max_n_comp) : 0;
  for (int j = threadIdx.x; j < n_win + max_n_comp; j += blockDim.x) {
    int v = -1;
    if (s >= 0) {
      if (j < n_win) {
        const int src = p - n_win + 1 + j;
        if (src >= 0) v = cu[s] + src;
      } else if (j - n_win < n_causal) {
        v = total_tokens + offs[s] + (j - n_win);
      }
    }
    out[t * ld + j] = v;
  }
}

// Decode rows: window = ctx - n_win + wi (>= 0); with m_prime > 0 the HCA
// compressed part ctx + offs[s] + ci for ci < min(ceil(ctx/m'), n_c, cols),
// with m_prime == 0 the compressed columns are set to -1 (the CSA indexer
// fills them afterwards).
__global__ void decode_idxs_kernel(const int32_t* context_lens, const int32_t* offs, int num_seqs, int n_win,
                                   int n_comp_cols, int m_prime, int32_t* out, int64_t ld) {
  const int s = blockIdx.x;
  const int ctx = context_lens[s];
  int n_causal = 0;
  if (m_prime > 0) {
    const int nc = offs[s + 1] - offs[s];
    n_causal = min(min((ctx + m_prime - 1) / m_prime, nc), n_comp_cols);
  }
  for (int j = threadIdx.x; j < n_win + n_comp_cols; j += blockDim.x) {
    int v = -1;
    if (j < n_win) {
      const int pos = ctx - n_win + j;
      if (pos >= 0) v = pos;
    } else if (j - n_win < n_causal) {
      v = ctx + offs[s] + (j - n_win);
    }
    out[s * ld + j] = v;
  }
}

// Slot offsets from lengths (is_cu = 0) or cu_seqlens (is_cu = 1): max(1,
// ceil(L / stride)) slots per non-empty sequence, cumulative (CSA:38-59).  One
// CTA: each thread scans a contiguous run of sequences, the run totals are
// scanned in shared memory.  A total above `capacity` (>= 0) records error 3
// and the offsets are clamped to the capacity.
__global__ void __launch_bounds__(1024) comp_offsets_kernel(const int32_t* lens, int num_seqs, int is_cu,
                                                            int stride, int64_t capacity, int32_t* offs) {
  __shared__ int64_t part[1024];
  const int t = threadIdx.x, nt = blockDim.x;
  const int per = (num_seqs + nt - 1) / nt;
  const int b0 = min(t * per, num_seqs), b1 = min(b0 + per, num_seqs);
  auto slots = [&](int s) -> int64_t {
    const int64_t L = is_cu ? static_cast<int64_t>(lens[s + 1]) - lens[s] : lens[s];
    return L > 0 ? ((L + stride - 1) / stride > 1 ? (L + stride - 1) / stride : int64_t{1}) : int64_t{0};
  };
  int64_t sum = 0;
  for (int s = b0; s < b1; ++s) sum += slots(s);
  part[t] = sum;
  __syncthreads();
  for (int off = 1; off < nt; off <<= 1) {  // inclusive Hillis-Steele scan of the run totals
    const int64_t v = t >= off ? part[t - off] : 0;
    __syncthreads();
    part[t] += v;
    __syncthreads();
  }
  int64_t run = part[t] - sum;  // exclusive prefix of this thread's run
  // past the capacity the offsets stop growing: later sequences get no slots,
  // so nothing that reads these offsets touches a row beyond the capacity
  const int64_t cap = capacity >= 0 ? capacity : INT64_MAX;
  if (t == 0) offs[0] = 0;
  for (int s = b0; s < b1; ++s) {
    run += slots(s);
    offs[s + 1] = static_cast<int32_t>(min(run, cap));
  }
  if (t == nt - 1 && part[t] > cap) record_error(3);
}

int comp_offsets_launch(const int32_t* lens, int num_seqs, int is_cu, int stride, int64_t capacity, int32_t* offs,
                        cudaStream_t st) {
  comp_offsets_kernel<<<1, 1024, 0, st>>>(lens, num_seqs, is_cu, stride, capacity, offs);
  return 0;
}

int token_to_seq_launch(const int32_t* cu, int num_seqs, int total_tokens, int32_t* out, cudaStream_t st) {
  if (total_tokens <= 0) return 0;
  token_to_seq_kernel<<<(total_tokens + 255) / 256, 256, 0, st>>>(cu, num_seqs, total_tokens, out);
  return 0;
}

int window_idxs_launch(const int32_t* cu, int num_seqs, int total_tokens, int n_win, int32_t* out, int64_t ld,
                       cudaStream_t st) {
  if (total_tokens <= 0 || n_win <= 0) return 0;
  window_idxs_kernel<<<total_tokens, 64, 0, st>>>(cu, num_seqs, total_tokens, n_win, out, ld);
  return 0;
}

int hca_idxs_launch(const int32_t* cu, const int32_t* offs, int num_seqs, int total_tokens, int n_win,
                    int max_n_comp, int m_prime, int32_t* out, int64_t ld, cudaStream_t st) {
  if (total_tokens <= 0 || n_win + max_n_comp <= 0) return 0;
  hca_idxs_kernel<<<total_tokens, 128, 0, st>>>(cu, offs, num_seqs, total_tokens, n_win, max_n_comp, m_prime, out,
                                                ld);
  return 0;
}

int decode_idxs_launch(const int32_t* context_lens, const int32_t* offs, int num_seqs, int n_win, int n_comp_cols,
                       int m_prime, int32_t* out, int64_t ld, cudaStream_t st) {
  if (num_seqs <= 0 || n_win + n_comp_cols <= 0) return 0;
  decode_idxs_kernel<<<num_seqs, 128, 0, st>>>(context_lens, offs, num_seqs, n_win, n_comp_cols, m_prime, out, ld);
  return 0;
}

// ---------------------------------------------------------------------------
// CSA Lightning indexer: scores + top-k, one CTA per query row
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float round_to_t(float x) {
  return Elem<T>::to_f(Elem<T>::from_f(x));
}
template <>
__device__ __forceinline__ float round_to_t<float>(float x) {
  return x;
}

// Top-k selection: up to kIdxRoundsMax picks by repeated block argmax, more
// by one bitonic sort of the (at most kIdxSortMax) causal slots.
constexpr int kIdxRoundsMax = 16;
constexpr int kIdxSortMax = 8192;

// Unscaled dot products q . ck[i] for slots i in [i_begin, i_end), rounded to
// T, handed to sink(i, score): 16-byte loads, lane l owns dims [8l, 8l+8) and
// [8l+256, 8l+264) (head_dim <= 512); a warp scores SPW slots per step with all
// their loads in flight.  Warp w of nwarps starts at slot i_begin + w * SPW.
template <typename T, int SPW, class Sink>
__device__ __forceinline__ void score_slots_vec(const T* q, const T* ck, int64_t sck0, int head_dim, int i_begin,
                                                int i_end, int warp, int nwarps, int lane, Sink&& sink) {
  const int nch = head_dim / 8;
  float qv[16];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int ch = lane + 32 * c;
    uint4 u = make_uint4(0, 0, 0, 0);
    if (ch < nch) u = *reinterpret_cast<const uint4*>(q + ch * 8);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = Elem<T>::unpack2(w[e]);
      qv[c * 8 + 2 * e] = f.x;
      qv[c * 8 + 2 * e + 1] = f.y;
    }
  }
  for (int i0 = i_begin + warp * SPW; i0 < i_end; i0 += nwarps * SPW) {
    uint4 kv[SPW][2];
#pragma unroll
    for (int si = 0; si < SPW; ++si)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int ch = lane + 32 * c;
        kv[si][c] = make_uint4(0, 0, 0, 0);
        if (i0 + si < i_end && ch < nch)
          kv[si][c] = *reinterpret_cast<const uint4*>(ck + static_cast<int64_t>(i0 + si) * sck0 + ch * 8);
      }
    float acc[SPW];
#pragma unroll
    for (int si = 0; si < SPW; ++si) {
      float sacc = 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint32_t w[4] = {kv[si][c].x, kv[si][c].y, kv[si][c].z, kv[si][c].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = Elem<T>::unpack2(w[e]);
          sacc = fmaf(qv[c * 8 + 2 * e], f.x, sacc);
          sacc = fmaf(qv[c * 8 + 2 * e + 1], f.y, sacc);
        }
      }
      acc[si] = warp_sum(sacc);
    }
    // lanes 0..SPW-1 hand over the scores (selects, not a register-indexed load)
    float mine = acc[0];
#pragma unroll
    for (int si = 1; si < SPW; ++si)
      if (lane == si) mine = acc[si];
    if (lane < SPW && i0 + lane < i_end) sink(i0 + lane, round_to_t<T>(mine));
  }
}

// Decode rows (one query per sequence, each against its own slots): the
// scores of a row split over CTAs of 256 slots each, written rounded to T into
// a scratch [rows, sld] that the selection (csa_indexer_kernel) reads -- one
// CTA per row alone leaves most SMs idle and its loads latency-bound.
template <typename T>
__global__ void __launch_bounds__(256) csa_decode_scores_kernel(const IndexerArgs a, T* scores, int64_t sld) {
  const int row = blockIdx.x;
  const int pos = a.context_lens[row];
  const int c0 = a.comp_offsets[row];
  const int nc = min(a.comp_offsets[row + 1] - c0, a.max_comp_per_seq);
  const int n_valid = pos <= 0 ? 0 : min(nc, (pos + a.m - 1) / a.m);
  const int i_begin = blockIdx.y * 256, i_end = min(n_valid, i_begin + 256);
  if (i_begin >= i_end) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const T* q = reinterpret_cast<const T*>(a.q) + static_cast<int64_t>(row) * a.sq[0] + (a.num_q_heads - 1) * a.sq[1];
  const T* ck = reinterpret_cast<const T*>(a.ck) + static_cast<int64_t>(c0) * a.sck[0] + (a.num_kv_heads - 1) * a.sck[1];
  T* out = scores + static_cast<int64_t>(row) * sld;
  score_slots_vec<T, 4>(q, ck, a.sck[0], a.head_dim, i_begin, i_end, warp, 8, lane,
                        [&](int i, float v) { out[i] = Elem<T>::from_f(v); });
}

// NT threads; SPW slots scored per warp step (all their loads in flight at
// once): 256 x 4 when there are many rows, 512 x 8 for the few long rows of
// decode, where one CTA per row leaves most SMs idle and the score loads are
// latency-bound.
template <typename T, int NT, int SPW>
__global__ void __launch_bounds__(NT) csa_indexer_kernel(const IndexerArgs a) {
  extern __shared__ float sc[];  // [max_comp_per_seq] scores, -inf once taken
  __shared__ float red_v[NT / 32];
  __shared__ int red_i[NT / 32];
  const int row = blockIdx.x;
  const bool decode = a.cu_seqlens == nullptr;
  int s, pos;
  if (decode) {
    s = row;
    pos = a.context_lens[s];
  } else {
    s = seq_of_token(a.cu_seqlens, a.num_seqs, row);
    if (s < 0) return;
    pos = row - a.cu_seqlens[s];
  }
  const int c0 = a.comp_offsets[s];
  // the score array holds max_comp_per_seq slots (a bound the caller derives)
  const int nc = min(a.comp_offsets[s + 1] - c0, a.max_comp_per_seq);
  if (nc <= 0) return;
  const int k_sel = min(a.top_k, nc);
  // slot i is causal iff i*m < pos  <=>  i < ceil(pos/m)
  const int n_valid = pos <= 0 ? 0 : min(nc, (pos + a.m - 1) / a.m);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const T* q = reinterpret_cast<const T*>(a.q) + row * a.sq[0] + (a.num_q_heads - 1) * a.sq[1];
  const T* ck = reinterpret_cast<const T*>(a.ck) + static_cast<int64_t>(c0) * a.sck[0] + (a.num_kv_heads - 1) * a.sck[1];
  bool vec = false;
  if constexpr (sizeof(T) == 2) {
    vec = a.sq[2] == 1 && a.sck[2] == 1 && a.head_dim % 8 == 0 && a.sck[0] % 8 == 0 &&
          ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(ck)) & 15) == 0;
  }
  if (a.scores) {
    // scores computed on the tensor cores (already rounded to T)
    const T* srow = reinterpret_cast<const T*>(a.scores) + static_cast<int64_t>(row) * a.sld;
    for (int i = threadIdx.x; i < n_valid; i += NT) sc[i] = Elem<T>::to_f(srow[i]);
  } else if (vec) {
    // 16-byte loads: lane l owns dims [8l, 8l+8) and [8l+256, 8l+264); a warp
    // scores SPW slots per step with all their loads in flight at once
    if constexpr (sizeof(T) == 2)
      score_slots_vec<T, SPW>(q, ck, a.sck[0], a.head_dim, 0, n_valid, warp, nwarps, lane,
                              [&](int i, float v) { sc[i] = v; });
  } else {
    float qr[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int d = lane + 32 * j;
      qr[j] = d < a.head_dim ? Elem<T>::to_f(q[d * a.sq[2]]) : 0.f;
    }
    for (int i = warp; i < n_valid; i += nwarps) {
      const T* kr = ck + static_cast<int64_t>(i) * a.sck[0];
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int d = lane + 32 * j;
        if (d < a.head_dim) acc += qr[j] * Elem<T>::to_f(kr[d * a.sck[2]]);
      }
      acc = warp_sum(acc);
      if (lane == 0) sc[i] = round_to_t<T>(acc);
    }
  }
  __syncthreads();
  const int64_t base = (decode ? static_cast<int64_t>(pos) : static_cast<int64_t>(a.total_tokens)) + c0;
  int32_t* out = a.out + static_cast<int64_t>(row) * a.ld + a.n_win;
  const int n_pick = min(k_sel, n_valid);
  if (n_pick > kIdxRoundsMax && n_valid <= kIdxSortMax) {
    // Many picks: sort the causal slots once.  Key = order-preserving bits of
    // the score (with -0 folded into +0, so equal scores compare equal as in
    // the rounds below) above the complemented slot index: descending key
    // order is descending score with ties to the lower slot.  Padding keys are
    // 0, below every real key.
    unsigned long long* key = reinterpret_cast<unsigned long long*>(sc);
    int n_pad = 1;
    while (n_pad < n_valid) n_pad <<= 1;
    // scores live in the first n_valid floats of the same buffer: read them
    // all before any key is written
    float own[kIdxSortMax / NT];
#pragma unroll
    for (int u = 0; u < kIdxSortMax / NT; ++u) {
      const int i = threadIdx.x + u * NT;
      own[u] = i < n_valid ? sc[i] + 0.f : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < kIdxSortMax / NT; ++u) {
      const int i = threadIdx.x + u * NT;
      if (i < n_pad) {
        unsigned long long kv = 0ull;
        if (i < n_valid) {
          uint32_t b = __float_as_uint(own[u]);
          b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
          kv = (static_cast<unsigned long long>(b) << 32) | (0xffffffffu - static_cast<uint32_t>(i));
        }
        key[i] = kv;
      }
    }
    __syncthreads();
    for (int kk = 2; kk <= n_pad; kk <<= 1) {
      for (int j = kk >> 1; j > 0; j >>= 1) {
        for (int i = threadIdx.x; i < n_pad; i += blockDim.x) {
          const int ixj = i ^ j;
          if (ixj > i) {
            const unsigned long long x = key[i], y = key[ixj];
            if (((i & kk) == 0) ? (x < y) : (x > y)) {
              key[i] = y;
              key[ixj] = x;
            }
          }
        }
        __syncthreads();
      }
    }
    for (int r = threadIdx.x; r < n_pick; r += blockDim.x)
      out[r] = static_cast<int32_t>(base + (0xffffffffu - static_cast<uint32_t>(key[r] & 0xffffffffull)));
    for (int r = n_pick + threadIdx.x; r < k_sel; r += blockDim.x) out[r] = static_cast<int32_t>(base + r);
    return;
  }
  for (int r = 0; r < n_pick; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n_valid; i += blockDim.x) {
      const float v = sc[i];
      if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      red_v[warp] = bv;
      red_i[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float v = red_v[0];
      int ix = red_i[0];
      for (int w = 1; w < nwarps; ++w)
        if (red_v[w] > v || (red_v[w] == v && red_i[w] < ix)) {
          v = red_v[w];
          ix = red_i[w];
        }
      // a slot already taken is marked with NaN, which never wins a comparison
      if (ix < n_valid) {
        out[r] = static_cast<int32_t>(base + ix);
        sc[ix] = __int_as_float(0x7fffffff);
      } else {
        out[r] = -1;
      }
    }
    __syncthreads();
  }
  for (int r = n_pick + threadIdx.x; r < k_sel; r += blockDim.x) out[r] = static_cast<int32_t>(base + r);
}

template <typename T, int NT, int SPW>
static int launch_indexer(const IndexerArgs& a, int rows, size_t smem, cudaStream_t st) {
  auto kern = csa_indexer_kernel<T, NT, SPW>;
  if (const int r = ensure_smem_attr(reinterpret_cast<const void*>(kern), static_cast<int>(smem))) return r;
  kern<<<rows, NT, smem, st>>>(a);
  return 0;
}

int csa_indexer_launch(const IndexerArgs& a, cudaStream_t st) {
  const int rows = a.cu_seqlens ? a.total_tokens : a.num_seqs;
  if (rows <= 0) return 0;
  if (a.head_dim > 512) return set_error(2, "csa indexer: head_dim > 512 is not supported");
  size_t smem = static_cast<size_t>(a.max_comp_per_seq > 0 ? a.max_comp_per_seq : 1) * sizeof(float);
  if (a.top_k > kIdxRoundsMax && a.max_comp_per_seq <= kIdxSortMax) {
    // room for the sort keys: 8 bytes per slot, padded to a power of two
    size_t n_pad = 1;
    while (n_pad < static_cast<size_t>(a.max_comp_per_seq)) n_pad <<= 1;
    if (n_pad * sizeof(unsigned long long) > smem) smem = n_pad * sizeof(unsigned long long);
  }
  if (smem > 200 * 1024) return set_error(2, "csa indexer: more than 51200 compressed slots in one sequence");
  IndexerArgs b = a;
  if (!a.scores) {
    // prefill rows: the dot products as one tensor-core GEMM per tile, then selection
    int64_t sld = 0;
    int err = 0;
    if (csa_scores_tc_launch(a, st, &sld, &err)) {
      if (err) return err;
      b.scores = a.ws;
      b.sld = sld;
      // up to 1024 slots per sequence: one warp per row sorts in registers
      if (csa_select_warp_launch(b, st)) return 0;
    } else if (!a.cu_seqlens && a.dtype != kF32 && a.ws && a.head_dim % 8 == 0 && a.head_dim <= 512 &&
               a.sq[2] == 1 && a.sck[2] == 1 && a.sq[0] % 8 == 0 && a.sq[1] % 8 == 0 && a.sck[0] % 8 == 0 &&
               a.sck[1] % 8 == 0 && ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.ck)) & 15) == 0 &&
               a.ws_bytes >= csa_scores_ws_bytes(rows, a.max_comp_per_seq, a.dtype)) {
      // decode rows: the scores split over CTAs of 256 slots, then the selection
      const int64_t ld = (static_cast<int64_t>(a.max_comp_per_seq) + 127) / 128 * 128;
      const dim3 grid(rows, static_cast<unsigned>((a.max_comp_per_seq + 255) / 256));
      if (a.dtype == kBF16)
        csa_decode_scores_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(a, reinterpret_cast<__nv_bfloat16*>(a.ws), ld);
      else
        csa_decode_scores_kernel<__half><<<grid, 256, 0, st>>>(a, reinterpret_cast<__half*>(a.ws), ld);
      b.scores = a.ws;
      b.sld = ld;
      // up to 2048 slots: the hybrid register / shared-memory sort
      if (csa_select_block_launch(b, rows, st)) return 0;
    }
  }
  // few rows (decode): wider CTAs with more score loads in flight
  const bool wide = rows < 2 * num_sms();
  if (a.dtype == kBF16) return wide ? launch_indexer<__nv_bfloat16, 512, 8>(b, rows, smem, st)
                                    : launch_indexer<__nv_bfloat16, 256, 4>(b, rows, smem, st);
  if (a.dtype == kF16) return wide ? launch_indexer<__half, 512, 8>(b, rows, smem, st)
                                   : launch_indexer<__half, 256, 4>(b, rows, smem, st);
  return launch_indexer<float, 256, 4>(b, rows, smem, st);
}

}  // namespace tak

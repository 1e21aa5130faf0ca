// The split-KV paged decode as device functions of one work unit and of the
// split combine, shared by the decode kernels (paged_decode.cu: one unit per
// CTA, the combine as a second launch) and the mixed prefill + decode kernel
// (mixed_step.cu: units pulled from a device work queue, the combine run by
// the last split to finish).  The algorithm is described in paged_decode.cu.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace tak {

struct DecodeParams {
  const void* q;
  int64_t sq_s, sq_h, sq_d;
  const int32_t* block_tables;
  int64_t sbt_s, sbt_b;
  const int32_t* context_lens;
  void* out;
  int64_t so_s, so_h, so_d;
  float* lse;    // [B, H] contiguous, may be null
  float* ws_o;   // [B, H, max_splits, D]
  float* ws_ml;  // [B, H, max_splits, 2]
  int B, H, Hkv, G, D, block_size, pages_per_split, max_splits, head_chunks;
  int max_ctx;  // max_blocks * block_size: rows past the block table are ignored
  float scale_log2;
};

// Shared-memory bytes of decode_unit (1024-byte aligned start).
template <int D, int CH, int NS>
struct DecodeSmem {
  static constexpr int STAGE = 2 * (D / 64) * CH * 128;
  static constexpr int MERGE = 4 * 16 * D * 4 + 4 * 16 * 2 * 4;
  static constexpr int BAR_OFF = NS * STAGE > MERGE ? NS * STAGE : MERGE;
  static constexpr int BYTES = BAR_OFF + 2 * NS * 8;
};

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// One split-KV work unit: split `split` of (KV head chunk y, sequence seq),
// run by a group of 160 threads (tid 0-159: warps 0-3 consume, warp 4 loads)
// on shared memory at `smem` (DecodeSmem<D, CH, NS>::BYTES, 1024-byte aligned).
// bar_all / bar_cons are the named barriers of the whole group and of its 128
// consumer threads.  Returns true when it wrote split partials (the sequence
// has several splits) that a combine must merge.
template <typename T, int D, int CH, int NS>
__device__ __forceinline__ bool decode_unit(const CUtensorMap* tmK, const CUtensorMap* tmV, const DecodeParams& p,
                                            int split, int y, int seq, uint8_t* smem, int tid, int bar_all,
                                            int bar_cons) {
  constexpr int NREG = D / 64;        // 64-element (128-byte) column blocks per row
  constexpr int TILE = CH * 128;      // bytes of one column block of CH rows
  constexpr int STAGE = 2 * NREG * TILE;
  constexpr int ACTIVE = CH / 16;     // consumer warps with rows in a chunk
  constexpr int MERGE = 4 * 16 * D * 4 + 4 * 16 * 2 * 4;   // epilogue buffers (reuse the ring)
  constexpr int BAR_OFF = NS * STAGE > MERGE ? NS * STAGE : MERGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* empty = full + NS;

  const int kvh = y / p.head_chunks;
  const int hc = y % p.head_chunks;
  const int h0 = kvh * p.G + hc * 16;
  const int gcnt = min(16, p.G - hc * 16);
  const int ctx = min(p.context_lens[seq], p.max_ctx);
  const int split_tokens = p.pages_per_split * p.block_size;
  const int tok0 = split * split_tokens;
  const int warp = tid >> 5, lane = tid & 31;

  if (ctx <= 0) {  // empty context: out = 0, lse = -inf (reference leaves it undefined)
    if (split == 0 && tid < 128) {
      for (int i = tid; i < gcnt * D; i += 128) {
        const int r = i / D, d = i % D;
        reinterpret_cast<T*>(p.out)[seq * p.so_s + (h0 + r) * p.so_h + d * p.so_d] = Elem<T>::from_f(0.f);
      }
      if (p.lse && tid < gcnt) p.lse[seq * p.H + h0 + tid] = -INFINITY;
    }
    return false;
  }
  if (tok0 >= ctx) return false;  // this split is past the end of the sequence
  const int tok1 = min(ctx, tok0 + split_tokens);
  const int n_chunks = (tok1 - tok0 + CH - 1) / CH;
  const int n_splits = (ctx + split_tokens - 1) / split_tokens;

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);
    }
    fence_barrier_init();
  }
  named_bar_sync(bar_all, 160);

  if (warp == 4) {
    // ---------------- producer: TMA loads of K / V chunks ----------------
    if (lane == 0) {
      tma_prefetch_desc(tmK);
      tma_prefetch_desc(tmV);
      for (int c = 0; c < n_chunks; ++c) {
        const int s = c % NS;
        if (c >= NS && !mbar_wait(&empty[s], ((c / NS) - 1) & 1)) break;
        const int tok = tok0 + c * CH;
        const int lpage = tok / p.block_size;
        const int row = tok % p.block_size;
        const int phys = p.block_tables[seq * p.sbt_s + lpage * p.sbt_b];
        uint8_t* st = smem + s * STAGE;
        mbar_arrive_expect_tx(&full[s], STAGE);
#pragma unroll
        for (int r = 0; r < NREG; ++r) tma_load_4d(st + r * TILE, tmK, &full[s], r * 64, row, kvh, phys);
#pragma unroll
        for (int r = 0; r < NREG; ++r) tma_load_4d(st + (NREG + r) * TILE, tmV, &full[s], r * 64, row, kvh, phys);
      }
    }
    return false;
  }

  // ---------------- consumers: warps 0-3 ----------------
  const int g = lane >> 2, t4 = lane & 3;
  const T* qp = reinterpret_cast<const T*>(p.q) + seq * p.sq_s;
  uint32_t qa[D / 16][4];
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = g + ((j & 1) ? 8 : 0);
      const int col = ks * 16 + 2 * t4 + ((j & 2) ? 8 : 0);
      float a = 0.f, b = 0.f;
      if (r < gcnt) {
        const T* src = qp + (h0 + r) * p.sq_h + col * p.sq_d;
        a = Elem<T>::to_f(src[0]);
        b = Elem<T>::to_f(src[p.sq_d]);
      }
      qa[ks][j] = Elem<T>::pack2(a, b);
    }
  }

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const uint32_t smem_base = smem_u32(smem);
  const int r0 = warp * 16;

  for (int c = 0; c < n_chunks; ++c) {
    const int s = c % NS;
    if (!mbar_wait(&full[s], (c / NS) & 1)) break;
    const int tokbase = tok0 + c * CH + r0;
    if (warp < ACTIVE && tokbase < tok1) {
      const uint32_t kbase = smem_base + s * STAGE;
      const uint32_t vbase = kbase + NREG * TILE;
      // rows past the end of the context may hold stale data: zero their V rows
      if (tokbase + 16 > tok1) {
        uint8_t* vt = smem + s * STAGE + NREG * TILE;
        for (int i = lane; i < 16 * NREG * 8; i += 32) {
          const int rr = i / (NREG * 8), cidx = i % (NREG * 8);
          if (tokbase + rr >= tok1)
            *reinterpret_cast<uint4*>(vt + (cidx / 8) * TILE + sw128(r0 + rr, cidx % 8)) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
        __syncwarp();
      }
      float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const int row = r0 + (mi >> 1) * 8 + rr;
        const int chunk = 2 * ks + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kbase + (chunk >> 3) * TILE + sw128(row, chunk & 7), b0, b1, b2, b3);
        Mma<T>::run(sacc[0], qa[ks], b0, b1);
        Mma<T>::run(sacc[1], qa[ks], b2, b3);
      }
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int tok = tokbase + nt * 8 + 2 * t4 + (j & 1);
          const float v = (tok < tok1) ? sacc[nt][j] * p.scale_log2 : -INFINITY;
          sacc[nt][j] = v;
          mx[j >> 1] = fmaxf(mx[j >> 1], v);
        }
      float alpha[2], muse[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
        const float mnew = fmaxf(m_run[r], mx[r]);
        muse[r] = (mnew == -INFINITY) ? 0.f : mnew;
        alpha[r] = fast_exp2(m_run[r] - muse[r]);
        m_run[r] = mnew;
      }
      float psum[2] = {0.f, 0.f};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float e = fast_exp2(sacc[nt][j] - muse[j >> 1]);
          sacc[nt][j] = e;
          psum[j >> 1] += e;
        }
      l_run[0] = l_run[0] * alpha[0] + psum[0];
      l_run[1] = l_run[1] * alpha[1] + psum[1];
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        o[i][0] *= alpha[0];
        o[i][1] *= alpha[0];
        o[i][2] *= alpha[1];
        o[i][3] *= alpha[1];
      }
      uint32_t pa[4];
      pa[0] = Elem<T>::pack2(sacc[0][0], sacc[0][1]);
      pa[1] = Elem<T>::pack2(sacc[0][2], sacc[0][3]);
      pa[2] = Elem<T>::pack2(sacc[1][0], sacc[1][1]);
      pa[3] = Elem<T>::pack2(sacc[1][2], sacc[1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        const int row = r0 + (mi & 1) * 8 + rr;
        const int chunk = 2 * dp + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vbase + (chunk >> 3) * TILE + sw128(row, chunk & 7), b0, b1, b2, b3);
        Mma<T>::run(o[2 * dp], pa, b0, b1);
        Mma<T>::run(o[2 * dp + 1], pa, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // ---------------- merge the 4 warps ----------------
  l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], 1);
  l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], 2);
  l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], 1);
  l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], 2);
  named_bar_sync(bar_cons, 128);  // all consumers done with the ring
  float* obuf = reinterpret_cast<float*>(smem);          // [4][16][D]
  float* mlbuf = obuf + 4 * 16 * D;                      // [4][16][2]
#pragma unroll
  for (int nt = 0; nt < D / 8; ++nt) {
    const int d = nt * 8 + 2 * t4;
    obuf[(warp * 16 + g) * D + d] = o[nt][0];
    obuf[(warp * 16 + g) * D + d + 1] = o[nt][1];
    obuf[(warp * 16 + g + 8) * D + d] = o[nt][2];
    obuf[(warp * 16 + g + 8) * D + d + 1] = o[nt][3];
  }
  if (t4 == 0) {
    mlbuf[(warp * 16 + g) * 2] = m_run[0];
    mlbuf[(warp * 16 + g) * 2 + 1] = l_run[0];
    mlbuf[(warp * 16 + g + 8) * 2] = m_run[1];
    mlbuf[(warp * 16 + g + 8) * 2 + 1] = l_run[1];
  }
  named_bar_sync(bar_cons, 128);
  for (int i = tid; i < gcnt * D; i += 128) {
    const int r = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, mlbuf[(w * 16 + r) * 2]);
    const float Mu = (M == -INFINITY) ? 0.f : M;
    float L = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float f = fast_exp2(mlbuf[(w * 16 + r) * 2] - Mu);
      L += mlbuf[(w * 16 + r) * 2 + 1] * f;
      acc += obuf[(w * 16 + r) * D + d] * f;
    }
    const int h = h0 + r;
    if (n_splits == 1) {
      reinterpret_cast<T*>(p.out)[seq * p.so_s + h * p.so_h + d * p.so_d] =
          Elem<T>::from_f(L > 0.f ? acc / L : 0.f);
      if (d == 0 && p.lse) p.lse[seq * p.H + h] = L > 0.f ? (M + __log2f(L)) * kLn2 : -INFINITY;
    } else {
      const int64_t slot = (static_cast<int64_t>(seq) * p.H + h) * p.max_splits + split;
      p.ws_o[slot * D + d] = acc;
      if (d == 0) {
        p.ws_ml[slot * 2] = M;
        p.ws_ml[slot * 2 + 1] = L;
      }
    }
  }
  return n_splits > 1;
}

// Merge the split partials of one (sequence, KV head, head chunk).  One warp
// per query head reduces the splits' maxima and weighted sums with warp
// shuffles (lane j holds splits j and j + 32; at most 64 splits), leaving each
// split's weight 2^(m_j - M) in shared memory; then each thread merges 4
// consecutive output elements of one head with all splits' 16-byte loads
// independent (one memory round trip, not a chain).  Run by 128 threads
// (tid 0-127) with scratch wts[16 * 64] and inv_l[16]; `bar` names their
// barrier.  Partials are read through L2 (another SM may have written them).
template <typename T>
__device__ __forceinline__ void decode_combine(const DecodeParams& p, int seq, int y, int tid, float* wts,
                                               float* inv_l, int bar) {
  const int kvh = y / p.head_chunks, hc = y % p.head_chunks;
  const int ctx = min(p.context_lens[seq], p.max_ctx);
  const int split_tokens = p.pages_per_split * p.block_size;
  const int n = (ctx + split_tokens - 1) / split_tokens;
  if (ctx <= 0 || n <= 1) return;
  const int h0 = kvh * p.G + hc * 16;
  const int gcnt = min(16, p.G - hc * 16);
  const int warp = tid >> 5, lane = tid & 31;
  for (int r = warp; r < gcnt; r += 4) {
    const float2* ml =
        reinterpret_cast<const float2*>(p.ws_ml + (static_cast<int64_t>(seq) * p.H + h0 + r) * p.max_splits * 2);
    float2 a = make_float2(-INFINITY, 0.f), b = make_float2(-INFINITY, 0.f);
    if (lane < n) a = __ldcg(ml + lane);
    if (lane + 32 < n) b = __ldcg(ml + lane + 32);
    const float M = warp_max(fmaxf(a.x, b.x));
    const float Mu = (M == -INFINITY) ? 0.f : M;
    const float wa = lane < n ? fast_exp2(a.x - Mu) : 0.f;
    const float wb = lane + 32 < n ? fast_exp2(b.x - Mu) : 0.f;
    const float L = warp_sum(a.y * wa + b.y * wb);
    if (lane < n) wts[r * n + lane] = wa;
    if (lane + 32 < n) wts[r * n + lane + 32] = wb;
    if (lane == 0) {
      inv_l[r] = L > 0.f ? 1.f / L : 0.f;
      if (p.lse) p.lse[seq * p.H + h0 + r] = L > 0.f ? (M + __log2f(L)) * kLn2 : -INFINITY;
    }
  }
  named_bar_sync(bar, 128);
  const int nvec = p.D / 4;
  for (int i = tid; i < gcnt * nvec; i += 128) {
    const int r = i / nvec, d = (i - r * nvec) * 4;
    const float4* src =
        reinterpret_cast<const float4*>(p.ws_o + ((static_cast<int64_t>(seq) * p.H + h0 + r) * p.max_splits) * p.D + d);
    const float* w = wts + r * n;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    int j = 0;
    for (; j + 8 <= n; j += 8) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldcg(src + static_cast<int64_t>(j + u) * nvec);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float wu = w[j + u];
        a.x = fmaf(wu, v[u].x, a.x);
        a.y = fmaf(wu, v[u].y, a.y);
        a.z = fmaf(wu, v[u].z, a.z);
        a.w = fmaf(wu, v[u].w, a.w);
      }
    }
    for (; j < n; ++j) {
      const float4 v = __ldcg(src + static_cast<int64_t>(j) * nvec);
      const float wu = w[j];
      a.x = fmaf(wu, v.x, a.x);
      a.y = fmaf(wu, v.y, a.y);
      a.z = fmaf(wu, v.z, a.z);
      a.w = fmaf(wu, v.w, a.w);
    }
    const float il = inv_l[r];
    T* o = reinterpret_cast<T*>(p.out) + seq * p.so_s + (h0 + r) * p.so_h + d * p.so_d;
    o[0] = Elem<T>::from_f(a.x * il);
    o[p.so_d] = Elem<T>::from_f(a.y * il);
    o[2 * p.so_d] = Elem<T>::from_f(a.z * il);
    o[3 * p.so_d] = Elem<T>::from_f(a.w * il);
  }
}

// Tensor maps and parameters of the 128-dim, 64-row-chunk split-KV decode
// (paged_decode.cu), its split count per sequence and (KV head x head chunk)
// groups; -1 when these arguments do not take that path, else a status code.
int decode_fast_setup_d128(const PagedDecodeArgs& a, CUtensorMap* mk, CUtensorMap* mv, DecodeParams* p,
                           int* max_splits, int* groups);

}  // namespace tak

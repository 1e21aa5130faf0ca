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

// ---------------------------------------------------------------------------
// fast path
// ---------------------------------------------------------------------------
// Two CTAs per SM for head dims up to 128; a 256-dim ring (192 KB of shared
// memory) fits one CTA per SM, which may then use the full register file.
template <typename T, int D, int CH, int NS>
__global__ void __launch_bounds__(160, D >= 256 ? 1 : 2)
    paged_decode_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                           const DecodeParams p) {
  constexpr int NREG = D / 64;        // 64-element (128-byte) column blocks per row
  constexpr int TILE = CH * 128;      // bytes of one column block of CH rows
  constexpr int STAGE = 2 * NREG * TILE;
  constexpr int ACTIVE = CH / 16;     // consumer warps with rows in a chunk
  constexpr int MERGE = 4 * 16 * D * 4 + 4 * 16 * 2 * 4;   // epilogue buffers (reuse the ring)
  constexpr int BAR_OFF = NS * STAGE > MERGE ? NS * STAGE : MERGE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* empty = full + NS;

  // let the split-KV combine grid (launched with programmatic stream
  // serialization) be scheduled as this grid's last wave runs; it still waits
  // for this whole grid to complete before reading any partial
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int split = blockIdx.x;
  const int kvh = blockIdx.y / p.head_chunks;
  const int hc = blockIdx.y % p.head_chunks;
  const int seq = blockIdx.z;
  const int h0 = kvh * p.G + hc * 16;
  const int gcnt = min(16, p.G - hc * 16);
  const int ctx = min(p.context_lens[seq], p.max_ctx);
  const int split_tokens = p.pages_per_split * p.block_size;
  const int tok0 = split * split_tokens;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (ctx <= 0) {  // empty context: out = 0, lse = -inf (reference leaves it undefined)
    if (split == 0 && tid < 128) {
      for (int i = tid; i < gcnt * D; i += 128) {
        const int r = i / D, d = i % D;
        reinterpret_cast<T*>(p.out)[seq * p.so_s + (h0 + r) * p.so_h + d * p.so_d] = Elem<T>::from_f(0.f);
      }
      if (p.lse && tid < gcnt) p.lse[seq * p.H + h0 + tid] = -INFINITY;
    }
    return;
  }
  if (tok0 >= ctx) return;  // this split is past the end of the sequence
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
  __syncthreads();

  if (warp == 4) {
    // ---------------- producer: TMA loads of K / V chunks ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
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
        for (int r = 0; r < NREG; ++r) tma_load_4d(st + r * TILE, &tmK, &full[s], r * 64, row, kvh, phys);
#pragma unroll
        for (int r = 0; r < NREG; ++r) tma_load_4d(st + (NREG + r) * TILE, &tmV, &full[s], r * 64, row, kvh, phys);
      }
    }
    return;
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
  asm volatile("bar.sync 1, 128;" ::: "memory");  // all consumers done with the ring
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
  asm volatile("bar.sync 1, 128;" ::: "memory");
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
}

// Merge the split partials of one (sequence, KV head, head chunk).  One warp
// per query head reduces the splits' maxima and weighted sums with warp
// shuffles (lane j holds splits j and j + 32; at most 64 splits), leaving each
// split's weight 2^(m_j - M) in shared memory; then each thread merges 4
// consecutive output elements of one head with all splits' 16-byte loads
// independent (one memory round trip, not a chain).  When launched with
// programmatic stream serialization the grid may start while the
// partial-writing grid is still running; griddepcontrol.wait holds it until
// that grid has completed.
template <typename T>
__global__ void __launch_bounds__(128) paged_decode_combine_kernel(const DecodeParams p) {
  __shared__ float wts[16 * 64];
  __shared__ float inv_l[16];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int kvh = blockIdx.y / p.head_chunks, hc = blockIdx.y % p.head_chunks, seq = blockIdx.x;
  const int ctx = min(p.context_lens[seq], p.max_ctx);
  const int split_tokens = p.pages_per_split * p.block_size;
  const int n = (ctx + split_tokens - 1) / split_tokens;
  if (ctx <= 0 || n <= 1) return;
  const int h0 = kvh * p.G + hc * 16;
  const int gcnt = min(16, p.G - hc * 16);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int r = warp; r < gcnt; r += 4) {
    const float2* ml =
        reinterpret_cast<const float2*>(p.ws_ml + (static_cast<int64_t>(seq) * p.H + h0 + r) * p.max_splits * 2);
    float2 a = make_float2(-INFINITY, 0.f), b = make_float2(-INFINITY, 0.f);
    if (lane < n) a = ml[lane];
    if (lane + 32 < n) b = ml[lane + 32];
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
  __syncthreads();
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
      for (int u = 0; u < 8; ++u) v[u] = src[static_cast<int64_t>(j + u) * nvec];
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
      const float4 v = src[static_cast<int64_t>(j) * nvec];
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

template <typename T, int D, int CH>
static int launch_fast(const PagedDecodeArgs& a, int pps, int max_splits, int head_chunks, cudaStream_t st) {
  constexpr int NS = 3;
  constexpr int STAGE = 2 * (D / 64) * CH * 128;
  constexpr int MERGE = 4 * 16 * D * 4 + 4 * 16 * 2 * 4;
  constexpr int SMEM = (NS * STAGE > MERGE ? NS * STAGE : MERGE) + 2 * NS * 8 + 1024;
  CUtensorMap mk, mv;
  if (encode_cache_map(&mk, a.k_cache, a.sk, a.num_blocks, a.num_kv_heads, a.cache_rows, D, CH)) return 3;
  if (encode_cache_map(&mv, a.v_cache, a.sv, a.num_blocks, a.num_kv_heads, a.cache_rows, D, CH)) return 3;
  DecodeParams p{};
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

// CSA and HCA compression of one KV stream in a single pass over HBM.
//
// Semantics: compress_kv_overlap (CSA:9-69: slot i of a sequence pools rows
// [i*m, min(i*m + 2m, L))) and compress_kv_simple (HCA:9-69: slot i pools rows
// [i*m', min((i+1)*m', L))) applied to the same K and V, as a plain mean (the
// reference) or as the softmax(gate)-weighted sum over each window's rows.
// Calling the two reference functions reads every K/V row twice; here each row
// crosses HBM once (plus an m-row halo per m'-row chunk for the CSA windows
// that straddle two chunks).
//
// Work split.  A "chunk" is one HCA slot: m' rows of one sequence (the last
// chunk of a sequence may be shorter).  A unit is (chunk, KV head, 128-column
// slice of K or V); units are dealt to a persistent grid (one CTA per SM) as
// contiguous, equal-sized runs, so every SM streams the same number of bytes.
//
// Warp roles (448 threads):
//   warp 12     TMA producer: per unit one tiled load of (m' + m) rows x 128
//               columns (256-byte rows, no swizzle) into a ring of stages.
//   warp 13     gate warp: per chunk the row weights 2^(g - block max) (1 for
//               the mean), the block sums and maxima of every m-row block, and
//               from them the two merge factors of each CSA slot (block b and
//               block b+1) and the factor of each block in the HCA slot, into
//               a small ring of chunk entries.  It runs ahead of the consumers,
//               so the gate loads never stall the data stream.
//   warps 0-11  consumers in three groups of four taking units round-robin
//               (three consumer warps per SM sub-partition hide each other's
//               latencies).  In a group, warp w owns a quarter of the
//               chunk's blocks (plus the next block, for its last CSA slot); lane
//               l owns columns
//               [4l, 4l+4) of the slice.  Per block: weighted row sum from
//               shared memory; CSA slot b-1 = prev * A[b-1] + cur * B[b-1],
//               written as it completes; HCA partial += cur * H[b].  The four
//               HCA partials meet in shared memory and the group's first warp
//               writes the slot.
// Every wait is an mbarrier wait bounded in time; a timed-out wait records a
// device error, raises the CTA's abort flag and the roles unwind (the producer
// first waits, bounded, for its loads in flight).
#include "common.cuh"
#include "kernels.h"

namespace tak {

namespace fc {
constexpr int kCols = 128;    // columns per unit (one 256-byte row segment)
constexpr int kRing = 8;      // chunk-statistics entries
constexpr int kConsumers = 4; // consumer warps per group
constexpr int kGroups = 3;    // consumer groups (units dealt round-robin)
constexpr int kThreads = (kGroups * kConsumers + 2) * 32;
}  // namespace fc

struct FusedCompressParams {
  const float* gate;
  int64_t sg;
  const int32_t* cu_seqlens;
  const int32_t* csa_offsets;
  const int32_t* hca_offsets;
  int num_seqs;
  int64_t num_units;
  int heads, slices, k_slices;  // slices per head: (D + Dv) / 128, the first k_slices are K
  int m, mp, nb, rows;          // CSA stride, HCA window, blocks per chunk (mp / m), rows per load (mp + m)
  int rows_pad;                 // rows rounded up to a multiple of 4 (row-weight array length)
  int stages, stage_bytes, entry_floats;
  void* csa_k; int64_t sck[3];
  void* csa_v; int64_t scv[3];
  void* hca_k; int64_t shk[3];
  void* hca_v; int64_t shv[3];
};

// Position in a CTA's run of units: unit = (chunk c, head, slice), chunk c =
// chunk i of sequence s.  Advanced incrementally (one binary search per CTA).
struct FcCursor {
  int64_t c;
  int s, i, head, slice;
};

// Last sequence s with offs[s] <= slot, searched by a whole warp 32 ways at a
// time (one coalesced probe and a ballot per level: one global round trip for
// up to 32 sequences, instead of a chain of dependent loads).  All 32 lanes
// must call it; every lane gets the result.
__device__ __forceinline__ static int fc_find_seq_warp(const int32_t* offs, int num_seqs, int64_t slot) {
  const int lane = threadIdx.x & 31;
  int lo = 0, hi = num_seqs;  // answer in [lo, hi)
  while (hi - lo > 32) {
    const int step = (hi - lo + 31) / 32;
    const int idx = lo + lane * step;
    const bool le = idx < hi && offs[idx] <= slot;
    const unsigned m = __ballot_sync(0xffffffffu, le);
    const int last = m ? 31 - __clz(m) : 0;
    lo = lo + last * step;
    hi = min(lo + step, hi);
  }
  const int idx = lo + lane;
  const bool le = idx < hi && offs[idx] <= slot;
  const unsigned m = __ballot_sync(0xffffffffu, le);
  return lo + (m ? 31 - __clz(m) : 0);
}

__device__ __forceinline__ static void fc_cursor_init(FcCursor& q, const FusedCompressParams& p, int64_t u) {
  const int64_t per = static_cast<int64_t>(p.heads) * p.slices;
  q.c = u / per;
  const int rem = static_cast<int>(u - q.c * per);
  q.head = rem / p.slices;
  q.slice = rem - q.head * p.slices;
  q.s = fc_find_seq_warp(p.hca_offsets, p.num_seqs, q.c);
  q.i = static_cast<int>(q.c - p.hca_offsets[q.s]);
}

__device__ __forceinline__ static void fc_next_chunk(FcCursor& q, const FusedCompressParams& p) {
  ++q.c;
  ++q.i;
  while (q.s + 1 < p.num_seqs && p.hca_offsets[q.s + 1] <= q.c) {
    ++q.s;
    q.i = static_cast<int>(q.c - p.hca_offsets[q.s]);
  }
}

// next unit; true when it starts a new chunk
__device__ __forceinline__ static bool fc_cursor_next(FcCursor& q, const FusedCompressParams& p) {
  if (++q.slice < p.slices) return false;
  q.slice = 0;
  if (++q.head < p.heads) return false;
  q.head = 0;
  fc_next_chunk(q, p);
  return true;
}

struct FcChunk {
  int avail;     // rows of the load that belong to the sequence
  int nslots;    // CSA slots of this chunk
  int64_t tok0;  // first token of the chunk
  int64_t slot0; // first CSA slot of the chunk
};

__device__ __forceinline__ static FcChunk fc_chunk(const FusedCompressParams& p, int s, int i) {
  FcChunk r;
  const int start = p.cu_seqlens[s];
  const int L = p.cu_seqlens[s + 1] - start;
  r.avail = min(p.rows, L - i * p.mp);
  r.tok0 = start + static_cast<int64_t>(i) * p.mp;
  const int c0 = p.csa_offsets[s];
  r.nslots = min(p.nb, (p.csa_offsets[s + 1] - c0) - i * p.nb);
  r.slot0 = c0 + static_cast<int64_t>(i) * p.nb;
  return r;
}

// 4 outputs as one 8-byte global store (st.global: never aliases shared memory)
template <typename T>
__device__ __forceinline__ static void fc_store4(T* dst, const float* o) {
  uint2 q;
  q.x = Elem<T>::pack2(o[0], o[1]);
  q.y = Elem<T>::pack2(o[2], o[3]);
  __stcg(reinterpret_cast<uint2*>(dst), q);
}

// (c0, c1) + (w, w) * (a0, a1) as one packed fp32x2 FMA
__device__ __forceinline__ static void fc_ffma2(float& c0, float& c1, float w, float a0, float a1) {
  uint64_t c = (static_cast<uint64_t>(__float_as_uint(c1)) << 32) | __float_as_uint(c0);
  const uint64_t ww = (static_cast<uint64_t>(__float_as_uint(w)) << 32) | __float_as_uint(w);
  const uint64_t aa = (static_cast<uint64_t>(__float_as_uint(a1)) << 32) | __float_as_uint(a0);
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(c) : "l"(ww), "l"(aa));
  c0 = __uint_as_float(static_cast<uint32_t>(c));
  c1 = __uint_as_float(static_cast<uint32_t>(c >> 32));
}

template <typename T>
__device__ __forceinline__ static void fc_accum(float* acc, uint2 x, float w) {
  const float2 a = Elem<T>::unpack2(x.x), b = Elem<T>::unpack2(x.y);
  fc_ffma2(acc[0], acc[1], w, a.x, a.y);
  fc_ffma2(acc[2], acc[3], w, b.x, b.y);
}

// M, NB: CSA stride and blocks per chunk when known at compile time (the
// reference's m = 4, m' = 128 shape: every row load of a warp is issued before
// the first use); 0, 0 = runtime sizes.
template <typename T, int M, int NB>
__global__ void __launch_bounds__(fc::kThreads, 1)
    compress_csa_hca_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                            const FusedCompressParams p) {
  using namespace fc;
  // The dynamic shared array is used as declared (no integer rounding of its
  // address), so the compiler keeps every pointer derived from it in the
  // shared space: shared loads, and no aliasing with the global stores.
  extern __shared__ __align__(128) uint8_t smem[];
  if (smem_u32(smem) & 127u) {  // the launch provides a 128-byte aligned window; checked, never expected
    if (threadIdx.x == 0) record_error(3);
    return;
  }
  float* ring = reinterpret_cast<float*>(smem + static_cast<size_t>(p.stages) * p.stage_bytes);
  float* hpart = ring + kRing * p.entry_floats;  // [groups][2][4 warps][128 columns]
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(hpart + kGroups * 2 * kConsumers * kCols) + 7) & ~uintptr_t(7));
  uint64_t* full = bars;
  uint64_t* empty = full + p.stages;
  uint64_t* cfull = empty + p.stages;
  uint64_t* cempty = cfull + kRing;
  uint64_t* hfull = cempty + kRing;      // [groups][2]
  uint64_t* hfree = hfull + 2 * kGroups; // [groups][2]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(hfree + 2 * kGroups);
  const int m = M > 0 ? M : p.m;
  const int nb = NB > 0 ? NB : p.nb;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t G = gridDim.x;
  const int64_t u0 = p.num_units * blockIdx.x / G, u1 = p.num_units * (blockIdx.x + 1) / G;
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
    }
    for (int e = 0; e < kRing; ++e) {
      mbar_init(&cfull[e], 1);
      mbar_init(&cempty[e], kGroups * kConsumers);
    }
    for (int e = 0; e < 2 * kGroups; ++e) {
      mbar_init(&hfull[e], kConsumers);
      mbar_init(&hfree[e], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (u0 >= u1) return;
  FcCursor cur;
  fc_cursor_init(cur, p, u0);

  if (warp == kGroups * kConsumers) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      bool ok = true;
      int64_t n = 0;
      int64_t tok0 = p.cu_seqlens[cur.s] + static_cast<int64_t>(cur.i) * p.mp;
      for (int64_t u = u0; u < u1; ++u, ++n) {
        const int st = static_cast<int>(n % p.stages);
        if (n >= p.stages) {
          if (*abort_flag || !mbar_wait_sleep(&empty[st], ((n / p.stages) & 1) ^ 1)) {
            ok = false;
            break;
          }
        }
        const bool is_k = cur.slice < p.k_slices;
        const int col = (is_k ? cur.slice : cur.slice - p.k_slices) * kCols;
        mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(p.stage_bytes));
        tma_load_3d(smem + static_cast<size_t>(st) * p.stage_bytes, is_k ? &tmK : &tmV, &full[st], col, cur.head,
                    static_cast<int>(tok0));
        if (fc_cursor_next(cur, p) && u + 1 < u1)
          tok0 = p.cu_seqlens[cur.s] + static_cast<int64_t>(cur.i) * p.mp;
      }
      if (!ok) *abort_flag = 1;
      // loads still in flight land before the CTA can exit
      for (int64_t k = n > p.stages ? n - p.stages : 0; k < n; ++k)
        mbar_wait_sleep(&full[k % p.stages], (k / p.stages) & 1);
    }
    return;
  }

  const int64_t c_first = cur.c;
  if (warp == kGroups * kConsumers + 1) {
    // ---------------- gate warp: chunk statistics ----------------
    // The gate logits of chunk c + 1 are loaded (one batch of independent
    // loads per lane) while the statistics of chunk c are computed.
    bool ok = true;
    const int64_t c_last = (u1 - 1) / (static_cast<int64_t>(p.heads) * p.slices);
    constexpr int kGateRegs = 8;  // rows <= 256 = 8 per lane
    float gv[kGateRegs];
    int avail = 0;
    auto load_gates = [&](float* dst, int& av) {
      const int start = p.cu_seqlens[cur.s];
      av = min(p.rows, p.cu_seqlens[cur.s + 1] - start - cur.i * p.mp);
      const int64_t tok0 = start + static_cast<int64_t>(cur.i) * p.mp;
#pragma unroll
      for (int j = 0; j < kGateRegs; ++j) {
        const int r = lane + 32 * j;
        dst[j] = -INFINITY;
        if (r < av) dst[j] = p.gate ? __ldg(p.gate + (tok0 + r) * p.sg) : 0.f;
      }
    };
    load_gates(gv, avail);
    for (int64_t c = c_first; c <= c_last; ++c) {
      const int64_t k = c - c_first;
      const int e = static_cast<int>(k % kRing);
      if (k >= kRing) {
        if (*abort_flag || !mbar_wait_sleep(&cempty[e], ((k / kRing) & 1) ^ 1)) {
          ok = false;
          break;
        }
      }
      float* W = ring + e * p.entry_floats;       // [rows_pad] row weights
      float2* AB = reinterpret_cast<float2*>(W + p.rows_pad);  // [nb + 1] CSA factors of blocks b, b + 1 in slot b
      float* H = reinterpret_cast<float*>(AB + (nb + 1));      // [nb + 1] HCA factor of block b
      float* BM = H + (nb + 1);                   // [nb + 1] block max logit
      float* BS = BM + (nb + 1);                  // [nb + 1] block weight sum
#pragma unroll
      for (int j = 0; j < kGateRegs; ++j) {
        const int r = lane + 32 * j;
        if (r < p.rows) W[r] = gv[j];
      }
      const int av = avail;
      if (c < c_last) {
        fc_next_chunk(cur, p);
        load_gates(gv, avail);
      }
      __syncwarp();
      for (int b = lane; b <= nb; b += 32) {
        const int r0 = b * m, r1 = min(r0 + m, av);
        float mx = -INFINITY;
        for (int r = r0; r < r1; ++r) mx = fmaxf(mx, W[r]);
        float sum = 0.f;
        for (int r = r0; r < r1; ++r) {
          const float x = mx == -INFINITY ? 0.f : __expf(W[r] - mx);
          W[r] = x;
          sum += x;
        }
        BM[b] = mx;
        BS[b] = sum;
      }
      __syncwarp();
      float mh = -INFINITY;
      for (int b = lane; b < nb; b += 32) mh = fmaxf(mh, BM[b]);
      mh = warp_max(mh);
      float hs = 0.f;
      for (int b = lane; b < nb; b += 32) {
        const float f = BM[b] == -INFINITY ? 0.f : __expf(BM[b] - mh);
        H[b] = f;
        hs += f * BS[b];
      }
      hs = warp_sum(hs);
      const float hinv = hs > 0.f ? 1.f / hs : 0.f;
      for (int b = lane; b < nb; b += 32) {
        H[b] *= hinv;
        const float ma = BM[b], mb = BM[b + 1], Mx = fmaxf(ma, mb);
        const float fa = ma == -INFINITY ? 0.f : __expf(ma - Mx);
        const float fb = mb == -INFINITY ? 0.f : __expf(mb - Mx);
        const float den = BS[b] * fa + BS[b + 1] * fb;
        const float inv = den > 0.f ? 1.f / den : 0.f;
        AB[b] = make_float2(fa * inv, fb * inv);
      }
      __threadfence_block();
      __syncwarp();
      if (lane == 0) mbar_arrive(&cfull[e]);
    }
    if (!ok) *abort_flag = 1;
    return;
  }

  // ---------------- consumers: group g = warps [4g, 4g + 4) takes units g, g + 3, ... ----------------
  bool ok = true;
  const int grp = warp / kConsumers, wg = warp % kConsumers;
  const int b0 = wg * nb / kConsumers, b1 = (wg + 1) * nb / kConsumers;
  int64_t released = c_first;  // chunks before this one are released by this warp
  int e = 0;
  FcChunk ch{};
  bool new_chunk = true;
  for (int a = 0; a < grp; ++a) fc_cursor_next(cur, p);  // first unit of this group (its chunk is waited for)
  int64_t n = grp, ng = 0;  // CTA-local unit number, this group's unit number
  for (int64_t u = u0 + grp; u < u1; u += kGroups, n += kGroups, ++ng) {
    if (new_chunk) {
      // release every chunk before the current one (in order, skipped ones included)
      for (; released < cur.c; ++released) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&cempty[(released - c_first) % kRing]);
      }
      const int64_t k = cur.c - c_first;
      e = static_cast<int>(k % kRing);
      if (*abort_flag || !mbar_wait_sleep(&cfull[e], (k / kRing) & 1)) {
        ok = false;
        break;
      }
      ch = fc_chunk(p, cur.s, cur.i);
    }
    const float* W = ring + e * p.entry_floats;
    const float2* AB = reinterpret_cast<const float2*>(W + p.rows_pad);
    const float* H = reinterpret_cast<const float*>(AB + (nb + 1));
    const int st = static_cast<int>(n % p.stages);
    if (*abort_flag || !mbar_wait_sleep(&full[st], (n / p.stages) & 1)) {
      ok = false;
      break;
    }
    const bool is_k = cur.slice < p.k_slices;
    const int head = cur.head;
    const int col = (is_k ? cur.slice : cur.slice - p.k_slices) * kCols + lane * 4;
    const uint8_t* data = smem + static_cast<size_t>(st) * p.stage_bytes + lane * 8;
    T* csa_out = reinterpret_cast<T*>(is_k ? p.csa_k : p.csa_v) + head * (is_k ? p.sck[1] : p.scv[1]) + col;
    const int64_t so0 = is_k ? p.sck[0] : p.scv[0];
    float hacc[4] = {0.f, 0.f, 0.f, 0.f};
    bool done = false, released_stage = false;
    if constexpr (M > 0 && NB > 0 && NB % kConsumers == 0) {
      constexpr int BPW = NB / kConsumers;  // blocks per warp
      constexpr int R = (BPW + 1) * M;      // rows per warp, the next warp's first block included
      if (ch.avail >= (b1 + 1) * M) {
        // rows in two register batches (blocks [0, H1] then [H1 + 1, BPW]) to
        // keep the warp under the register budget of three consumer groups
        constexpr int H1 = BPW / 2;
        const uint8_t* rowp = data + static_cast<size_t>(b0 * M) * (kCols * 2);
        float prev[4] = {0.f, 0.f, 0.f, 0.f};
        uint2 x[(H1 + 1) * M > R - (H1 + 1) * M ? (H1 + 1) * M : R - (H1 + 1) * M];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int bb0 = half == 0 ? 0 : H1 + 1, bb1 = half == 0 ? H1 : BPW;
#pragma unroll
          for (int j = 0; j < (bb1 - bb0 + 1) * M; ++j)
            x[j] = *reinterpret_cast<const uint2*>(rowp + (bb0 * M + j) * (kCols * 2));
          if (half == 1) {
            // the rows are in registers: hand the stage back to the producer
            asm volatile("" ::"r"(x[0].x), "r"(x[(bb1 - bb0 + 1) * M - 1].y));
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
            released_stage = true;
          }
#pragma unroll
          for (int b = bb0; b <= bb1; ++b) {
            const int xo = (b - bb0) * M;
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            if constexpr (M % 4 == 0) {
#pragma unroll
              for (int k4 = 0; k4 < M; k4 += 4) {
                const float4 w4 = *reinterpret_cast<const float4*>(W + (b0 + b) * M + k4);
                fc_accum<T>(acc, x[xo + k4 + 0], w4.x);
                fc_accum<T>(acc, x[xo + k4 + 1], w4.y);
                fc_accum<T>(acc, x[xo + k4 + 2], w4.z);
                fc_accum<T>(acc, x[xo + k4 + 3], w4.w);
              }
            } else {
#pragma unroll
              for (int k = 0; k < M; ++k) fc_accum<T>(acc, x[xo + k], W[(b0 + b) * M + k]);
            }
            if (b > 0 && b0 + b - 1 < ch.nslots) {
              const float2 f = AB[b0 + b - 1];
              float o[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) o[q] = prev[q] * f.x + acc[q] * f.y;
              fc_store4(csa_out + (ch.slot0 + b0 + b - 1) * so0, o);
            }
            if (b < BPW) {
              const float h = H[b0 + b];
#pragma unroll
              for (int q = 0; q < 4; ++q) hacc[q] = fmaf(acc[q], h, hacc[q]);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) prev[q] = acc[q];
          }
        }
        done = true;
      }
    }
    if (!done && b0 < b1) {
      float prev[4] = {0.f, 0.f, 0.f, 0.f};
      for (int b = b0; b <= b1; ++b) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const int r0 = b * m, r1 = min(r0 + m, ch.avail);
        for (int r = r0; r < r1; ++r)
          fc_accum<T>(acc, *reinterpret_cast<const uint2*>(data + r * (kCols * 2)), W[r]);
        if (b > b0 && b - 1 < ch.nslots) {
          const float2 f = AB[b - 1];
          float o[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) o[q] = prev[q] * f.x + acc[q] * f.y;
          fc_store4(csa_out + (ch.slot0 + b - 1) * so0, o);
        }
        if (b < b1) {
          const float h = H[b];
#pragma unroll
          for (int q = 0; q < 4; ++q) hacc[q] = fmaf(acc[q], h, hacc[q]);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) prev[q] = acc[q];
      }
    }
    if (!released_stage) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }

    // HCA slot: the group's four partial sums meet in shared memory
    const int hb = grp * 2 + static_cast<int>(ng & 1);
    const int64_t hk = ng >> 1;
    if (hk >= 1 && !mbar_wait_sleep(&hfree[hb], (hk - 1) & 1)) {
      ok = false;
      break;
    }
    float* hp = hpart + hb * (kConsumers * kCols);
    *reinterpret_cast<float4*>(hp + wg * kCols + lane * 4) = make_float4(hacc[0], hacc[1], hacc[2], hacc[3]);
    __threadfence_block();
    __syncwarp();
    if (lane == 0) mbar_arrive(&hfull[hb]);
    if (wg == 0) {
      if (!mbar_wait_sleep(&hfull[hb], hk & 1)) {
        ok = false;
        break;
      }
      float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) {
        const float4 v4 = *reinterpret_cast<const float4*>(hp + w * kCols + lane * 4);
        o[0] += v4.x;
        o[1] += v4.y;
        o[2] += v4.z;
        o[3] += v4.w;
      }
      T* hca_out = reinterpret_cast<T*>(is_k ? p.hca_k : p.hca_v);
      const int64_t* sh = is_k ? p.shk : p.shv;
      fc_store4(hca_out + cur.c * sh[0] + head * sh[1] + col, o);
      __syncwarp();
      if (lane == 0) mbar_arrive(&hfree[hb]);
    }
    new_chunk = false;
    for (int a = 0; a < kGroups; ++a) new_chunk |= fc_cursor_next(cur, p);
  }
  if (!ok) *abort_flag = 1;
}

static bool fc_aligned(const void* ptr, int bytes) { return (reinterpret_cast<uintptr_t>(ptr) % bytes) == 0; }

// The fused kernel handles 16-bit TND inputs with CSA windows of 2m, HCA
// windows of m' = a multiple of m, m' + m <= 256 rows, head dims that are
// multiples of 128, TMA-compatible K/V strides and 8-byte aligned outputs.
// Anything else runs the two single-pass kernels one after the other.
template <typename T>
static int compress_csa_hca_typed(const CompressArgs& csa, const CompressArgs& hca, cudaStream_t st,
                                  bool* handled) {
  using namespace fc;
  *handled = false;
  const int m = csa.stride, mp = hca.stride;
  if (csa.cu_seqlens == nullptr || csa.total_rows <= 0 || csa.total_rows >= (int64_t(1) << 31) || csa.window != 2 * m || hca.window != mp || mp % m != 0 || mp + m > 256)
    return 0;
  const int D = csa.head_dim, Dv = csa.head_dim_v, Hkv = csa.num_kv_heads;
  if (D % kCols != 0 || Dv % kCols != 0) return 0;
  const int64_t* tens[] = {csa.sk, csa.sv};
  for (const int64_t* s : tens) {
    if (s[2] != 1 || s[0] <= 0 || s[0] % 8 != 0) return 0;
    if (Hkv > 1 && (s[1] <= 0 || s[1] % 8 != 0)) return 0;
  }
  if (!fc_aligned(csa.k, 16) || !fc_aligned(csa.v, 16)) return 0;
  const int64_t* outs[] = {csa.sck, csa.scv, hca.sck, hca.scv};
  for (const int64_t* s : outs)
    if (s[2] != 1 || s[0] % 4 != 0 || s[1] % 4 != 0) return 0;
  if (!fc_aligned(csa.ck, 8) || !fc_aligned(csa.cv, 8) || !fc_aligned(hca.ck, 8) || !fc_aligned(hca.cv, 8))
    return 0;

  FusedCompressParams p{};
  p.gate = csa.gate;
  p.sg = csa.sg[0];
  p.cu_seqlens = csa.cu_seqlens;
  p.csa_offsets = csa.comp_offsets;
  p.hca_offsets = hca.comp_offsets;
  p.num_seqs = csa.num_seqs;
  p.heads = Hkv;
  p.k_slices = D / kCols;
  p.slices = (D + Dv) / kCols;
  p.num_units = hca.num_compressed * Hkv * p.slices;
  p.m = m;
  p.mp = mp;
  p.nb = mp / m;
  p.rows = mp + m;
  p.stage_bytes = p.rows * kCols * 2;
  p.rows_pad = (p.rows + 3) & ~3;
  p.entry_floats = (p.rows_pad + 5 * (p.nb + 1) + 3) & ~3;
  p.csa_k = csa.ck;
  p.csa_v = csa.cv;
  p.hca_k = hca.ck;
  p.hca_v = hca.cv;
  for (int i = 0; i < 3; ++i) {
    p.sck[i] = csa.sck[i];
    p.scv[i] = csa.scv[i];
    p.shk[i] = hca.sck[i];
    p.shv[i] = hca.scv[i];
  }
  const int fixed = kRing * p.entry_floats * 4 + kGroups * 2 * kConsumers * kCols * 4 + 8 +
                    8 * (2 * kRing + 4 * kGroups) + 16 + 128;
  const int budget = 220 * 1024;
  p.stages = min(8, (budget - fixed) / p.stage_bytes);
  if (p.stages < 2) return 0;
  const int smem = fixed + 8 * 2 * p.stages + p.stages * p.stage_bytes;

  // K and V as [T, Hkv, D] (3D maps; with one KV head the middle stride is unused)
  CUtensorMap tm[2];
  const void* bases[2] = {csa.k, csa.v};
  const int dims_last[2] = {D, Dv};
  for (int t = 0; t < 2; ++t) {
    const int64_t* s = t == 0 ? csa.sk : csa.sv;
    const uint64_t dims[3] = {static_cast<uint64_t>(dims_last[t]), static_cast<uint64_t>(Hkv),
                              static_cast<uint64_t>(csa.total_rows)};
    const uint64_t strides[2] = {static_cast<uint64_t>(Hkv > 1 ? s[1] * 2 : static_cast<int64_t>(dims_last[t]) * 2),
                                 static_cast<uint64_t>(s[0] * 2)};
    const uint32_t box[3] = {static_cast<uint32_t>(kCols), 1u, static_cast<uint32_t>(p.rows)};
    const uint32_t es[3] = {1, 1, 1};
    const int r = encode_tiled(&tm[t], CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, bases[t], dims, strides, box, es,
                               CU_TENSOR_MAP_SWIZZLE_NONE);
    if (r) return r;
  }
  const int grid = static_cast<int>(p.num_units < num_sms() ? p.num_units : num_sms());
  auto kern = (m == 4 && mp == 128) ? compress_csa_hca_kernel<T, 4, 32> : compress_csa_hca_kernel<T, 0, 0>;
  if (const int r = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem)) return r;
  kern<<<grid, kThreads, smem, st>>>(tm[0], tm[1], p);
  note_kernel("compress_csa_hca");
  *handled = true;
  return 0;
}

int compress_csa_hca_launch(const CompressArgs& csa, const CompressArgs& hca, cudaStream_t st) {
  if (hca.num_compressed == 0 || csa.num_kv_heads == 0) return 0;
  int err = 0;
  if (compress_dual_launch(csa, hca, st, &err)) return err;
  bool handled = false;
  int r = 0;
  if (csa.dtype == kBF16) r = compress_csa_hca_typed<__nv_bfloat16>(csa, hca, st, &handled);
  else if (csa.dtype == kF16) r = compress_csa_hca_typed<__half>(csa, hca, st, &handled);
  if (r || handled) return r;
  r = compress_launch(csa, st);
  return r ? r : compress_launch(hca, st);
}

}  // namespace tak

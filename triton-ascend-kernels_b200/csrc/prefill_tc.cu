// Varlen flash prefill on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Semantics: attention/flash_attention_prefill.py of the reference (kernel
// FP:11-102): per sequence of cu_seqlens and query head h, softmax(scale *
// Q K^T [+ causal mask]) V with KV head h / (H / H_kv), output acc / (l + 1e-6)
// (FP:97), plus the natural-log LSE.
//
// One CTA = up to 256 query rows of one sequence x one query head, as two
// 128-row tiles A and B that share every K/V block (head dims 64 and 128; a
// 256-dim head's O fills 256 TMEM columns, so there a CTA owns one 128-row
// tile and single-stage K/V rings: 64 KB each for Q, K and V).  Row blocks are 256-row
// blocks aligned to global token positions (clipped to the sequence owning the
// block's first row) plus one "head piece" per sequence for its rows before
// the first aligned boundary, so the schedule needs no host-side table (the
// reference builds one with a host loop, FP:144-153).  Causal tiles stop at
// their diagonal block (the reference sweeps every block, FP:60).  Aligned
// blocks are issued last-first (longest work first).
//
// Warp roles (576 threads):
//   warp 16     TMA producer: both Q tiles once, then K and V blocks of 128
//               rows into 2-stage rings (128-byte swizzle, 64-column boxes).
//   warp 17     TMEM allocator + tcgen05.mma issuer (the whole warp runs it,
//               one elected lane issues).  Per K/V block j and tile t:
//               PV_t(j) (TS-MMA: P read from TMEM, V from smem, MN-major),
//               then S_t(j+1) = Q_t K^T (SS-MMA, M=N=128) once PV_t(j) has
//               completed (S_t and P_t share TMEM columns).
//   warps 0-7   softmax of tile A, warps 8-15 softmax of tile B, two threads
//               per row (thread = TMEM lane; warp w and its partner w ^ 4 take
//               score columns [0,64) and [64,128)): load S, mask only on
//               boundary blocks, exchange the halves' row maxima through
//               shared memory (an mbarrier per warp pair), online max with lazy
//               rescaling (O and l rescaled only when the max grows by more
//               than 2^8), P = 2^(s - m) on the MUFU unit, packed to 16 bits
//               into the half's own first 32 S columns; epilogue adds the
//               halves' row sums, normalises and stores each half of the row
//               and its LSE.  Two warps per row on each SM sub-partition keep
//               the exponent pipe busier than one; while one tile's softmax
//               runs the tensor core works on the other tile.
// TMEM: O_A [0,128), O_B [128,256), S/P_A [256,384), S/P_B [384,512); with
// one tile (D = 256), O_A [0,256) and S/P_A [256,384).
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace tak {

struct PrefillTcParams {
  const int32_t* cu_seqlens;
  int num_seqs, total_tokens, H, Hkv, G, n_aligned, causal;
  void* out;
  int64_t so_t, so_h;
  float* lse;
  float scale_log2;
};

namespace pf {
constexpr int BM = 128, BN = 128;
constexpr int TILE = 128 * 128;                   // one 64-column block of 128 rows (bytes)
constexpr int NBAR = 25;
constexpr float kRescaleThreshold = 8.f;          // log2 units
// Shared-memory layout and tiling of head dim D: NT query tiles of 128 rows
// per CTA, NST-stage K and V rings, NB 64-column boxes per row.
template <int D>
struct Cfg {
  static constexpr int NB = D / 64;
  static constexpr int NT = D >= 256 ? 1 : 2;
  static constexpr int NST = D >= 256 ? 1 : 2;
  static constexpr int ROWS = NT * BM;
  static constexpr int QOFF = 0;
  static constexpr int KOFF = NT * NB * TILE;
  static constexpr int VOFF = KOFF + NST * NB * TILE;
  static constexpr int BAROFF = VOFF + NST * NB * TILE;
  // softmax partner exchange: row maxima [block parity][tile][half][row] and
  // row sums [tile][half][row]
  static constexpr int XOFF = BAROFF + NBAR * 8 + 16 + 8;
  static constexpr int SMEM = XOFF + (2 * 2 * 2 * 128 + 2 * 2 * 128) * 4 + 1024;
  static_assert(SMEM <= 232448, "shared memory");
};
constexpr int NWARP = 18;  // 16 softmax warps, producer, MMA issuer
}  // namespace pf

__device__ __forceinline__ int pf_find_seq(const int32_t* cu, int n, int t) {
  int lo = 0, hi = n - 1, ans = -1;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    if (cu[mid] <= t) {
      ans = mid;
      lo = mid + 1;
    } else {
      hi = mid - 1;
    }
  }
  return ans;
}

template <typename T, int D>
__global__ void __launch_bounds__(pf::NWARP * 32, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const PrefillTcParams p) {
  using namespace pf;
  using C = Cfg<D>;
  constexpr int NB = C::NB, NST = C::NST, ROWS = C::ROWS;
  constexpr int QOFF = C::QOFF, KOFF = C::KOFF, VOFF = C::VOFF;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAROFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2] per tile
  uint64_t* p_full = bars + 11;  // [2] per tile
  uint64_t* o_done = bars + 13;  // [2] per tile
  uint64_t* pair_mb = bars + 15; // [2][4] per tile and lane quadrant: the two softmax warps' exchange
  uint64_t* p_half = bars + 23;  // [2] per tile: the first 32-key chunk of each half of P stored
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  // blockIdx.x = slot * H + h: the heads of one row block are adjacent (they
  // share K/V through L2) and the grid has no 65535 limit on row blocks
  const int h = static_cast<int>(blockIdx.x % static_cast<unsigned>(p.H));
  const int slot = static_cast<int>(blockIdx.x / static_cast<unsigned>(p.H));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = p.num_seqs;
  const int cu_end = p.cu_seqlens[S];

  // ---------------- which rows does this CTA own (CTA-uniform) ----------------
  int s, row0, row1;
  if (slot < p.n_aligned) {
    row0 = (p.n_aligned - 1 - slot) * ROWS;
    if (row0 >= cu_end) return;
    s = pf_find_seq(p.cu_seqlens, S, row0);
    row1 = min(row0 + ROWS, static_cast<int>(p.cu_seqlens[s + 1]));
  } else if (slot < p.n_aligned + S) {
    s = slot - p.n_aligned;
    const int st = p.cu_seqlens[s], en = p.cu_seqlens[s + 1];
    if (st % ROWS == 0 || st >= en) return;
    row0 = st;
    row1 = min((st / ROWS + 1) * ROWS, en);
  } else {
    // rows past the last sequence: zeros (FP:189)
    for (int t = cu_end + warp; t < p.total_tokens; t += NWARP) {
      T* o = reinterpret_cast<T*>(p.out) + static_cast<int64_t>(t) * p.so_t + static_cast<int64_t>(h) * p.so_h;
      for (int d = lane; d < D; d += 32) o[d] = Elem<T>::from_f(0.f);
      if (lane == 0 && p.lse) p.lse[static_cast<int64_t>(t) * p.H + h] = -INFINITY;
    }
    return;
  }
  const int seq_start = p.cu_seqlens[s];
  const int seq_len = p.cu_seqlens[s + 1] - seq_start;
  const int rows_t[2] = {min(BM, row1 - row0), max(0, row1 - row0 - BM)};
  const int p0_t[2] = {row0 - seq_start, row0 - seq_start + BM};
  int n_t[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int keys = rows_t[t] <= 0 ? 0 : (p.causal ? min(seq_len, p0_t[t] + rows_t[t]) : seq_len);
    n_t[t] = (keys + BN - 1) / BN;
  }
  const int n_kv = max(n_t[0], n_t[1]);
  const int kvh = h / p.G;

  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 8; ++i) mbar_init(&pair_mb[i], 64);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 256);
      mbar_init(&p_half[i], 256);
      mbar_init(&o_done[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 17) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = *tmem_holder;
  const uint32_t sbase = smem_u32(smem);

  if (warp == 16) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const int nq = rows_t[1] > 0 ? 2 : 1;
      mbar_arrive_expect_tx(q_full, nq * NB * TILE);
      for (int t = 0; t < nq; ++t)
        for (int b = 0; b < NB; ++b)
          tma_load_3d(smem + QOFF + (t * NB + b) * TILE, &tmQ, q_full, b * 64, h, row0 + t * BM);
      for (int j = 0; j < n_kv && !*abort_flag; ++j) {
        const int st = j % NST;
        const int key0 = seq_start + j * BN;
        if (j >= NST && !mbar_wait_sleep(&k_empty[st], ((j / NST) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], NB * TILE);
        for (int b = 0; b < NB; ++b)
          tma_load_3d(smem + KOFF + (st * NB + b) * TILE, &tmK, &k_full[st], b * 64, kvh, key0);
        if (j >= NST && !mbar_wait_sleep(&v_empty[st], ((j / NST) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&v_full[st], NB * TILE);
        for (int b = 0; b < NB; ++b)
          tma_load_3d(smem + VOFF + (st * NB + b) * TILE, &tmV, &v_full[st], b * 64, kvh, key0);
      }
    }
  } else if (warp == 17) {
    // ---------------- MMA issuer ----------------
    // The whole warp runs the issuer (one elected lane issues each MMA and
    // commit); its waits suspend in hardware and are made warp-uniform, so the
    // warp stays converged and takes no issue slots from the softmax warps
    // sharing its SM sub-partition.
    {
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait_sleep(bar, parity));
      };
      constexpr int AB = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      const uint32_t idesc_qk = tc_idesc_f16(AB, BM, BN, 0);
      const uint32_t idesc_pv = tc_idesc_f16(AB, BM, D, 1);
      // Shared-memory descriptors are built once; a k-step adds its byte offset
      // >> 4 to the 14-bit address field (shared addresses stay below 256 KB, so
      // the field never carries).  Rebuilding both descriptors for every MMA
      // made the single issuing thread, not the tensor core, the bottleneck.
      const uint64_t q_desc0 = tc_sdesc_sw128(sbase + QOFF, 16, 1024);
      const uint64_t k_desc0 = tc_sdesc_sw128(sbase + KOFF, 16, 1024);
      const uint64_t v_desc0 = tc_sdesc_sw128(sbase + VOFF, TILE, 1024);
      constexpr uint64_t kTileStep = (NB * TILE) >> 4;  // next Q tile / next K or V stage
      auto qk = [&](int t, int j) {
        const uint64_t qd = q_desc0 + (t ? kTileStep : 0), kd = k_desc0 + ((j % NST) ? kTileStep : 0);
        const uint32_t d_tmem = taddr + 256 + t * 128;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t koff = static_cast<uint64_t>(((kk >> 2) * TILE + (kk & 3) * 32) >> 4);
          tc_mma_ss_w(d_tmem, qd + koff, kd + koff, idesc_qk, kk > 0 ? 1u : 0u);
        }
        tc_commit_w(&s_full[t]);
      };
      // P.V in two parts: part 0 takes the K16 steps of P's first 32-key
      // chunk in each column half (keys 0-31 and 64-95, steps 0, 1, 4, 5),
      // issued as soon as the softmax has stored that chunk, so it runs while
      // the softmax computes the second chunk; part 1 the rest, then the commit
      auto pv = [&](int t, int j, int part) {
        const uint64_t vd = v_desc0 + ((j % NST) ? kTileStep : 0);
        const uint32_t p_tmem = taddr + 256 + t * 128;
#pragma unroll
        for (int i = 0; i < BN / 32; ++i) {
          const int kk = (i >> 1) * 4 + part * 2 + (i & 1);
          tc_mma_ts_w(taddr + t * 128, p_tmem + (kk >> 2) * 64 + (kk & 3) * 8,
                      vd + static_cast<uint64_t>((kk * 2048) >> 4), idesc_pv,
                      (j > 0 || part > 0 || i > 0) ? 1u : 0u);
        }
        if (part == 1) tc_commit_w(&o_done[t]);
      };
      bool ok = n_kv > 0 && wait(q_full, 0) && wait(&k_full[0], 0);
      if (ok) {
        tc_fence_after();
        if (n_t[0] > 0) qk(0, 0);
        if (n_t[1] > 0) qk(1, 0);
        tc_commit_w(&k_empty[0]);
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        if (__any_sync(0xffffffffu, *abort_flag != 0)) {
          ok = false;
          break;
        }
        // Per tile: P.V of block j, then (once that P.V has read P) S of block
        // j + 1, so a tile's next softmax can start while the other tile's
        // softmax is still running.
        const int st = j % NST;
        if (!(ok = wait(&v_full[st], (j / NST) & 1))) break;
        const bool next = j + 1 < n_kv;
        bool k_next = false;  // K block j + 1 waited for
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (j < n_t[t]) {
            if (!(ok = wait(&p_half[t], j & 1))) break;
            tc_fence_after();
            pv(t, j, 0);
            if (!(ok = wait(&p_full[t], j & 1))) break;
            tc_fence_after();
            pv(t, j, 1);
            if (t == 1 || j >= n_t[1]) tc_commit_w(&v_empty[st]);
            if (j + 1 < n_t[t]) {
              if (!k_next && !(ok = wait(&k_full[(j + 1) % NST], ((j + 1) / NST) & 1))) break;
              k_next = true;
              // this tile's S/P columns are rewritten only after its PV of block j has read P
              if (!(ok = wait(&o_done[t], j & 1))) break;
              tc_fence_after();
              qk(t, j + 1);
            }
          }
        }
        if (!ok) break;
        if (next) {
          // every tile with block j + 1 has issued its S MMA; the commit frees the K stage
          // (a tile without block j + 1 issues none, and then k_full of block j + 1 may
          // not have been waited for: wait here so the stage's phases stay in step)
          if (!k_next && !(ok = wait(&k_full[(j + 1) % NST], ((j + 1) / NST) & 1))) break;
          tc_commit_w(&k_empty[(j + 1) % NST]);
        }
      }
      if (!ok && n_kv > 0) *abort_flag = 1;
    }
  } else if (warp < 16) {
    // ---------------- softmax + epilogue: warps 0-7 tile A, warps 8-15 tile B ----------------
    // Two threads per row: warp w covers TMEM lane quadrant w % 4 and score
    // columns [64 hf, 64 hf + 64) of its tile, hf = (w / 4) % 2; its partner
    // warp w ^ 4 covers the other half of the same rows.
    const int t = warp >> 3;
    const int hf = (warp >> 2) & 1;
    const int qd = warp & 3;
    const int r = qd * 32 + lane;
    const int nt = n_t[t];
    const bool row_ok = r < rows_t[t];
    const int lim = !row_ok ? 0 : (p.causal ? min(seq_len, p0_t[t] + r + 1) : seq_len);
    // blocks below this bound need no mask for any row of the tile
    const int lim_all = p.causal ? min(seq_len, p0_t[t] + 1) : seq_len;
    const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t s_tmem = taddr + lane_off + 256 + t * 128;
    const uint32_t o_tmem = taddr + lane_off + t * 128 + hf * (D / 2);  // this thread's half of O's columns
    float* const xmax = reinterpret_cast<float*>(smem + C::XOFF);       // [2][2][2][128]
    float* const xl = xmax + 2 * 2 * 2 * 128;                           // [2][2][128]
    uint64_t* const xbar = &pair_mb[t * 4 + qd];  // phase j: block j's maxima; phase nt: the row sums
    float m_run = -INFINITY, m_used = -INFINITY, l = 0.f;
    bool ok = true;
    const float sl2 = p.scale_log2;
    const uint64_t sl2x2 = (static_cast<uint64_t>(__float_as_uint(sl2)) << 32) | __float_as_uint(sl2);
    for (int j = 0; j < nt; ++j) {
      if (!(ok = mbar_wait_sleep(&s_full[t], j & 1))) break;
      tc_fence_after();
      const bool interior = (j + 1) * BN <= lim_all;
      const int nvalid = lim - j * BN - hf * 64;  // valid columns of this half
      // pass 1: this half's row max over its 64 scores
      float mx = -INFINITY;
      {
        uint32_t sr[64];
        tmem_ld32(s_tmem + hf * 64, sr);
        tmem_ld32(s_tmem + hf * 64 + 32, sr + 32);
        tmem_ld_wait();
        if (interior) {
          // four independent chains of three-input maxima (two scores each)
          float m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
          for (int c = 0; c < 64; c += 8) {
            mx = fmax3(mx, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
            m1 = fmax3(m1, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
            m2 = fmax3(m2, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
            m3 = fmax3(m3, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
          }
          mx = fmax3(mx, m1, fmaxf(m2, m3));
        } else {
#pragma unroll
          for (int c = 0; c < 64; ++c) mx = fmaxf(mx, c < nvalid ? __uint_as_float(sr[c]) : -INFINITY);
        }
      }
      // the row max over both halves (exchange buffers alternate by block, so
      // a write of block j + 2 follows the partner's read of block j)
      float* xm = xmax + ((j & 1) * 4 + t * 2) * 128;
      xm[hf * 128 + r] = mx;
      mbar_arrive(xbar);
      if (!(ok = mbar_wait(xbar, j & 1))) break;
      mx = fmaxf(mx, xm[(hf ^ 1) * 128 + r]);
      const float m_new = fmaxf(m_run, mx * sl2);
      const bool need = m_new != -INFINITY && m_new > m_used + kRescaleThreshold;
      const bool rescale_o = need && m_used != -INFINITY;
      if (__any_sync(0xffffffffu, rescale_o)) {
        if (!(ok = mbar_wait(&o_done[t], (j - 1) & 1))) break;
        tc_fence_after();
        const float f = rescale_o ? fast_exp2(m_used - m_new) : 1.f;
        uint32_t orow[32];
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tmem_ld32(o_tmem + c * 32, orow);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) orow[i] = __float_as_uint(__uint_as_float(orow[i]) * f);
          tmem_st32(o_tmem + c * 32, orow);
        }
        tmem_st_wait();
        l *= f;
      }
      if (need) m_used = m_new;
      m_run = m_new;
      const float mu = m_used == -INFINITY ? 0.f : m_used;
      // pass 2: P = 2^(s*scale - m) of this half's 64 keys, 32 at a time,
      // packed into this half's own first 32 S columns (key pair c of the half
      // in column 64 hf + c; chunk c4 lands on columns already read)
      float ls0 = 0.f, ls1 = 0.f;
      uint64_t lsx2 = 0;  // packed row-sum pair of the interior path (two +0.0f)
      const uint64_t nmux2 = (static_cast<uint64_t>(__float_as_uint(-mu)) << 32) | __float_as_uint(-mu);
#pragma unroll
      for (int c4 = 0; c4 < 2; ++c4) {
        uint32_t sr[32], pk[16];
        tmem_ld32(s_tmem + hf * 64 + c4 * 32, sr);
        tmem_ld_wait();
        if (interior) {
          // two scores per packed fp32 FMA and per packed row-sum add (same
          // rounding as the scalar forms)
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            uint64_t x = (static_cast<uint64_t>(sr[2 * c + 1]) << 32) | sr[2 * c];
            asm("fma.rn.f32x2 %0, %0, %1, %2;" : "+l"(x) : "l"(sl2x2), "l"(nmux2));
            const float a = fast_exp2(__uint_as_float(static_cast<uint32_t>(x)));
            const float bb = fast_exp2(__uint_as_float(static_cast<uint32_t>(x >> 32)));
            const uint64_t ab = (static_cast<uint64_t>(__float_as_uint(bb)) << 32) | __float_as_uint(a);
            asm("add.rn.f32x2 %0, %0, %1;" : "+l"(lsx2) : "l"(ab));
            pk[c] = Elem<T>::pack2(a, bb);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const int e = 32 * c4 + 2 * c;
            const float a = (e < nvalid) ? fast_exp2(fmaf(__uint_as_float(sr[2 * c]), sl2, -mu)) : 0.f;
            const float bb = (e + 1 < nvalid) ? fast_exp2(fmaf(__uint_as_float(sr[2 * c + 1]), sl2, -mu)) : 0.f;
            ls0 += a;
            ls1 += bb;
            pk[c] = Elem<T>::pack2(a, bb);
          }
        }
        tmem_st16(s_tmem + hf * 64 + 16 * c4, pk);
        if (c4 == 0) {
          // the first chunk of P: the issuer starts P.V on it
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(&p_half[t]);
        }
      }
      ls0 += __uint_as_float(static_cast<uint32_t>(lsx2));
      ls1 += __uint_as_float(static_cast<uint32_t>(lsx2 >> 32));
      l += ls0 + ls1;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }
    if (ok && nt > 0) ok = mbar_wait(&o_done[t], (nt - 1) & 1);
    if (!ok) *abort_flag = 1;
    if (nt > 0) {
      // the row sum over both halves
      xl[(t * 2 + hf) * 128 + r] = l;
      mbar_arrive(xbar);
      if (ok) ok = mbar_wait(xbar, nt & 1);
      const float l_tot = l + xl[(t * 2 + (hf ^ 1)) * 128 + r];
      tc_fence_after();
      const float f = (m_used == -INFINITY) ? 0.f : fast_exp2(m_used - m_run);
      const float inv = (l_tot > 0.f && ok) ? f / (l_tot * f + 1e-6f) : 0.f;
      T* orow = reinterpret_cast<T*>(p.out) + static_cast<int64_t>(row0 + t * BM + r) * p.so_t +
                static_cast<int64_t>(h) * p.so_h + hf * (D / 2);
      // this thread's D / 2 columns of O, up to 64 per TMEM round trip
      constexpr int HD = D / 2;
      constexpr int CW = HD < 64 ? HD : 64;
#pragma unroll
      for (int c0 = 0; c0 < HD; c0 += CW) {
        float o[CW];
#pragma unroll
        for (int c = 0; c < CW / 32; ++c)
          tmem_ld32(o_tmem + c0 + c * 32, reinterpret_cast<uint32_t*>(o) + c * 32);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int c = 0; c < CW / 8; ++c) {
            uint4 u;
            u.x = Elem<T>::pack2(o[8 * c + 0] * inv, o[8 * c + 1] * inv);
            u.y = Elem<T>::pack2(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
            u.z = Elem<T>::pack2(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
            u.w = Elem<T>::pack2(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
            *reinterpret_cast<uint4*>(orow + c0 + 8 * c) = u;
          }
        }
      }
      if (row_ok && hf == 0) {
        if (p.lse)
          p.lse[static_cast<int64_t>(row0 + t * BM + r) * p.H + h] =
              (l_tot > 0.f && ok) ? (m_used + __log2f(l_tot)) * kLn2 : -INFINITY;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 17) {
    tc_fence_after();
    tmem_dealloc(taddr, 512);
  }
}

static int encode_tnd_map(CUtensorMap* m, const void* base, const int64_t* st, int64_t T, int64_t heads, int d) {
  const uint64_t dims[3] = {static_cast<uint64_t>(d), static_cast<uint64_t>(heads), static_cast<uint64_t>(T)};
  const uint64_t strides[2] = {static_cast<uint64_t>(st[1] * 2), static_cast<uint64_t>(st[0] * 2)};
  const uint32_t box[3] = {64, 1, 128};
  const uint32_t es[3] = {1, 1, 1};
  return encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, base, dims, strides, box, es, CU_TENSOR_MAP_SWIZZLE_128B);
}

static bool tma_ok(const void* ptr, const int64_t* st) {
  if (reinterpret_cast<uintptr_t>(ptr) & 15) return false;
  if (st[2] != 1) return false;
  return st[0] > 0 && st[1] > 0 && (st[0] * 2) % 16 == 0 && (st[1] * 2) % 16 == 0;
}

template <typename T, int D>
static int launch_prefill_tc(const PrefillArgs& a, cudaStream_t st) {
  using C = pf::Cfg<D>;
  const int64_t n_aligned = (static_cast<int64_t>(a.total_tokens) + C::ROWS - 1) / C::ROWS;
  CUtensorMap mq, mk, mv;
  if (int r = encode_tnd_map(&mq, a.q, a.sq, a.total_tokens, a.num_q_heads, D)) return r;
  if (int r = encode_tnd_map(&mk, a.k, a.sk, a.total_tokens, a.num_kv_heads, D)) return r;
  if (int r = encode_tnd_map(&mv, a.v, a.sv, a.total_tokens, a.num_kv_heads, D)) return r;
  PrefillTcParams p{};
  p.cu_seqlens = a.cu_seqlens;
  p.num_seqs = a.num_seqs;
  p.total_tokens = a.total_tokens;
  p.H = a.num_q_heads;
  p.Hkv = a.num_kv_heads;
  p.G = a.num_q_heads / a.num_kv_heads;
  p.n_aligned = static_cast<int>(n_aligned);
  p.causal = a.causal;
  p.out = a.out;
  p.so_t = a.so[0];
  p.so_h = a.so[1];
  p.lse = a.lse;
  p.scale_log2 = a.scale * kLog2e;
  // one CTA per (row block, query head); the last row-block slot per head zeroes
  // the rows past the last sequence
  const dim3 grid(static_cast<unsigned>((n_aligned + a.num_seqs + 1) * a.num_q_heads));
  auto kern = prefill_tc_kernel<T, D>;
  if (const int r = ensure_smem_attr(reinterpret_cast<const void*>(kern), C::SMEM)) return r;
  kern<<<grid, pf::NWARP * 32, C::SMEM, st>>>(mq, mk, mv, p);
  note_kernel("prefill_tc");
  return 0;
}

int prefill_tc_launch(const PrefillArgs& a, cudaStream_t st, bool* handled) {
  *handled = false;
  if (a.dtype == kF32 || a.head_dim != a.head_dim_v) return 0;
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return 0;
  if (!tma_ok(a.q, a.sq) || !tma_ok(a.k, a.sk) || !tma_ok(a.v, a.sv)) return 0;
  if (a.so[2] != 1 || (a.so[0] % 8) || (a.so[1] % 8) || (reinterpret_cast<uintptr_t>(a.out) & 15)) return 0;
  // the grid's one dimension holds (row blocks + sequences + 1) x heads CTAs
  const int rows = a.head_dim >= 256 ? pf::BM : 2 * pf::BM;
  const int64_t ctas = ((static_cast<int64_t>(a.total_tokens) + rows - 1) / rows + a.num_seqs + 1) * a.num_q_heads;
  if (ctas > 2147483647) return 0;
  int r;
  const bool bf = a.dtype == kBF16;
  switch (a.head_dim) {
    case 64: r = bf ? launch_prefill_tc<__nv_bfloat16, 64>(a, st) : launch_prefill_tc<__half, 64>(a, st); break;
    case 128: r = bf ? launch_prefill_tc<__nv_bfloat16, 128>(a, st) : launch_prefill_tc<__half, 128>(a, st); break;
    default: r = bf ? launch_prefill_tc<__nv_bfloat16, 256>(a, st) : launch_prefill_tc<__half, 256>(a, st); break;
  }
  *handled = true;
  return r;
}

}  // namespace tak

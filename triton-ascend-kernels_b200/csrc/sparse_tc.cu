// Top-k sparse attention (prefill and decode forms) on the 5th-generation
// tensor cores.
//
// Semantics: attention/sparse_attn_fwd.py of the reference (kernel SA:10-98):
// token t, query head h attends to rows topk_idxs[t, :] of K/V (negative =
// masked; past the last row = masked here), softmax with an optional per-head
// sink logit that enters only the denominator (SA:86-92), l = 0 -> output 0
// (SA:94-95); plus the natural-log LSE.  Also covers the MLA-style latent
// layout the reference cannot express (Dqk = 576 = 512 latent + 64 rope,
// Dv = 512, V a view of K's first 512 columns).
//
// Decode form (kernel SA:105-246): one query token per request; slot c of the
// request's index row is a window slot for c < num_win (index = logical
// position, valid when 0 <= idx < ctx, read from the paged cache through the
// block table) and a compressed slot otherwise (valid when idx >= ctx, row
// idx - ctx of the compressed K/V).  Only the producer's row addressing and the
// validity mask differ from the prefill form.
//
// A unit = one query token x one group of up to 64 query heads sharing a KV
// head (MQA: all 64 heads of the token).  The 64 head rows are the MMA's
// M = 64 dimension, so every gathered K/V row is read once for all heads.
// Prefill runs one persistent CTA per SM, each taking units blockIdx.x,
// blockIdx.x + gridDim.x, ...; the pipelines (gathers, MMAs, softmax) run on
// across a unit boundary, so the next unit's Q and first rows load while the
// current unit finishes.  Decode runs one unit per CTA.
//
// Tensor memory (M = 64 uses half of each 32-lane quadrant):
//   lanes 0-15 of each quadrant: S (two 64-column buffers, columns 0-127) and
//            Q as the QK MMA's A operand (columns 128 .. 128 + Dqk/2; the A
//            operand and the accumulator of one MMA sit on the same lanes),
//            plus O's columns past 512 for a 576-dim V;
//   lanes 16-31: O (up to 512 fp32 columns).
// Keeping Q out of shared memory leaves room for three gather stages of the
// 576-dim latent rows (3 x 72 KB), so the gathers of two tiles are in flight
// while the tensor core works on a third.
//
// Warp roles (288 threads):
//   warps 4-7 gather producers: per unit its Q rows (one TMA into a K ring
//            stage), then for each tile of 64 indices, cp.async 16-byte copies
//            of the gathered rows (8 lanes per 128-byte line, so every warp
//            instruction moves 4 full lines) written straight into the
//            128-byte-swizzled layout the MMA reads; K and V have rings of
//            their own unless V is a prefix view of K (then the K rows serve
//            both); masked rows are zero-filled; a tile's raw indices are
//            loaded two tiles ahead and its row addresses formed one ahead.
//   warp 8   TMEM allocator + tcgen05.mma issuer (one elected lane):
//            S_j = Q K_j^T (M=64, N=64, K=16 x Dqk/16, A from TMEM), O += P_j
//            V_j (M=64, N<=256 per instruction, P from shared memory).  Issue
//            order is greedy: whichever of "QK of the next loaded tile" and
//            "PV of the next softmaxed tile" is ready goes first, the barriers
//            tested without waiting (mbarrier.test_wait), so QK(j+1) runs on
//            the tensor core while the softmax of tile j runs.
//   warps 0-3 move each unit's Q from shared memory into TMEM (once the
//            previous unit's last S is read), then run the softmax:
//            TMEM loads of shape 16x32bx2 let all 32 threads of a warp work
//            on its 16 head rows (two threads per row, 32 columns each); lazy
//            rescaling of O (only when the max grows by > 2^8); P written to
//            shared memory (K-major, swizzled) for the PV MMA; epilogue folds
//            the sink, normalises and stores the rows.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace tak {

struct SparseTcParams {
  const int32_t* topk;
  int64_t stk0, stk1;
  int k_topk;
  int64_t kv_rows;
  const float* sink;
  void* out;
  int64_t so_t, so_h;
  float* lse;
  int H, Hkv, G, head_chunks;
  float scale_log2;
  // Row sources, in elements.  Prefill: row r < rows1 of head h is k + r*k_s0 +
  // h*k_sh, row r >= rows1 is ck + (r - rows1)*ck_s0 + h*ck_sh.  Decode: k/v are
  // the paged caches (page stride k_s0, head k_sh, row in page k_sr) and ck/cv
  // the compressed rows (row stride ck_s0, head ck_sh).
  int64_t rows1;
  const void* k;
  const void* v;
  const void* ck;
  const void* cv;
  int64_t k_s0, k_sh, k_sr, v_s0, v_sh, v_sr;
  int64_t ck_s0, ck_sh, cv_s0, cv_sh;
  const int32_t* bt;
  int64_t sbt0, sbt1;
  const int32_t* ctx_lens;
  int64_t ncomp;
  int num_win, block_size;
  int64_t wreach;      // block-table width x block_size: window positions at or past it are masked
  int64_t num_blocks;  // pages of the cache: a window position on a page id outside [0, num_blocks) is masked
  // work units: unit u = (token u / Y, KV head x head chunk u % Y); a CTA
  // takes units blockIdx.x, blockIdx.x + gridDim.x, ...
  int64_t n_units;
  int Y;
};

// Validity of slot c holding index j (decode: by slot position, SA:151-171 for
// the window slots [0, num_win) and SA:197-210 for the compressed ones).  A
// window slot must also lie inside its block-table row and name a page of the
// cache (the reference reads past both unchecked); bt_row is the request's
// block-table row.
template <bool DECODE>
__device__ __forceinline__ bool sp_slot_valid(const SparseTcParams& p, int c, int64_t j, int ctx,
                                              const int32_t* bt_row) {
  if (!DECODE) return j >= 0 && j < p.kv_rows;
  if (c >= p.num_win) return j >= ctx && j - ctx < p.ncomp;
  if (j < 0 || j >= ctx || j >= p.wreach) return false;
  const int64_t page = bt_row[(j / p.block_size) * p.sbt1];
  return page >= 0 && page < p.num_blocks;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// 16 TMEM lanes x 32 columns per half-warp: threads 0-15 read columns
// [c, c+32) of lanes base+t, threads 16-31 columns [c+32, c+64) of lanes base+t-16.
__device__ __forceinline__ void tmem_ld16x2(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32], 32;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16x2(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x32bx2.x32.b32 [%0], 32, {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 16 lanes x 16 columns per half-warp (the x16 form of tmem_st16x2): threads
// 0-15 write columns [c, c+16) of lanes base+t, threads 16-31 columns
// [c+16, c+32) of lanes base+t-16.
__device__ __forceinline__ void tmem_st16x2_x16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x32bx2.x16.b32 [%0], 16, {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Shared-memory plan of one head-dim variant.  K stages hold DQK columns of
// 64 gathered rows; V stages (only when V is not a prefix view of K) DV
// columns.  Each unit's Q (64 x DQK) passes through the K ring as one item
// before it moves to TMEM.  Stage counts are the most that fit next to P (at
// most 4; at least 2 K stages for every variant, so a unit's Q and its first
// tile are in flight together).
template <int DQK, int DV, bool SHARED>
struct SpLayout {
  static constexpr int BLK = 64 * 128;  // 64 rows x 128 B: one 64-column block of a 64-row tile
  static constexpr int NQB = DQK / 64, NVB = DV / 64;
  static constexpr int KST = NQB * BLK;
  static constexpr int VST = SHARED ? 0 : NVB * BLK;
  static constexpr int BUDGET = 232448 - 1024 - BLK - 512;  // opt-in maximum - alignment - P - barriers
  static constexpr int NPAIR = BUDGET / (KST + VST) < 4 ? BUDGET / (KST + VST) : 4;
  static constexpr int NSK = SHARED ? (BUDGET / KST < 4 ? BUDGET / KST : 4)
                                    : (NPAIR >= 2 ? NPAIR : (2 * KST + VST <= BUDGET ? 2 : 1));
  static constexpr int NSV = SHARED ? 0 : (NPAIR >= 2 ? NPAIR : 1);
  static constexpr int KOFF = 0;
  static constexpr int VOFF = KOFF + NSK * KST;
  static constexpr int POFF = VOFF + NSV * VST;
  static constexpr int BAROFF = POFF + BLK;
  static constexpr int NBAR = 24;
  static constexpr int SMEM = BAROFF + NBAR * 8 + 16 + 1024;
  // TMEM columns: S [0, 128) and Q [128, 128 + DQK/2) on lanes 0-15, then O's
  // columns past 512 (576-dim V); O [0, min(DV, 512)) on lanes 16-31
  static constexpr int QCOL = 128;
  static constexpr int OMAIN = DV < 512 ? DV : 512;
  static constexpr int OTAIL = DV - OMAIN;
  static constexpr int TCOL = QCOL + DQK / 2;
  static_assert(TCOL + OTAIL <= 512, "TMEM columns");
  static constexpr int TMEM_NEED = (TCOL + OTAIL) > OMAIN ? (TCOL + OTAIL) : OMAIN;
  static constexpr int TMEM_COLS = TMEM_NEED <= 256 ? 256 : 512;  // a power of two
  static_assert(SMEM <= 232448, "shared memory");
  static_assert(NSK >= 2 && (SHARED || NSV >= 1), "stages: a unit's Q item and a tile share the K ring");
  static_assert(OTAIL == 0 || OTAIL == 64, "a V wider than 512 columns has one 64-column tail");
};

template <typename T, int DQK, int DV, bool SHARED, bool DECODE>
__global__ void __launch_bounds__(288, 1)
    sparse_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const SparseTcParams p) {
  using L = SpLayout<DQK, DV, SHARED>;
  constexpr int BN = 64;
  constexpr int NPROD = 128;  // producer threads
  constexpr int NSK = L::NSK, NSV = L::NSV;
  constexpr int NSVd = SHARED ? 1 : NSV;  // V ring size as a divisor (unused when V is K's rows)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAROFF);
  uint64_t* o_free = bars + 0;   // per unit: its epilogue has read O (128 arrivals)
  uint64_t* q_tmem = bars + 1;   // per unit: its Q is in TMEM (128 arrivals)
  uint64_t* k_full = bars + 2;   // [4] K ring items: a unit's Q, then its tiles' K rows
  uint64_t* k_empty = bars + 6;  // [4]
  uint64_t* v_full = bars + 10;  // [4]
  uint64_t* v_empty = bars + 14; // [4]
  uint64_t* s_full = bars + 18;  // [2]
  uint64_t* p_full = bars + 20;
  uint64_t* p_free = bars + 21;
  uint64_t* o_done = bars + 22;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + L::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  // This CTA's units: blockIdx.x + i * gridDim.x for i < n_my.  Tiles are
  // counted over all of them (J = i * n_tiles + j), and so are the K ring's
  // items: unit i's Q is item i * (n_tiles + 1), its tile j the items after
  // it.  Every barrier phase follows these global counts.
  const int n_tiles = (p.k_topk + BN - 1) / BN;
  const int64_t u0 = blockIdx.x;
  const int n_my = u0 < p.n_units ? static_cast<int>((p.n_units - 1 - u0) / gridDim.x + 1) : 0;
  auto unit_of = [&](int i) -> int64_t { return u0 + static_cast<int64_t>(i) * gridDim.x; };
  auto q_item = [&](int i) -> int { return i * (n_tiles + 1); };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    mbar_init(o_free, 128);
    mbar_init(q_tmem, 128);
    for (int i = 0; i < NSK; ++i) {
      mbar_init(&k_full[i], NPROD);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < NSV; ++i) {
      mbar_init(&v_full[i], NPROD);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) mbar_init(&s_full[i], 1);
    mbar_init(p_full, 128);
    mbar_init(p_free, 1);
    mbar_init(o_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc(tmem_holder, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = *tmem_holder;
  const uint32_t sbase = smem_u32(smem);

  if (warp >= 4 && warp < 8) {
    // ---------------- gather producers ----------------
    const int pt = tid - 128;                 // 0..127
    const int rsub = pt >> 3, chunk = pt & 7;  // row within a 16-row group, 16-byte chunk within a line
    if (pt == 0) tma_prefetch_desc(&tmQ);
    const T* kb = reinterpret_cast<const T*>(p.k);
    const T* vb = reinterpret_cast<const T*>(p.v);
    // Two-stage index pipeline: the raw indices of this thread's 4 slots of a
    // tile are loaded two tiles ahead (no branch on them, so the loads stay in
    // flight), and turned into row addresses one tile ahead; a branch on an
    // index that has just been loaded would stall the producer for a full
    // memory latency every tile.  Tiles are numbered over all of the CTA's
    // units, so the pipeline runs on across a unit boundary.
    // Two cursors walk the CTA's tiles in order -- one loading raw indices,
    // one forming row addresses -- and redo the per-unit arithmetic (token,
    // KV head, lengths) only when they cross into the next unit.
    struct Cursor {
      int i, j;                 // unit of the CTA, tile within it
      bool in;                  // i < n_my
      const int32_t* ir;        // the unit's index row
      int kvh, ctx;
      const int32_t* bt_row;
    };
    auto open_unit = [&](Cursor& c) {
      c.in = c.i < n_my;
      const int64_t u = c.in ? unit_of(c.i) : 0;
      const int t = static_cast<int>(u / p.Y);
      c.ir = p.topk + static_cast<int64_t>(t) * p.stk0;
      c.kvh = static_cast<int>(u % p.Y) / p.head_chunks;
      c.ctx = (DECODE && c.in) ? p.ctx_lens[t] : 0;
      c.bt_row = DECODE ? p.bt + static_cast<int64_t>(t) * p.sbt0 : nullptr;
    };
    auto advance = [&](Cursor& c) {
      if (++c.j == n_tiles) {
        c.j = 0;
        ++c.i;
        open_unit(c);
      }
    };
    Cursor cl{0, 0, false, nullptr, 0, 0, nullptr}, cm{0, 0, false, nullptr, 0, 0, nullptr};
    open_unit(cl);
    open_unit(cm);
    // raw indices of the load cursor's tile, then advance it
    auto load_idx = [&](int32_t* rr) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int c = cl.j * BN + g * 16 + rsub;
        rr[g] = (cl.in && c < p.k_topk) ? cl.ir[c * p.stk1] : -1;
      }
      advance(cl);
    };
    // K (and V unless shared) row addresses of the make cursor's tile (null =
    // masked), then advance it
    auto make_rows = [&](const int32_t* rr, const T** kr, const T** vr) {
      const int kvh = cm.kvh, ctx = cm.ctx;
      const int32_t* bt_row = cm.bt_row;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int c = cm.j * BN + g * 16 + rsub;
        const int64_t r = rr[g];
        kr[g] = nullptr;
        vr[g] = nullptr;
        if (!(cm.in && c < p.k_topk) || !sp_slot_valid<DECODE>(p, c, r, ctx, bt_row)) continue;
        if (!DECODE) {
          if (r < p.rows1) {
            kr[g] = kb + r * p.k_s0 + kvh * p.k_sh;
            if (!SHARED) vr[g] = vb + r * p.v_s0 + kvh * p.v_sh;
          } else {  // the second source (compressed rows appended after the K/V rows)
            const int64_t cr = r - p.rows1;
            kr[g] = reinterpret_cast<const T*>(p.ck) + cr * p.ck_s0 + kvh * p.ck_sh;
            if (!SHARED) vr[g] = reinterpret_cast<const T*>(p.cv) + cr * p.cv_s0 + kvh * p.cv_sh;
          }
        } else if (c < p.num_win) {  // window slot: logical position -> page, row in page (SA:160-166)
          const int64_t page = bt_row[(r / p.block_size) * p.sbt1];
          const int64_t off = r % p.block_size;
          kr[g] = kb + page * p.k_s0 + kvh * p.k_sh + off * p.k_sr;
          if (!SHARED) vr[g] = vb + page * p.v_s0 + kvh * p.v_sh + off * p.v_sr;
        } else {  // compressed slot: row idx - ctx (SA:205-210)
          const int64_t cr = r - ctx;
          kr[g] = reinterpret_cast<const T*>(p.ck) + cr * p.ck_s0 + kvh * p.ck_sh;
          if (!SHARED) vr[g] = reinterpret_cast<const T*>(p.cv) + cr * p.cv_s0 + kvh * p.cv_sh;
        }
      }
      advance(cm);
    };
    const T* cur[4];
    const T* nxt[4];
    const T* vcur[4];
    const T* vnxt[4];
    int32_t ia[4], ib[4];  // raw indices of tiles J + 1 and J + 2
    bool ok = true;
    int item = 0, J = 0;
    // the Q of unit i (TMA), one K ring item
    auto issue_q = [&](int i) -> bool {
      const int sq = item % NSK;
      if (item >= NSK && !mbar_wait_sleep(&k_empty[sq], ((item / NSK) - 1) & 1)) return false;
      if (pt == 0) {
        const int64_t u = unit_of(i);
        const int y = static_cast<int>(u % p.Y);
        const int h0 = (y / p.head_chunks) * p.G + (y % p.head_chunks) * 64;
        uint8_t* qst = smem + L::KOFF + sq * L::KST;
        mbar_arrive_expect_tx(&k_full[sq], L::NQB * L::BLK);
#pragma unroll 1
        for (int cb = 0; cb < L::NQB; ++cb)
          tma_load_2d(qst + cb * L::BLK, &tmQ, &k_full[sq], cb * 64, static_cast<int>(u / p.Y) * p.H + h0);
      } else {
        mbar_arrive(&k_full[sq]);
      }
      ++item;
      return true;
    };
    // the first Q goes out before the index pipeline is primed, so its copy
    // overlaps the first index loads' memory latency
    if (n_my > 0 && n_tiles > 0) ok = issue_q(0);
    load_idx(ia);
    make_rows(ia, cur, vcur);
    load_idx(ia);
    for (int i = 0; i < n_my && n_tiles > 0 && ok; ++i) {
      if (i > 0 && !(ok = issue_q(i))) break;
      for (int j = 0; j < n_tiles && ok; ++j, ++J, ++item) {
        load_idx(ib);               // tile J + 2
        make_rows(ia, nxt, vnxt);   // tile J + 1
        // ---- K rows of tile J ----
        const int sk = item % NSK;
        if (item >= NSK) ok = mbar_wait_sleep(&k_empty[sk], ((item / NSK) - 1) & 1);
        if (!ok) break;
        uint8_t* kst = smem + L::KOFF + sk * L::KST;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int row = g * 16 + rsub;
          const bool valid = cur[g] != nullptr;
          // masked rows: a zero-byte copy (zero fill) from an in-bounds address
          const T* src = (valid ? cur[g] : kb) + chunk * 8;
          const uint32_t dst_off = row * 128 + ((chunk ^ (row & 7)) << 4);
#pragma unroll
          for (int cb = 0; cb < L::NQB; ++cb) cp_async_16(kst + cb * L::BLK + dst_off, src + cb * 64, valid);
        }
        cp_async_mbar_arrive(&k_full[sk]);
        if constexpr (!SHARED) {
          // ---- V rows of tile J ----
          const int sv = J % NSV;
          if (J >= NSV && !(ok = mbar_wait_sleep(&v_empty[sv], ((J / NSV) - 1) & 1))) break;
          uint8_t* vst = smem + L::VOFF + sv * L::VST;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int row = g * 16 + rsub;
            const bool valid = vcur[g] != nullptr;
            const T* src = (valid ? vcur[g] : vb) + chunk * 8;
            const uint32_t dst_off = row * 128 + ((chunk ^ (row & 7)) << 4);
#pragma unroll
            for (int cb = 0; cb < L::NVB; ++cb) cp_async_16(vst + cb * L::BLK + dst_off, src + cb * 64, valid);
          }
          cp_async_mbar_arrive(&v_full[sv]);
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          cur[g] = nxt[g];
          vcur[g] = vnxt[g];
          ia[g] = ib[g];
        }
      }
    }
    if (!ok) *abort_flag = 1;
    cp_async_wait_all();
  } else if (warp == 8) {
    // ---------------- MMA issuer (greedy order) ----------------
    // The whole warp runs the issuer: one elected lane issues each MMA and
    // commit, every barrier probe is made warp-uniform (all lanes must see the
    // phase complete), and an idle pass sleeps briefly so the spinning warp
    // leaves its SM sub-partition's issue slots to the softmax and gather warps.
    const int NT = n_my * n_tiles;
    if (NT > 0) {
      auto ready = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_test_wait(smem_u32(bar), parity));
      };
      constexpr int AB = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      constexpr int NPV = L::OMAIN < 256 ? L::OMAIN : 256;
      const uint32_t idesc_qk = tc_idesc_f16(AB, 64, BN, 0);
      const uint32_t idesc_pv = tc_idesc_f16(AB, 64, NPV, 1);
      const uint32_t idesc_tail = tc_idesc_f16(AB, 64, 64, 1);
      // descriptors built once, advanced per k-step by constant offsets (see prefill_tc.cu)
      const uint64_t k_desc0 = tc_sdesc_sw128(sbase + L::KOFF, 16, 1024);
      const uint64_t v_desc0 =
          SHARED ? tc_sdesc_sw128(sbase + L::KOFF, L::BLK, 1024) : tc_sdesc_sw128(sbase + L::VOFF, L::BLK, 1024);
      constexpr uint64_t kKStep = static_cast<uint64_t>(L::KST >> 4);
      constexpr uint64_t kVStep = static_cast<uint64_t>((SHARED ? L::KST : L::VST) >> 4);
      const uint64_t p_desc = tc_sdesc_sw128(sbase + L::POFF, 16, 1024);
      const uint32_t q_tmem_addr = taddr + L::QCOL;          // lanes 0-15
      const uint32_t o_main = taddr + (16u << 16);           // lanes 16-31
      const uint32_t o_tail = taddr + L::TCOL;               // lanes 0-15
      bool ok = true;
      int nq = 0, np = 0;  // next QK / PV to issue (tiles over all of this CTA's units)
      // their units, tiles within the unit and K ring items, kept incrementally
      int iq = 0, jq = 0, itq = 1, ip = 0, jp = 0, itp = 1;
      // The wait limit runs from the first idle check after the last MMA
      // issued: progress only sets a flag, so no timer read sits on the issue path.
      uint64_t t0 = globaltimer();
      bool moved = false;
      uint32_t spins = 0;
      while (ok && np < NT) {
        bool did = false;
        // QK of tile nq: its unit's Q in TMEM (first tile of a unit), its K
        // rows loaded, and its S buffer consumed (nq <= np + 1)
        if (nq < NT && nq <= np + 1) {
          const int it = itq;
          if ((jq > 0 || ready(q_tmem, iq & 1)) && ready(&k_full[it % NSK], (it / NSK) & 1)) {
            fence_proxy_async_smem();
            tc_fence_after();
            const int sk = it % NSK;
            const uint32_t d_tmem = taddr + (nq & 1) * 64;
            const uint64_t kd = k_desc0 + sk * kKStep;
#pragma unroll
            for (int kk = 0; kk < DQK / 16; ++kk) {
              const uint64_t koff = static_cast<uint64_t>(((kk >> 2) * L::BLK + (kk & 3) * 32) >> 4);
              tc_mma_ts_w(d_tmem, q_tmem_addr + kk * 8, kd + koff, idesc_qk, kk > 0 ? 1u : 0u);
            }
            tc_commit_w(&s_full[nq & 1]);
            if (!SHARED) tc_commit_w(&k_empty[sk]);  // K rows are done once S is computed
            ++nq;
            ++itq;
            if (++jq == n_tiles) {  // the next unit: its Q item comes first
              jq = 0;
              ++iq;
              ++itq;
            }
            did = true;
          }
        }
        // PV of tile np once its P is in shared memory (and, unshared, its V
        // rows loaded); a unit's first PV overwrites O, so it also waits for
        // the previous unit's epilogue to have read O
        if (np < nq) {
          if ((jp > 0 || ip == 0 || ready(o_free, (ip - 1) & 1)) && ready(p_full, np & 1) &&
              (SHARED || ready(&v_full[np % NSVd], (np / NSVd) & 1))) {
            if (!SHARED) fence_proxy_async_smem();
            tc_fence_after();
            const int sv = SHARED ? itp % NSK : np % NSVd;
            const uint64_t vd = v_desc0 + sv * kVStep;
#pragma unroll
            for (int half = 0; half < (L::OMAIN + 255) / 256; ++half) {
#pragma unroll
              for (int kk = 0; kk < BN / 16; ++kk) {
                const uint64_t a = p_desc + static_cast<uint64_t>((kk * 32) >> 4);
                const uint64_t b = vd + static_cast<uint64_t>((half * 4 * L::BLK + kk * 2048) >> 4);
                tc_mma_ss_w(o_main + half * 256, a, b, idesc_pv, (jp > 0 || kk > 0) ? 1u : 0u);
              }
            }
            if constexpr (L::OTAIL > 0) {
#pragma unroll
              for (int kk = 0; kk < BN / 16; ++kk) {
                const uint64_t a = p_desc + static_cast<uint64_t>((kk * 32) >> 4);
                const uint64_t b = vd + static_cast<uint64_t>((8 * L::BLK + kk * 2048) >> 4);
                tc_mma_ss_w(o_tail, a, b, idesc_tail, (jp > 0 || kk > 0) ? 1u : 0u);
              }
            }
            tc_commit_w(o_done);
            if (SHARED) tc_commit_w(&k_empty[sv]);
            else tc_commit_w(&v_empty[sv]);
            tc_commit_w(p_free);
            ++np;
            ++itp;
            if (++jp == n_tiles) {
              jp = 0;
              ++ip;
              ++itp;
            }
            did = true;
          }
        }
        if (did) {
          moved = true;
        } else {
          __nanosleep(32);
          if ((++spins & 255u) == 0u) {
            const uint64_t now = globaltimer();
            if (moved) {
              t0 = now;
              moved = false;
            }
            if (__any_sync(0xffffffffu, now - t0 > TAK_WAIT_LIMIT_NS * 4 || *abort_flag != 0)) {
              if (lane == 0) record_error(1);
              ok = false;
            }
          }
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp < 4) {
    // ---------------- Q into TMEM, softmax + epilogue: warps 0-3, 16 head rows per warp ----------------
    const int t16 = lane & 15, hi = lane >> 4;
    const int row = 16 * warp + t16;
    const uint32_t s_lane = static_cast<uint32_t>(32 * warp) << 16;       // S, Q, O tail: lanes 0-15
    const uint32_t o_lane = static_cast<uint32_t>(32 * warp + 16) << 16;  // O: lanes 16-31
    // Q of unit i (its K ring item) -> TMEM columns QCOL + k/2 (two 16-bit
    // elements per column): per instruction, threads 0-15 take box 2n and
    // threads 16-31 box 2n + 1 of their rows.  Called once every QK of the
    // previous unit has completed (its last S has been read).  The ring stage
    // is handed back once all 128 threads have arrived on q_tmem, i.e. have
    // read it.
    auto move_q = [&](int i) -> bool {
      const int it = q_item(i), sq = it % NSK;
      if (!mbar_wait(&k_full[sq], (it / NSK) & 1)) return false;
      const uint8_t* qrow = smem + L::KOFF + sq * L::KST + row * 128;
#pragma unroll 1
      for (int n = 0; n < L::NQB / 2; ++n) {
        uint32_t r[32];
        const uint8_t* box = qrow + (2 * n + hi) * L::BLK;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 u = *reinterpret_cast<const uint4*>(box + ((c ^ (row & 7)) << 4));
          r[4 * c] = u.x;
          r[4 * c + 1] = u.y;
          r[4 * c + 2] = u.z;
          r[4 * c + 3] = u.w;
        }
        tmem_st16x2(taddr + s_lane + L::QCOL + 64 * n, r);
      }
      if constexpr (L::NQB % 2) {
        // the odd last box: threads 0-15 its first 32 elements, threads 16-31 the rest
        uint32_t r[16];
        const uint8_t* box = qrow + (L::NQB - 1) * L::BLK;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 u = *reinterpret_cast<const uint4*>(box + (((4 * hi + c) ^ (row & 7)) << 4));
          r[4 * c] = u.x;
          r[4 * c + 1] = u.y;
          r[4 * c + 2] = u.z;
          r[4 * c + 3] = u.w;
        }
        tmem_st16x2_x16(taddr + s_lane + L::QCOL + 32 * (L::NQB - 1), r);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(q_tmem);
      if (tid == 0) {
        if (!mbar_wait(q_tmem, i & 1)) return false;
        fence_proxy_async_smem();
        mbar_arrive(&k_empty[sq]);
      }
      return true;
    };
    bool ok = true;
    if (n_tiles > 0 && n_my > 0) ok = move_q(0);
    int J = 0;  // tiles over all of this CTA's units
    for (int i = 0; i < n_my; ++i) {
      const int64_t u = unit_of(i);
      const int t = static_cast<int>(u / p.Y);
      const int y = static_cast<int>(u % p.Y);
      const int h0 = (y / p.head_chunks) * p.G + (y % p.head_chunks) * 64;
      const int nrows = min(64, p.G - (y % p.head_chunks) * 64);
      const bool row_ok = row < nrows;
      const int head = h0 + row;
      const bool has_sink = p.sink != nullptr;
      const float sink_log2 = (has_sink && row_ok) ? p.sink[head] * kLog2e : -INFINITY;
      const int32_t* idx_row = p.topk + static_cast<int64_t>(t) * p.stk0;
      const int ctx = DECODE ? p.ctx_lens[t] : 0;
      const int32_t* bt_row = DECODE ? p.bt + static_cast<int64_t>(t) * p.sbt0 : nullptr;
      float m_run = -INFINITY, m_used = -INFINITY, l = 0.f;
      auto tile_mask = [&](int j) -> uint32_t {
        // validity of this thread's 32 columns of tile j (lane l: columns l and l+32)
        const int c0 = j * BN + lane, c1 = c0 + 32;
        const int64_t r0 = c0 < p.k_topk ? static_cast<int64_t>(idx_row[c0 * p.stk1]) : -1;
        const int64_t r1 = c1 < p.k_topk ? static_cast<int64_t>(idx_row[c1 * p.stk1]) : -1;
        const uint32_t lo =
            __ballot_sync(0xffffffffu, c0 < p.k_topk && sp_slot_valid<DECODE>(p, c0, r0, ctx, bt_row));
        const uint32_t hi_m =
            __ballot_sync(0xffffffffu, c1 < p.k_topk && sp_slot_valid<DECODE>(p, c1, r1, ctx, bt_row));
        return hi ? hi_m : lo;
      };
      // O columns [c*64, c*64 + 64) of this warp's rows: lanes 16-31 below 512, the tail on lanes 0-15
      auto o_addr = [&](int c) -> uint32_t {
        return c * 64 < L::OMAIN ? taddr + o_lane + c * 64 : taddr + s_lane + L::TCOL + (c * 64 - L::OMAIN);
      };
      uint32_t vnext = (ok && n_tiles > 0) ? tile_mask(0) : 0u;
      for (int j = 0; ok && j < n_tiles; ++j, ++J) {
        const int b = J & 1;
        const uint32_t vbits = vnext;
        if (j + 1 < n_tiles) vnext = tile_mask(j + 1);
        if (!(ok = mbar_wait_sleep(&s_full[b], (J >> 1) & 1))) break;
        tc_fence_after();
        uint32_t sr[32];
        tmem_ld16x2(taddr + s_lane + b * 64, sr);
        tmem_ld_wait();
        // the unit's last S is in registers, so all of its QKs have completed:
        // the next unit's Q may replace it in TMEM while this tile finishes
        if (j == n_tiles - 1 && i + 1 < n_my && !(ok = move_q(i + 1))) break;
        // every column of the warp's tile valid (the common case): no per-score tests
        const bool all_valid = __all_sync(0xffffffffu, vbits == 0xffffffffu);
        float mx = -INFINITY;
        if (all_valid) {
          float m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            mx = fmax3(mx, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
            m1 = fmax3(m1, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
            m2 = fmax3(m2, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
            m3 = fmax3(m3, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
          }
          mx = fmax3(mx, m1, fmaxf(m2, m3));
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if ((vbits >> c) & 1u) mx = fmaxf(mx, __uint_as_float(sr[c]));
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float m_new = fmaxf(m_run, mx * p.scale_log2);
        const bool need = m_new != -INFINITY && m_new > m_used + 8.f;
        const bool resc = need && m_used != -INFINITY;
        if (__any_sync(0xffffffffu, resc)) {
          if (!(ok = mbar_wait(o_done, (J - 1) & 1))) break;
          tc_fence_after();
          const float f = resc ? fast_exp2(m_used - m_new) : 1.f;
          uint32_t orow[32];
#pragma unroll 1
          for (int c = 0; c < DV / 64; ++c) {
            tmem_ld16x2(o_addr(c), orow);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) orow[i] = __float_as_uint(__uint_as_float(orow[i]) * f);
            tmem_st16x2(o_addr(c), orow);
          }
          tmem_st_wait();
          l *= f;
        }
        if (need) m_used = m_new;
        m_run = m_new;
        const float mu = m_used == -INFINITY ? 0.f : m_used;
        uint32_t pk[16];
        float ls = 0.f;
        if (all_valid) {
          // two scores per packed fp32 FMA (same rounding as the scalar form) and per packed row-sum add
          const uint64_t sl2x2 = (static_cast<uint64_t>(__float_as_uint(p.scale_log2)) << 32) |
                                 __float_as_uint(p.scale_log2);
          const uint64_t nmux2 = (static_cast<uint64_t>(__float_as_uint(-mu)) << 32) | __float_as_uint(-mu);
          uint64_t lsx2 = 0;
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
          ls = __uint_as_float(static_cast<uint32_t>(lsx2)) + __uint_as_float(static_cast<uint32_t>(lsx2 >> 32));
        } else {
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const float a = ((vbits >> (2 * c)) & 1u) ? fast_exp2(__uint_as_float(sr[2 * c]) * p.scale_log2 - mu) : 0.f;
            const float bb =
                ((vbits >> (2 * c + 1)) & 1u) ? fast_exp2(__uint_as_float(sr[2 * c + 1]) * p.scale_log2 - mu) : 0.f;
            ls += a + bb;
            pk[c] = Elem<T>::pack2(a, bb);
          }
        }
        l += ls;
        if (J >= 1 && !(ok = mbar_wait_sleep(p_free, (J - 1) & 1))) break;
        uint8_t* prow = smem + L::POFF + row * 128;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int chunk = (hi * 4 + k) ^ (row & 7);
          *reinterpret_cast<uint4*>(prow + chunk * 16) = make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
        }
        fence_proxy_async_smem();
        mbar_arrive(p_full);
      }
      if (ok && n_tiles > 0) ok = mbar_wait(o_done, (J - 1) & 1);
      if (!ok) *abort_flag = 1;
      tc_fence_after();
      const float l_tot = l + __shfl_xor_sync(0xffffffffu, l, 16);
      const float M = fmaxf(m_run, sink_log2);
      const float f = (m_used == -INFINITY) ? 0.f : fast_exp2(m_used - M);
      const float Lsum = l_tot * f + (has_sink && row_ok ? fast_exp2(sink_log2 - M) : 0.f);
      const float inv = (Lsum > 0.f && ok) ? f / Lsum : 0.f;
      T* orow_g = reinterpret_cast<T*>(p.out) + static_cast<int64_t>(t) * p.so_t + static_cast<int64_t>(head) * p.so_h;
#pragma unroll 1
      for (int c = 0; c < DV / 64; ++c) {
        uint32_t o[32];
        if (n_tiles > 0) {
          tmem_ld16x2(o_addr(c), o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (row_ok) {
          T* dst = orow_g + c * 64 + hi * 32;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            uint4 u;
            u.x = Elem<T>::pack2(__uint_as_float(o[8 * k + 0]) * inv, __uint_as_float(o[8 * k + 1]) * inv);
            u.y = Elem<T>::pack2(__uint_as_float(o[8 * k + 2]) * inv, __uint_as_float(o[8 * k + 3]) * inv);
            u.z = Elem<T>::pack2(__uint_as_float(o[8 * k + 4]) * inv, __uint_as_float(o[8 * k + 5]) * inv);
            u.w = Elem<T>::pack2(__uint_as_float(o[8 * k + 6]) * inv, __uint_as_float(o[8 * k + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + 8 * k) = u;
          }
        }
      }
      if (row_ok && hi == 0 && p.lse)
        p.lse[static_cast<int64_t>(t) * p.H + head] = (Lsum > 0.f && ok) ? (M + __log2f(Lsum)) * kLn2 : -INFINITY;
      // O has been read: the next unit's first P.V may overwrite it
      tc_fence_before();
      mbar_arrive(o_free);
      if (!ok) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(taddr, L::TMEM_COLS);
  }
}

// 2-D view [rows, cols] of a 16-bit tensor, box {64 columns, box_rows rows}, 128-byte swizzle.
static int encode_rows_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t row_stride,
                           int box_rows) {
  const uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {static_cast<uint64_t>(row_stride * 2)};
  const uint32_t box[2] = {64, static_cast<uint32_t>(box_rows)};
  const uint32_t es[2] = {1, 1};
  return encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, base, dims, strides, box, es, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <typename T, int DQK, int DV, bool SHARED, bool DECODE>
static int launch_sparse_tc_mode(const SparseArgs& a, cudaStream_t st) {
  using L = SpLayout<DQK, DV, SHARED>;
  const int G = a.num_q_heads / a.num_kv_heads;
  CUtensorMap mq;
  // q as [T * H, Dqk] rows (TMA); gathered K/V rows by cp.async from their row addresses
  if (int r = encode_rows_map(&mq, a.q, static_cast<int64_t>(a.num_tokens) * a.num_q_heads, DQK, a.sq[1], 64)) return r;
  SparseTcParams p{};
  p.topk = a.topk;
  p.stk0 = a.stk[0];
  p.stk1 = a.stk[1];
  p.k_topk = a.k_topk;
  p.kv_rows = a.kv_rows;
  p.sink = a.sink;
  p.out = a.out;
  p.so_t = a.so[0];
  p.so_h = a.so[1];
  p.lse = a.lse;
  p.H = a.num_q_heads;
  p.Hkv = a.num_kv_heads;
  p.G = G;
  p.head_chunks = (G + 63) / 64;
  p.scale_log2 = a.scale * kLog2e;
  p.k = a.k;
  p.v = a.v;
  p.k_s0 = a.sk[0];
  p.k_sh = a.sk[1];
  p.v_s0 = a.sv[0];
  p.v_sh = a.sv[1];
  p.rows1 = a.decode ? 0 : a.rows1;
  if (!a.decode && a.rows1 < a.kv_rows) {
    p.ck = a.ck;
    p.cv = a.cv;
    p.ck_s0 = a.sck[0];
    p.ck_sh = a.sck[1];
    p.cv_s0 = a.scv[0];
    p.cv_sh = a.scv[1];
  }
  if (a.decode) {
    p.k_sr = a.sk[2];
    p.v_sr = a.sv[2];
    p.ck = a.ck;
    p.cv = a.cv;
    p.ck_s0 = a.sck[0];
    p.ck_sh = a.sck[1];
    p.cv_s0 = a.scv[0];
    p.cv_sh = a.scv[1];
    p.bt = a.block_tables;
    p.sbt0 = a.sbt[0];
    p.sbt1 = a.sbt[1];
    p.ctx_lens = a.context_lens;
    p.ncomp = a.num_compressed;
    p.num_win = a.num_win;
    p.block_size = a.block_size;
    p.wreach = static_cast<int64_t>(a.max_blocks) * a.block_size;
    p.num_blocks = a.num_blocks;
  }
  // units (token, KV head group).  Prefill runs persistent CTAs (one per SM,
  // each walking its share of the units, so that the next unit's Q and rows
  // stream in while the current one finishes); decode, with one unit per
  // request, one unit per CTA
  p.Y = a.num_kv_heads * p.head_chunks;
  p.n_units = static_cast<int64_t>(a.num_tokens) * p.Y;
  const int64_t ctas = a.decode ? p.n_units : std::min<int64_t>(p.n_units, num_sms());
  // a CTA counts its tiles and K ring items (a unit's Q, then its tiles) in
  // 32-bit integers: sizes past that take the generic kernel
  if (ctas > 0 && ((p.n_units + ctas - 1) / ctas) * ((static_cast<int64_t>(a.k_topk) + 63) / 64 + 1) > INT32_MAX)
    return -1;
  auto kern = sparse_tc_kernel<T, DQK, DV, SHARED, DECODE>;
  if (const int r = ensure_smem_attr(reinterpret_cast<const void*>(kern), L::SMEM)) return r;
  kern<<<static_cast<unsigned>(ctas), 288, L::SMEM, st>>>(mq, p);
  note_kernel("sparse_tc");
  return 0;
}

template <typename T, int DQK, int DV, bool SHARED>
static int launch_sparse_tc(const SparseArgs& a, cudaStream_t st) {
  return a.decode ? launch_sparse_tc_mode<T, DQK, DV, SHARED, true>(a, st)
                  : launch_sparse_tc_mode<T, DQK, DV, SHARED, false>(a, st);
}

// A gathered row source takes 16-byte copies: base 16-byte aligned, innermost
// stride 1 and every stride the kernel steps by a multiple of 8 elements (the
// head stride only when there is more than one KV head).
static bool rows_ok(const void* ptr, const int64_t* s, int nd, int hkv) {
  if (reinterpret_cast<uintptr_t>(ptr) & 15) return false;
  if (s[nd - 1] != 1) return false;
  for (int i = 0; i < nd - 1; ++i) {
    if (i == 1 && hkv == 1) continue;
    if (s[i] % 8) return false;
  }
  return true;
}

static bool same_view(const void* a, const int64_t* sa, const void* b, const int64_t* sb, int nd) {
  if (a != b) return false;
  for (int i = 0; i < nd; ++i)
    if (sa[i] != sb[i]) return false;
  return true;
}

// Head-dim variants on the tensor cores; -1 = no variant (generic kernel).
// shared: V is a prefix view of K (its rows come from the same gathers).
template <typename T>
static int route_sparse_tc(const SparseArgs& a, cudaStream_t st, bool shared, int dq, int dv) {
  if (dq == 576 && dv == 512) return shared ? launch_sparse_tc<T, 576, 512, true>(a, st)
                                            : launch_sparse_tc<T, 576, 512, false>(a, st);
  if (dq == 576 && dv == 576) return shared ? launch_sparse_tc<T, 576, 576, true>(a, st)
                                            : launch_sparse_tc<T, 576, 576, false>(a, st);
  if (dq == 512 && dv == 512) return shared ? launch_sparse_tc<T, 512, 512, true>(a, st)
                                            : launch_sparse_tc<T, 512, 512, false>(a, st);
  if (dq == dv && dq == 256) return launch_sparse_tc<T, 256, 256, false>(a, st);
  if (dq == dv && dq == 128) return launch_sparse_tc<T, 128, 128, false>(a, st);
  if (dq == dv && dq == 64) return launch_sparse_tc<T, 64, 64, false>(a, st);
  return -1;
}

int sparse_tc_launch(const SparseArgs& a, cudaStream_t st, bool* handled) {
  *handled = false;
  if (a.dtype == kF32) return 0;
  const int G = a.num_q_heads / a.num_kv_heads;
  if (G > 64 && G % 64 != 0) return 0;
  if (a.num_tokens > 2147483647 / 64) return 0;
  // Q rows are TMA row coordinates t * H + h (int32), and decode launches one
  // CTA per (token, KV head group) unit in one grid dimension
  if (static_cast<int64_t>(a.num_tokens) * a.num_q_heads > 2147483647LL) return 0;
  // q rows [T * H, Dqk] must be dense over heads
  if ((reinterpret_cast<uintptr_t>(a.q) & 15) || a.sq[2] != 1 || a.sq[0] != static_cast<int64_t>(a.num_q_heads) * a.sq[1] ||
      (a.sq[1] * 2) % 16 != 0)
    return 0;
  bool shared;
  if (!a.decode) {
    if (!rows_ok(a.k, a.sk, 3, a.num_kv_heads) || !rows_ok(a.v, a.sv, 3, a.num_kv_heads)) return 0;
    shared = same_view(a.v, a.sv, a.k, a.sk, 3);
    if (a.rows1 < a.kv_rows) {  // a second row source
      if (!rows_ok(a.ck, a.sck, 3, a.num_kv_heads) || !rows_ok(a.cv, a.scv, 3, a.num_kv_heads)) return 0;
      shared = shared && same_view(a.cv, a.scv, a.ck, a.sck, 3);
    }
  } else {
    // with no compressed rows every compressed slot is masked and ck/cv are never read
    const bool comp = a.num_compressed > 0;
    if (!rows_ok(a.k, a.sk, 4, a.num_kv_heads) || !rows_ok(a.v, a.sv, 4, a.num_kv_heads) || a.block_size <= 0 ||
        (comp && (!rows_ok(a.ck, a.sck, 3, a.num_kv_heads) || !rows_ok(a.cv, a.scv, 3, a.num_kv_heads))))
      return 0;
    shared = same_view(a.v, a.sv, a.k, a.sk, 4) && (!comp || same_view(a.cv, a.scv, a.ck, a.sck, 3));
  }
  shared = shared && a.head_dim_v <= a.head_dim;
  if (a.so[2] != 1 || (a.so[0] % 8) || (a.so[1] % 8) || (reinterpret_cast<uintptr_t>(a.out) & 15)) return 0;
  const int dq = a.head_dim, dv = a.head_dim_v;
  int r = -1;
  if (a.dtype == kBF16) r = route_sparse_tc<__nv_bfloat16>(a, st, shared, dq, dv);
  else r = route_sparse_tc<__half>(a, st, shared, dq, dv);
  if (r < 0) return 0;
  *handled = true;
  return r;
}

}  // namespace tak

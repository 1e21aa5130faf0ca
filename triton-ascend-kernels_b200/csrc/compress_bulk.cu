// KV compression (CSA windows of two strides, HCA windows of one) streamed
// through shared memory by bulk copies: the pooling of compress_kv_overlap
// (CSA:9-69) and compress_kv_simple (HCA:9-69) for rows that come from a TND
// tensor or straight from a paged cache (the page gather of the decode wrappers,
// CSA:225-253 and HCA:204-230, fused into the pooling).  Plain mean only (the
// reference's pooling); gated pooling stays on compress_stream_kernel.
//
// Work split.  A persistent grid (about four CTAs per SM in all) gives each
// CTA an equal run of consecutive slots; the rows those slots pool (plus the
// one-stride halo of the run's last CSA window) stream through a ring of
// shared-memory stages, each stage a chunk of CH rows of one sequence (its K
// rows, then its V rows).  The last warp is the producer: plain cp.async.bulk
// copies (no tensor map; any layout whose strides keep rows 16-byte aligned),
// one per page piece and tensor when rows are contiguous within a page, else
// one per row, into a stage as soon as every consumer warp has released it,
// completing on the stage's mbarrier, so block-table loads and copy issue never
// stall the consumers.  Every consumer
// thread owns one 16-byte vector (8 elements) of the [K | V] row, adds
// the chunk's rows into the current stride-sized block, and writes a slot as
// soon as its last block completes (a CSA slot is block i + block i+1).
// With V a view of K (MLA latent caches) the caller passes no V and pools K
// once.
//
// Waits are mbarrier waits that suspend the warp in hardware between probes
// (spinning warps would take issue slots from the consumers) and are bounded
// in time; a timed-out wait records a device
// error and the waiting warp leaves its loop (the producer waits, bounded, for
// the copies it issued before it exits).
#include <algorithm>
#include <cstdio>

#include "common.cuh"
#include "kernels.h"

namespace tak {

namespace cb {
constexpr int kMaxStages = 16;
constexpr int kRingBytes = 48 * 1024;  // four CTAs per SM
constexpr int kChunkBytes = 8 * 1024;  // rows per chunk: ~8 KB, between 8 and 32 rows
}  // namespace cb

__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// The segment of a CTA's slot run that lies in one sequence, and the rows it
// pools: slots [i0, i1) of sequence s, rows [r, r_end) (r advances chunk by chunk).
struct BulkSeg {
  int64_t slot, seg_end;
  int s, i0, i1, L, r, r_end;
  int64_t tok0;
};

template <int WIN_BLOCKS>
__device__ __forceinline__ void bulk_seg_open(BulkSeg& g, const CompressArgs& a, int64_t gend) {
  const bool paged = a.cu_seqlens == nullptr;
  while (g.s + 1 < a.num_seqs && a.comp_offsets[g.s + 1] <= g.slot) ++g.s;
  g.seg_end = min(gend, static_cast<int64_t>(a.comp_offsets[g.s + 1]));
  g.i0 = static_cast<int>(g.slot - a.comp_offsets[g.s]);
  g.i1 = static_cast<int>(g.seg_end - a.comp_offsets[g.s]);
  g.L = paged ? a.context_lens[g.s] : (a.cu_seqlens[g.s + 1] - a.cu_seqlens[g.s]);
  g.tok0 = paged ? 0 : a.cu_seqlens[g.s];
  g.r = g.i0 * a.stride;
  g.r_end = min((g.i1 + WIN_BLOCKS - 1) * a.stride, g.L);
}

// Move past a chunk of `ch` rows; opens the next segment when this one is done.
// Returns false when the run is exhausted.
template <int WIN_BLOCKS>
__device__ __forceinline__ bool bulk_seg_next(BulkSeg& g, const CompressArgs& a, int64_t gend, int ch) {
  g.r += ch;
  if (g.r < g.r_end) return true;
  g.slot = g.seg_end;
  if (g.slot >= gend) return false;
  bulk_seg_open<WIN_BLOCKS>(g, a, gend);
  return true;
}

// MC: the stride m when it is known at compile time (4: the reference's CSA),
// else 0.  With MC > 0 and chunks a multiple of MC rows, every chunk starts on
// a block boundary and whole blocks are summed in fresh registers and emitted
// with no per-row tests.
template <typename T, int WIN_BLOCKS, int MC>
__global__ void __launch_bounds__(288) compress_bulk_kernel(const CompressArgs a, int ch, int nst, int span) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int nk = a.head_dim / 8, nv = a.head_dim_v / 8;
  const int ncw = (nk + nv + 31) / 32;  // consumer warps; warp ncw is the producer
  const uint32_t kbytes = nk * 16, vbytes = nv * 16, row_bytes = kbytes + vbytes;
  const uint32_t stage_bytes = row_bytes * ch;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + nst * stage_bytes);
  uint64_t* empty = full + nst;
  const int h = blockIdx.y;
  const int j = threadIdx.x, warp = j >> 5, lane = j & 31;
  const bool paged = a.cu_seqlens == nullptr;
  const int m = a.stride;
  // equal runs of the slots that exist (num_compressed may be a capacity above the total)
  const int64_t total = min(a.num_compressed, static_cast<int64_t>(a.comp_offsets[a.num_seqs]));
  const int64_t slots_per_cta = (total + gridDim.x - 1) / gridDim.x;
  const int64_t g0 = static_cast<int64_t>(blockIdx.x) * slots_per_cta;
  const int64_t gend = min(g0 + slots_per_cta, total);
  if (g0 >= gend) return;

  if (j == 0) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], ncw);
    }
    fence_barrier_init();
  }
  __syncthreads();

  BulkSeg cur_seg;
  cur_seg.slot = g0;
  cur_seg.s = find_slot_seq(a.comp_offsets, a.num_seqs, g0);
  bulk_seg_open<WIN_BLOCKS>(cur_seg, a, gend);

  if (warp == ncw) {
    // ---------------- producer: chunk q -> stage q % nst ----------------
    BulkSeg& pc = cur_seg;
    const T* kb = reinterpret_cast<const T*>(a.k);
    const T* vb = reinterpret_cast<const T*>(a.v);
    int issued = 0;
    for (bool more = true; more; ++issued) {
      const int st = issued % nst;
      if (issued >= nst && !mbar_wait_sleep(&empty[st], ((issued / nst) - 1) & 1, 2000)) break;
      const int n = min(ch, pc.r_end - pc.r);
      // stage layout: the chunk's K rows, then its V rows
      uint8_t* dst = smem + st * stage_bytes;
      uint8_t* vdst = dst + ch * kbytes;
      // this lane's rows [a0, a1) of the chunk and their sources; a paged
      // piece past the block-table row or on a page outside the cache is
      // zero-filled here instead of copied
      const int r0 = pc.r;
      int a0 = r0, a1 = r0;
      int64_t ko = 0, vo = 0;
      bool valid = true;
      if (span) {
        // rows contiguous within a page (or a sequence): one copy per page
        // piece and tensor; lane t takes the piece in the chunk's t-th page
        if (paged) {
          const int pg = r0 / a.block_size + lane;
          a0 = max(r0, pg * a.block_size);
          a1 = max(a0, min(r0 + n, (pg + 1) * a.block_size));
          if (a0 < a1) {
            const int64_t page = paged_row_page(a, pc.s, a0);
            valid = page >= 0;
            const int64_t off = a0 - static_cast<int64_t>(pg) * a.block_size;
            ko = page * a.sk[0] + h * a.sk[1] + off * a.sk[2];
            vo = page * a.sv[0] + h * a.sv[1] + off * a.sv[2];
          }
        } else if (lane == 0) {
          a1 = r0 + n;
          ko = (pc.tok0 + r0) * a.sk[0] + h * a.sk[1];
          vo = (pc.tok0 + r0) * a.sv[0] + h * a.sv[1];
        }
      } else if (lane < n) {
        const int r = r0 + lane;
        a0 = r;
        a1 = r + 1;
        if (paged) {
          const int64_t page = paged_row_page(a, pc.s, r);
          valid = page >= 0;
          const int64_t off = r % a.block_size;
          ko = page * a.sk[0] + h * a.sk[1] + off * a.sk[2];
          vo = page * a.sv[0] + h * a.sv[1] + off * a.sv[2];
        } else {
          ko = (pc.tok0 + r) * a.sk[0] + h * a.sk[1];
          vo = (pc.tok0 + r) * a.sv[0] + h * a.sv[1];
        }
      }
      const int nrow = a1 - a0;
      if (nrow > 0 && !valid) {
        // zero rows, stored before the arrive below publishes the stage
        uint4* zk = reinterpret_cast<uint4*>(dst + (a0 - r0) * kbytes);
        for (uint32_t i = 0; i < nrow * kbytes / 16; ++i) zk[i] = make_uint4(0u, 0u, 0u, 0u);
        uint4* zv = reinterpret_cast<uint4*>(vdst + (a0 - r0) * vbytes);
        for (uint32_t i = 0; i < nrow * vbytes / 16; ++i) zv[i] = make_uint4(0u, 0u, 0u, 0u);
        fence_proxy_async_smem();
      }
      const uint32_t copy_bytes = (nrow > 0 && valid) ? nrow * row_bytes : 0u;
      uint32_t stage_tx = copy_bytes;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) stage_tx += __shfl_xor_sync(0xffffffffu, stage_tx, o);
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(&full[st], stage_tx);
      __syncwarp();
      if (copy_bytes) {
        bulk_copy_g2s(dst + (a0 - r0) * kbytes, kb + ko, nrow * kbytes, &full[st]);
        if (vbytes) bulk_copy_g2s(vdst + (a0 - r0) * vbytes, vb + vo, nrow * vbytes, &full[st]);
      }
      more = bulk_seg_next<WIN_BLOCKS>(pc, a, gend, ch);
    }
    // leave no copy in flight into this CTA's shared memory: the last phase of
    // every stage used has landed (bounded waits)
    if (lane == 0)
      for (int q = max(0, issued - nst); q < issued; ++q) mbar_wait(&full[q % nst], (q / nst) & 1);
    return;
  }

  // ---------------- consumers: thread j owns 16-byte vector j of the [K | V] row ----------------
  const bool active = j < nk + nv;
  const bool is_k = j < nk;
  const int d0 = (is_k ? j : j - nk) * 8;
  const int64_t* so = is_k ? a.sck : a.scv;
  const int64_t so0 = so[0];
  T* const dst_base = reinterpret_cast<T*>(is_k ? a.ck : a.cv) + h * so[1] + d0;
  const float inv_full = 1.f / static_cast<float>(WIN_BLOCKS * m);
  BulkSeg& cc = cur_seg;
  float prev[8], cur[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) prev[e] = cur[e] = 0.f;
  int blk = cc.i0;                              // block being accumulated
  int blk_end = min((blk + 1) * m, cc.r_end);  // row after its last row
  // where the slot finished by block `blk` goes (slot blk, or blk - 1 for CSA)
  T* optr = dst_base + (static_cast<int64_t>(a.comp_offsets[cc.s]) + blk - (WIN_BLOCKS - 1)) * so0;
  auto emit_slot = [&](int emit, const float* acc2, const float* acc1) {
    const int wr0 = emit * m;
    const float inv = wr0 + WIN_BLOCKS * m <= cc.L ? inv_full : 1.f / static_cast<float>(cc.L - wr0);
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = (acc2 ? acc2[e] + acc1[e] : acc1[e]) * inv;
    if (!active) return;
    uint4 q;
    q.x = Elem<T>::pack2(o[0], o[1]);
    q.y = Elem<T>::pack2(o[2], o[3]);
    q.z = Elem<T>::pack2(o[4], o[5]);
    q.w = Elem<T>::pack2(o[6], o[7]);
    __stcg(reinterpret_cast<uint4*>(dst_base + (static_cast<int64_t>(a.comp_offsets[cc.s]) + emit) * so0), q);
  };
  // this thread's vector in a stage ([K rows | V rows]) and its row pitch;
  // idle lanes (past the row's last vector) read K vector 0 and store nothing
  const uint32_t col_off = !active ? 0u : is_k ? j * 16u : ch * kbytes + (j - nk) * 16u;
  const uint32_t pitch = (active && !is_k) ? vbytes : kbytes;
  for (int q = 0, more = 1; more; ++q) {
    const int st = q % nst;
    if (!mbar_wait_sleep(&full[st], (q / nst) & 1, 2000)) break;
    const int n = min(ch, cc.r_end - cc.r);
    const uint8_t* src = smem + st * stage_bytes + col_off;
    auto row_acc = [&](float* acc, int k, bool first) {
      const uint4 u = *reinterpret_cast<const uint4*>(src + k * pitch);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f2 = Elem<T>::unpack2(w[e]);
        acc[2 * e] = first ? f2.x : acc[2 * e] + f2.x;
        acc[2 * e + 1] = first ? f2.y : acc[2 * e + 1] + f2.y;
      }
    };
    auto finish_block = [&]() {
      // block `blk` (in cur) is complete: emit the slot it finishes
      const int emit = WIN_BLOCKS == 1 ? blk : blk - 1;
      if (emit >= cc.i0 && emit < cc.i1) {
        const int wr0 = emit * m;
        if (wr0 + WIN_BLOCKS * m <= cc.L) {
          if (active) {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = (WIN_BLOCKS == 2 ? prev[e] + cur[e] : cur[e]) * inv_full;
            uint4 qv;
            qv.x = Elem<T>::pack2(o[0], o[1]);
            qv.y = Elem<T>::pack2(o[2], o[3]);
            qv.z = Elem<T>::pack2(o[4], o[5]);
            qv.w = Elem<T>::pack2(o[6], o[7]);
            __stcg(reinterpret_cast<uint4*>(optr), qv);
          }
        } else {
          emit_slot(emit, WIN_BLOCKS == 2 ? prev : nullptr, cur);
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        prev[e] = cur[e];
        cur[e] = 0.f;
      }
      ++blk;
      blk_end = min((blk + 1) * m, cc.r_end);
      optr += so0;
    };
    int k = 0;
    if (MC > 0) {
      // whole blocks: MC rows summed straight into cur (empty at a block start)
      for (; k + MC <= n && cc.r + k + MC == blk_end; k += MC) {
        row_acc(cur, k, true);
#pragma unroll
        for (int i = 1; i < MC; ++i) row_acc(cur, k + i, false);
        finish_block();
      }
    }
    while (k < n) {
      // rows of this chunk that belong to block `blk` (a partial block: the
      // sequence end, or any block when MC == 0)
      const int kend = min(n, blk_end - cc.r);
#pragma unroll 4
      for (; k < kend; ++k) row_acc(cur, k, false);
      if (cc.r + kend == blk_end) finish_block();
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);  // this warp is done with the stage
    const bool seg_done = cc.r + ch >= cc.r_end;
    // CSA: the last slot's window ends at the sequence end (block i1 may not exist)
    if (seg_done && WIN_BLOCKS == 2 && cc.i1 * m >= cc.L && cc.i1 - 1 >= cc.i0 && cc.i1 - 1 == blk - 1)
      emit_slot(cc.i1 - 1, nullptr, prev);
    more = bulk_seg_next<WIN_BLOCKS>(cc, a, gend, ch);
    if (seg_done && more) {
#pragma unroll
      for (int e = 0; e < 8; ++e) prev[e] = cur[e] = 0.f;
      blk = cc.i0;
      blk_end = min((blk + 1) * m, cc.r_end);
      optr = dst_base + (static_cast<int64_t>(a.comp_offsets[cc.s]) + blk - (WIN_BLOCKS - 1)) * so0;
    }
  }
}

// ---------------------------------------------------------------------------
// CSA (window 2m, stride m) and HCA (window = stride = m') pooling of the same
// TND rows in one pass, gated (softmax of the gate logits over each window) or
// plain mean (all logits 0): compress_kv_overlap (CSA:9-69) and
// compress_kv_simple (HCA:9-69) on one K/V stream.  One CTA per (HCA slot, KV
// head): its m' rows and the m-row halo of its last CSA window stream through
// the same bulk-copy ring as compress_bulk_kernel.  While the producer's first
// copies are in flight the consumer warps load the slot's gate logits and turn
// them into row weights 2^(g - block max), per-block sums, the two merge
// factors of every CSA slot (its blocks b and b+1) and the factor of every
// block in the HCA slot, all in shared memory; rows are then accumulated per
// m-row block, each CSA slot written as its second block completes, and the
// HCA slot at the end.  With slots of m' rows the grid has one CTA per slot,
// and four CTAs per SM keep every slot of a long batch resident at once.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cb_consumer_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// MC = 4 (the reference's CSA stride) with chunks a multiple of 8 rows: every
// full chunk is whole block pairs, summed into two register sets that swap
// roles, with no per-row tests.
template <typename T, int MC>
__global__ void __launch_bounds__(288) compress_dual_kernel(const CompressArgs csa, const CompressArgs hca, int ch,
                                                            int nst, int span) {
  extern __shared__ __align__(128) uint8_t smem[];
  const CompressArgs& a = csa;  // K, V, gate, cu_seqlens, input strides and head dims are shared
  const int nk = a.head_dim / 8, nv = a.head_dim_v / 8;
  const int ncw = (nk + nv + 31) / 32;  // consumer warps; warp ncw is the producer
  const uint32_t kbytes = nk * 16, vbytes = nv * 16, row_bytes = kbytes + vbytes;
  const uint32_t stage_bytes = row_bytes * ch;
  const int m = csa.stride, mp = hca.stride;
  const int rows_max = mp + m, nb_max = rows_max / m + 1;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + nst * stage_bytes);
  uint64_t* empty = full + nst;
  float* gw = reinterpret_cast<float*>(empty + nst);  // [rows_max] logits, then row weights
  float* bm = gw + rows_max;                          // [nb_max] block max logit
  float* bs = bm + nb_max;                            // [nb_max] block weight sum
  // [nb_max] CSA slot j: factors of blocks j, j + 1 (8-byte aligned: gw is 16-byte aligned)
  float2* fab = reinterpret_cast<float2*>(gw + ((rows_max + 2 * nb_max + 1) & ~1));
  float* bh = reinterpret_cast<float*>(fab + nb_max);  // [nb_max] HCA factor of block b

  const int u = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Launched as a programmatic dependent: no global memory is read before the
  // grid ahead in the stream has completed (its outputs may be this grid's
  // inputs), and from here on the grid after this one may be scheduled, so a
  // chain of these launches overlaps each grid's launch with the drain of the
  // one before.  Without the launch attribute both are no-ops.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (u >= hca.comp_offsets[hca.num_seqs]) return;  // num_compressed may be a capacity
  const int s = find_slot_seq(hca.comp_offsets, hca.num_seqs, u);
  const int i = u - hca.comp_offsets[s];
  const int64_t tok0 = a.cu_seqlens[s];
  const int L = a.cu_seqlens[s + 1] - a.cu_seqlens[s];
  const int r_begin = i * mp;
  const int nrows_h = min(mp, L - r_begin);    // rows of the HCA slot
  const int nrows = min(mp + m, L - r_begin);  // plus the halo of its last CSA window
  const int nb = (nrows + m - 1) / m, nbh = (nrows_h + m - 1) / m;
  const int c0 = csa.comp_offsets[s];
  const int j_begin = r_begin / m;  // local CSA slot j is slot j_begin + j of the sequence
  const int nj = max(0, min(mp / m, csa.comp_offsets[s + 1] - c0 - j_begin));

  if (tid == 0) {
    for (int q = 0; q < nst; ++q) {
      mbar_init(&full[q], 1);
      mbar_init(&empty[q], ncw);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == ncw) {
    // ---------------- producer: chunk q (rows [q*ch, q*ch + n)) -> stage q % nst ----------------
    const T* kb = reinterpret_cast<const T*>(a.k) + (tok0 + r_begin) * a.sk[0] + h * a.sk[1];
    const T* vb = reinterpret_cast<const T*>(a.v) + (tok0 + r_begin) * a.sv[0] + h * a.sv[1];
    int issued = 0;
    for (int r0 = 0; r0 < nrows; r0 += ch, ++issued) {
      const int st = issued % nst;
      if (issued >= nst && !mbar_wait_sleep(&empty[st], ((issued / nst) - 1) & 1, 2000)) break;
      const int n = min(ch, nrows - r0);
      uint8_t* dst = smem + st * stage_bytes;
      uint8_t* vdst = dst + ch * kbytes;
      if (lane == 0) mbar_arrive_expect_tx(&full[st], n * row_bytes);
      __syncwarp();
      if (span) {  // rows of a sequence are contiguous: one copy per tensor
        if (lane == 0) {
          bulk_copy_g2s(dst, kb + r0 * a.sk[0], n * kbytes, &full[st]);
          if (vbytes) bulk_copy_g2s(vdst, vb + r0 * a.sv[0], n * vbytes, &full[st]);
        }
      } else if (lane < n) {
        bulk_copy_g2s(dst + lane * kbytes, kb + (r0 + lane) * a.sk[0], kbytes, &full[st]);
        if (vbytes) bulk_copy_g2s(vdst + lane * vbytes, vb + (r0 + lane) * a.sv[0], vbytes, &full[st]);
      }
    }
    // leave no copy in flight into this CTA's shared memory (bounded waits)
    if (lane == 0)
      for (int q = max(0, issued - nst); q < issued; ++q) mbar_wait(&full[q % nst], (q / nst) & 1);
    return;
  }

  // ---------------- consumers: window weights from the gate logits ----------------
  const int nct = ncw * 32;
  for (int r = tid; r < nrows; r += nct)
    gw[r] = a.gate ? __ldg(a.gate + (tok0 + r_begin + r) * a.sg[0]) : 0.f;
  cb_consumer_sync(nct);
  for (int b = tid; b < nb; b += nct) {
    const int r0 = b * m, r1 = min(r0 + m, nrows);
    float mx = -INFINITY;
    for (int r = r0; r < r1; ++r) mx = fmaxf(mx, gw[r]);
    float sum = 0.f;
    for (int r = r0; r < r1; ++r) {
      // a block whose logits are all -inf (masked rows) carries no weight
      const float w = mx == -INFINITY ? 0.f : __expf(gw[r] - mx);
      gw[r] = w;
      sum += w;
    }
    bm[b] = mx;
    bs[b] = sum;
  }
  cb_consumer_sync(nct);
  if (warp == 0) {
    // HCA slot: softmax over its rows = blocks [0, nbh) merged at their maxima
    float mh = -INFINITY;
    for (int b = lane; b < nbh; b += 32) mh = fmaxf(mh, bm[b]);
    mh = warp_max(mh);
    float hs = 0.f;
    for (int b = lane; b < nbh; b += 32) {
      const float f = bm[b] == -INFINITY ? 0.f : __expf(bm[b] - mh);
      bh[b] = f;
      hs += f * bs[b];
    }
    hs = warp_sum(hs);
    const float hinv = hs > 0.f ? 1.f / hs : 0.f;
    for (int b = lane; b < nbh; b += 32) bh[b] *= hinv;
    // CSA slot j: blocks j and j + 1 (the second missing at the sequence end)
    for (int j = lane; j < nj; j += 32) {
      const bool two = j + 1 < nb;
      const float ma = bm[j], mb = two ? bm[j + 1] : -INFINITY, Mx = fmaxf(ma, mb);
      const float fa = ma == -INFINITY ? 0.f : __expf(ma - Mx);
      const float fb = mb == -INFINITY ? 0.f : __expf(mb - Mx);
      const float den = bs[j] * fa + (two ? bs[j + 1] * fb : 0.f);
      const float inv = den > 0.f ? 1.f / den : 0.f;
      fab[j] = make_float2(fa * inv, fb * inv);
    }
  }
  cb_consumer_sync(nct);

  // ---------------- consumers: thread tid owns 16-byte vector tid of the [K | V] row ----------------
  const bool active = tid < nk + nv;
  const bool is_k = tid < nk;
  const int d0 = (is_k ? tid : tid - nk) * 8;
  const uint32_t col_off = !active ? 0u : is_k ? tid * 16u : ch * kbytes + (tid - nk) * 16u;
  const uint32_t pitch = (active && !is_k) ? vbytes : kbytes;
  const int64_t so0 = is_k ? csa.sck[0] : csa.scv[0];
  T* csa_out = reinterpret_cast<T*>(is_k ? csa.ck : csa.cv) + (static_cast<int64_t>(c0) + j_begin) * so0 +
               h * (is_k ? csa.sck[1] : csa.scv[1]) + d0;
  T* hca_out = reinterpret_cast<T*>(is_k ? hca.ck : hca.cv) +
               static_cast<int64_t>(hca.comp_offsets[s] + i) * (is_k ? hca.sck[0] : hca.scv[0]) +
               h * (is_k ? hca.sck[1] : hca.scv[1]) + d0;
  auto store8 = [&](T* dst, const float* o) {
    uint4 q;
    q.x = Elem<T>::pack2(o[0], o[1]);
    q.y = Elem<T>::pack2(o[2], o[3]);
    q.z = Elem<T>::pack2(o[4], o[5]);
    q.w = Elem<T>::pack2(o[6], o[7]);
    __stcg(reinterpret_cast<uint4*>(dst), q);
  };
  float prev[8], cur[8], hacc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) prev[e] = cur[e] = hacc[e] = 0.f;
  int blk = 0, blk_end = min(m, nrows);
  // one row into an accumulator (first: overwrite)
  auto row_acc = [&](float* acc, const uint8_t* src, float w, bool first) {
    const uint4 u4 = *reinterpret_cast<const uint4*>(src);
    const uint32_t wd[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f2 = Elem<T>::unpack2(wd[e]);
      acc[2 * e] = first ? w * f2.x : fmaf(w, f2.x, acc[2 * e]);
      acc[2 * e + 1] = first ? w * f2.y : fmaf(w, f2.y, acc[2 * e + 1]);
    }
  };
  // block b (in c, the previous block in pv) is complete: CSA slot b - 1, HCA share
  auto finish = [&](int b, const float* pv, const float* c) {
    if (b >= 1 && b - 1 < nj && active) {
      const float2 f = fab[b - 1];
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = fmaf(pv[e], f.x, c[e] * f.y);
      store8(csa_out + static_cast<int64_t>(b - 1) * so0, o);
    }
    if (b < nbh) {
      const float hf = bh[b];
#pragma unroll
      for (int e = 0; e < 8; ++e) hacc[e] = fmaf(c[e], hf, hacc[e]);
    }
  };
  int q = 0;
  for (int r0 = 0; r0 < nrows; r0 += ch, ++q) {
    const int st = q % nst;
    if (!mbar_wait_sleep(&full[st], (q / nst) & 1, 2000)) break;
    const int n = min(ch, nrows - r0);
    const uint8_t* src = smem + st * stage_bytes + col_off;
    int k = 0;
    if (MC == 4) {
      // whole block pairs: A = block blk, B = block blk + 1; prev holds block blk - 1
      for (; k + 8 <= n; k += 8) {
        const float4 wa = *reinterpret_cast<const float4*>(gw + r0 + k);
        const float4 wb = *reinterpret_cast<const float4*>(gw + r0 + k + 4);
        row_acc(cur, src + (k + 0) * pitch, wa.x, true);
        row_acc(cur, src + (k + 1) * pitch, wa.y, false);
        row_acc(cur, src + (k + 2) * pitch, wa.z, false);
        row_acc(cur, src + (k + 3) * pitch, wa.w, false);
        finish(blk, prev, cur);
        row_acc(prev, src + (k + 4) * pitch, wb.x, true);
        row_acc(prev, src + (k + 5) * pitch, wb.y, false);
        row_acc(prev, src + (k + 6) * pitch, wb.z, false);
        row_acc(prev, src + (k + 7) * pitch, wb.w, false);
        finish(blk + 1, cur, prev);
        blk += 2;
      }
      blk_end = min((blk + 1) * m, nrows);
#pragma unroll
      for (int e = 0; e < 8; ++e) cur[e] = 0.f;
    }
    for (; k < n; ++k) {
      const int r = r0 + k;
      row_acc(cur, src + k * pitch, gw[r], false);
      if (r + 1 == blk_end) {
        finish(blk, prev, cur);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          prev[e] = cur[e];
          cur[e] = 0.f;
        }
        ++blk;
        blk_end = min((blk + 1) * m, nrows);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
  if (!active) return;
  // the last CSA slot whose second block is past the sequence end
  if (nb - 1 < nj) {
    const float fa = fab[nb - 1].x;
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = prev[e] * fa;
    store8(csa_out + static_cast<int64_t>(nb - 1) * so0, o);
  }
  store8(hca_out, hacc);
}

// One-pass CSA + HCA pooling on the bulk-copy pipeline; false (nothing
// launched) for shapes it does not take.
template <typename T>
static bool compress_dual_typed(const CompressArgs& csa, const CompressArgs& hca, cudaStream_t st, int* err) {
  const CompressArgs& a = csa;
  if (!a.cu_seqlens || !hca.cu_seqlens) return false;
  if (csa.window != 2 * csa.stride || hca.window != hca.stride || hca.stride % csa.stride) return false;
  if (csa.stride > 64 || hca.stride + csa.stride > 2048) return false;
  const int nk = a.head_dim / 8, nv = a.head_dim_v / 8;
  if (a.head_dim % 8 || a.head_dim_v % 8 || nk + nv > 256 || nk == 0 || !a.v) return false;
  if (a.sk[2] != 1 || a.sv[2] != 1 || a.sk[0] % 8 || a.sk[1] % 8 || a.sv[0] % 8 || a.sv[1] % 8) return false;
  if ((reinterpret_cast<uintptr_t>(a.k) | reinterpret_cast<uintptr_t>(a.v)) & 15) return false;
  for (const CompressArgs* o : {&csa, &hca}) {
    if (o->sck[2] != 1 || o->scv[2] != 1 || o->sck[0] % 8 || o->sck[1] % 8 || o->scv[0] % 8 || o->scv[1] % 8)
      return false;
    if ((reinterpret_cast<uintptr_t>(o->ck) | reinterpret_cast<uintptr_t>(o->cv)) & 15) return false;
  }
  const int row_bytes = (nk + nv) * 16;
  const int ch = max(8, min(32, cb::kChunkBytes / row_bytes));
  const int nst = max(2, min(cb::kMaxStages, cb::kRingBytes / (row_bytes * ch)));
  const int rows_max = hca.stride + csa.stride, nb_max = rows_max / csa.stride + 1;
  const int smem = nst * row_bytes * ch + 2 * nst * 8 + (rows_max + 6 * nb_max + 4) * 4;
  const int threads = ((nk + nv + 31) / 32 + 1) * 32;
  const int span = (a.sk[0] * 2 == nk * 16 && a.sv[0] * 2 == nv * 16) ? 1 : 0;
  auto kern = (csa.stride == 4 && ch % 8 == 0) ? compress_dual_kernel<T, 4> : compress_dual_kernel<T, 0>;
  if ((*err = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem))) return true;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(hca.num_compressed), a.num_kv_heads);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, csa, hca, ch, nst, span);
  if (e != cudaSuccess) {
    char buf[160];
    std::snprintf(buf, sizeof(buf), "CSA + HCA compression: launch failed: %s", cudaGetErrorString(e));
    *err = set_error(3, buf);
    return true;
  }
  note_kernel("compress_dual");
  return true;
}

bool compress_dual_launch(const CompressArgs& csa, const CompressArgs& hca, cudaStream_t st, int* err) {
  *err = 0;
  if (csa.dtype == kBF16) return compress_dual_typed<__nv_bfloat16>(csa, hca, st, err);
  if (csa.dtype == kF16) return compress_dual_typed<__half>(csa, hca, st, err);
  return false;
}

// Takes plain-mean pooling of 16-bit rows whose every stride is a multiple of
// 8 elements, with windows of one or two strides.  Returns false (nothing
// launched) for anything else.
template <typename T>
static bool compress_bulk_typed(const CompressArgs& a, cudaStream_t st, int* err) {
  const bool paged = a.cu_seqlens == nullptr;
  if (a.gate) return false;
  if (!(a.window == a.stride || a.window == 2 * a.stride)) return false;
  const int nk = a.head_dim / 8, nv = a.head_dim_v / 8;
  if (a.head_dim % 8 || a.head_dim_v % 8 || nk + nv > 256 || nk == 0) return false;
  const int nd = paged ? 4 : 3;
  if (a.sk[nd - 1] != 1 || (a.v && a.sv[nd - 1] != 1)) return false;
  for (int i = 0; i < nd - 1; ++i) {
    if (a.sk[i] % 8) return false;
    if (a.v && a.sv[i] % 8) return false;
  }
  if ((reinterpret_cast<uintptr_t>(a.k) | reinterpret_cast<uintptr_t>(a.v)) & 15) return false;
  if (a.sck[2] != 1 || a.sck[0] % 8 || a.sck[1] % 8 || (reinterpret_cast<uintptr_t>(a.ck) & 15)) return false;
  if (a.cv && (a.scv[2] != 1 || a.scv[0] % 8 || a.scv[1] % 8 || (reinterpret_cast<uintptr_t>(a.cv) & 15)))
    return false;
  const int row_bytes = (nk + nv) * 16;
  const int ch = max(8, min(32, cb::kChunkBytes / row_bytes));
  const int nst = max(2, min(cb::kMaxStages, cb::kRingBytes / (row_bytes * ch)));
  const int smem = nst * row_bytes * ch + nst * 16;
  const int threads = ((nk + nv + 31) / 32 + 1) * 32;  // consumer warps + the producer warp
  // ~4 CTAs per SM over all KV heads; each CTA takes an equal run of the slots
  // (sized on the device from the offsets)
  const int64_t target = static_cast<int64_t>(num_sms()) * 4;
  const int64_t per_head = std::max<int64_t>(1, (target + a.num_kv_heads - 1) / a.num_kv_heads);
  const unsigned ctas = static_cast<unsigned>(std::min<int64_t>(per_head, a.num_compressed));
  const dim3 grid(ctas, a.num_kv_heads);
  // rows whose pitch equals the copied bytes are contiguous within a page (a
  // sequence, for TND): the producer copies page pieces instead of single rows
  const int64_t kp = paged ? a.sk[2] : a.sk[0], vp = paged ? a.sv[2] : a.sv[0];
  const int span = (kp * 2 == nk * 16 && (!a.v || vp * 2 == nv * 16)) ? 1 : 0;
  void (*kern)(const CompressArgs, int, int, int);
  const bool m4 = a.stride == 4 && ch % 4 == 0;
  if (a.window == a.stride) kern = m4 ? compress_bulk_kernel<T, 1, 4> : compress_bulk_kernel<T, 1, 0>;
  else kern = m4 ? compress_bulk_kernel<T, 2, 4> : compress_bulk_kernel<T, 2, 0>;
  if ((*err = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem))) return true;
  kern<<<grid, threads, smem, st>>>(a, ch, nst, span);
  note_kernel("compress_bulk");
  *err = 0;
  return true;
}

bool compress_bulk_launch(const CompressArgs& a, cudaStream_t st, int* err) {
  *err = 0;
  if (a.dtype == kBF16) return compress_bulk_typed<__nv_bfloat16>(a, st, err);
  if (a.dtype == kF16) return compress_bulk_typed<__half>(a, st, err);
  return false;
}

}  // namespace tak

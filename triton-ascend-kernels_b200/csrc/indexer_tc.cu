// Lightning-indexer scores on the 5th-generation tensor cores (prefill rows).
//
// The reference scores every query row of a sequence against the sequence's
// compressed keys with one matmul (CSA:144): s[t, i] = q[t, H-1, :] .
// k~[c0(s) + i, H_kv-1, :], the last query head and the last KV head deciding
// the selection (the per-head writes of CSA:136-162 leave the last head's
// choice), the product rounded to the input dtype (the matmul's output).  Here
// that product is a tcgen05 GEMM: a CTA computes a 128-row x 128-slot tile of
// one sequence (K = head_dim in 64-column blocks), fp32 in tensor memory,
// rounds it to the input dtype and writes it to a score scratch [T, ld] that
// the selection kernel (csa_indexer_kernel) reads instead of computing the dot
// products on CUDA cores -- which re-read every compressed key from L2 once per
// query row.  Tiles entirely above the causal limit (slot i needs i*m < pos)
// are skipped; a row block that crosses a sequence boundary is computed once
// per sequence it touches, each time storing only its own rows.
//
// Warp roles (192 threads):
//   warp 4   TMA producer: per 64-column block one load of the 128 query rows
//            (head H-1) and one of the 128 compressed rows (head H_kv-1), both
//            with the 128-byte swizzle, into a 3-stage ring;
//   warp 5   TMEM allocator + single-thread tcgen05.mma issuer (M = N = 128,
//            K = 16 per instruction, descriptors built once per stage);
//   warps 0-3 epilogue: thread = tile row = TMEM lane, 4 loads of 32 columns,
//            rounding, 16-byte stores of the row's 128 scores.
// Every wait is an mbarrier wait bounded in time; a timed-out wait records a
// device error and the roles unwind (the producer first waits, bounded, for
// its loads in flight).
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace tak {

namespace it {
constexpr int kStages = 3;  // 99 KB of shared memory: two CTAs per SM
constexpr int kTile = 128;
constexpr int kBlk = 128 * 128;  // one 64-column block of a 128-row tile (bytes)
constexpr int kStage = 2 * kBlk;
constexpr int kBarOff = kStages * kStage;
constexpr int kSmem = kBarOff + 256 + 1024;
}  // namespace it

struct ScoreParams {
  const int32_t* cu;
  const int32_t* offs;
  int num_seqs, total_tokens, m, kblocks;
  int qcol0, kcol0;  // TMA x coordinate of head H-1 in q, of head H_kv-1 in the compressed keys
  void* scores;
  int64_t ld;
};

__device__ __forceinline__ void it_tma_2d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Sequences whose rows meet row block [row0, row0 + 128) and whose causal
// slots reach slot block cb: calls f(s, lo, hi) with the block's rows [lo, hi)
// of sequence s.  Every thread walks the same list.
template <class F>
__device__ __forceinline__ void it_for_items(const ScoreParams& p, int row0, int cb, F&& f) {
  int lo_s = 0, hi_s = p.num_seqs - 1, s0 = 0;
  while (lo_s <= hi_s) {  // last sequence starting at or before row0
    const int mid = (lo_s + hi_s) >> 1;
    if (p.cu[mid] <= row0) {
      s0 = mid;
      lo_s = mid + 1;
    } else {
      hi_s = mid - 1;
    }
  }
  for (int s = s0; s < p.num_seqs && p.cu[s] < row0 + it::kTile; ++s) {
    const int a = max(row0, p.cu[s]), b = min(row0 + it::kTile, p.cu[s + 1]);
    if (a >= b) continue;
    const int max_pos = b - 1 - p.cu[s];
    const int nc = p.offs[s + 1] - p.offs[s];
    const int nvalid = min(nc, (max_pos + p.m - 1) / p.m);
    if (cb * it::kTile >= nvalid) continue;
    f(s, a, b);
  }
}

template <typename T>
__global__ void __launch_bounds__(192, 1)
    csa_scores_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const ScoreParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + it::kBarOff);
  uint64_t* full = bars;                   // [kStages]
  uint64_t* empty = bars + it::kStages;    // [kStages]
  uint64_t* acc_full = bars + 2 * it::kStages;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int row0 = blockIdx.x * it::kTile, cb = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // nothing to do: leave before allocating anything
  int n_items = 0;
  it_for_items(p, row0, cb, [&](int, int, int) { ++n_items; });
  if (n_items == 0) return;

  if (threadIdx.x == 0) {
    for (int i = 0; i < it::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_holder, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = *tmem_holder;

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      int q = 0;
      bool ok = true;
      it_for_items(p, row0, cb, [&](int s, int, int) {
        const int boff = p.offs[s] + cb * it::kTile;
        for (int kb = 0; kb < p.kblocks && ok; ++kb, ++q) {
          const int st = q % it::kStages;
          if (q >= it::kStages && !(ok = mbar_wait(&empty[st], ((q / it::kStages) - 1) & 1))) break;
          if (*abort_flag) {
            ok = false;
            break;
          }
          uint8_t* dst = smem + st * it::kStage;
          mbar_arrive_expect_tx(&full[st], it::kStage);
          it_tma_2d(dst, &tmQ, &full[st], p.qcol0 + kb * 64, row0);
          it_tma_2d(dst + it::kBlk, &tmK, &full[st], p.kcol0 + kb * 64, boff);
        }
      });
      if (!ok) *abort_flag = 1;
      // leave no load in flight into this CTA's shared memory
      for (int j = max(0, q - it::kStages); j < q; ++j) mbar_wait(&full[j % it::kStages], (j / it::kStages) & 1);
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr int AB = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      const uint32_t idesc = tc_idesc_f16(AB, 128, 128, 0);
      const uint32_t sbase = smem_u32(smem);
      int q = 0, n = 0;
      bool ok = true;
      it_for_items(p, row0, cb, [&](int, int, int) {
        if (!ok) return;
        if (n >= 1 && !(ok = mbar_wait(acc_empty, (n - 1) & 1))) return;
        tc_fence_after();
        for (int kb = 0; kb < p.kblocks; ++kb, ++q) {
          const int st = q % it::kStages;
          if (!(ok = mbar_wait(&full[st], (q / it::kStages) & 1)) || *abort_flag) {
            ok = false;
            return;
          }
          tc_fence_after();
          const uint64_t a_desc = tc_sdesc_sw128(sbase + st * it::kStage, 16, 1024);
          const uint64_t b_desc = tc_sdesc_sw128(sbase + st * it::kStage + it::kBlk, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc_mma_ss(taddr, a_desc + 2 * kk, b_desc + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&empty[st]);
        }
        tc_commit(acc_full);
        ++n;
      });
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ---------------- epilogue: thread = tile row = TMEM lane ----------------
    const int r = 32 * warp + lane;
    const int row = row0 + r;
    int n = 0;
    bool ok = true;
    it_for_items(p, row0, cb, [&](int, int lo, int hi) {
      if (!ok) return;
      if (!(ok = mbar_wait(acc_full, n & 1))) {
        *abort_flag = 1;
        return;
      }
      tc_fence_after();
      const bool mine = row >= lo && row < hi && row < p.total_tokens;
      T* dst = reinterpret_cast<T*>(p.scores) + static_cast<int64_t>(row) * p.ld + cb * it::kTile;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(taddr + (static_cast<uint32_t>(32 * warp) << 16) + c * 32, v);
        tmem_ld_wait();
        if (mine) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 u;
            u.x = Elem<T>::pack2(__uint_as_float(v[8 * g + 0]), __uint_as_float(v[8 * g + 1]));
            u.y = Elem<T>::pack2(__uint_as_float(v[8 * g + 2]), __uint_as_float(v[8 * g + 3]));
            u.z = Elem<T>::pack2(__uint_as_float(v[8 * g + 4]), __uint_as_float(v[8 * g + 5]));
            u.w = Elem<T>::pack2(__uint_as_float(v[8 * g + 6]), __uint_as_float(v[8 * g + 7]));
            *reinterpret_cast<uint4*>(dst + c * 32 + 8 * g) = u;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      ++n;
    });
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(taddr, 128);
  }
}

// ---------------------------------------------------------------------------
// Selection from the tensor-core scores: one warp per query row, the whole
// bitonic sort in registers.  A score is a 16-bit value (rounded to the input
// dtype) and a slot index fits 16 bits, so key = order-preserving score bits
// (-0 folded into +0) above the complemented slot: descending key order is
// descending score, ties to the lower slot (the order of csa_indexer_kernel).
// Lane l holds keys l*E .. l*E + E-1 of N = 32*E (padding keys 0, below every
// real key); compare-exchange partners closer than E are in the same lane,
// farther ones one shuffle away.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ uint32_t it_key(T v, int slot) {
  uint32_t b = Elem<T>::bits(v);
  if (b == 0x8000u) b = 0u;  // -0 sorts with +0
  b = (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
  return (b << 16) | (0xffffu - static_cast<uint32_t>(slot));
}

template <int E>
__device__ __forceinline__ void it_warp_sort_desc(uint32_t (&k)[E], int lane) {
  constexpr int N = 32 * E;
#pragma unroll
  for (int kk = 2; kk <= N; kk <<= 1) {
#pragma unroll
    for (int j = kk >> 1; j > 0; j >>= 1) {
      if (j >= E) {
        const int lm = j / E;
        const bool lower = (lane & lm) == 0;
#pragma unroll
        for (int r = 0; r < E; ++r) {
          const uint32_t o = __shfl_xor_sync(0xffffffffu, k[r], lm);
          const bool desc = ((lane * E + r) & kk) == 0;  // this pair's segment sorts descending
          const uint32_t hi = max(k[r], o), lo = min(k[r], o);
          k[r] = (desc == lower) ? hi : lo;
        }
      } else {
#pragma unroll
        for (int r = 0; r < E; ++r) {
          if (r & j) continue;
          const int r2 = r | j;
          const bool desc = ((lane * E + r) & kk) == 0;
          const uint32_t hi = max(k[r], k[r2]), lo = min(k[r], k[r2]);
          k[r] = desc ? hi : lo;
          k[r2] = desc ? lo : hi;
        }
      }
    }
  }
}

template <typename T, int E>
__device__ __forceinline__ void it_select_row(const T* srow, int n_valid, int n_pick, int64_t base, int32_t* out,
                                              int lane) {
  uint32_t k[E];
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const int i = lane * E + r;
    k[r] = i < n_valid ? it_key<T>(srow[i], i) : 0u;
  }
  it_warp_sort_desc<E>(k, lane);
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const int rank = lane * E + r;
    if (rank < n_pick) out[rank] = static_cast<int32_t>(base + (0xffffu - (k[r] & 0xffffu)));
  }
}

// Rows of up to 1024 causal slots (the kernel is launched only when every
// sequence has at most 1024 slots); 8 rows per 256-thread CTA.
template <typename T>
__global__ void __launch_bounds__(256) csa_select_warp_kernel(const IndexerArgs a) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= a.total_tokens) return;
  int lo_s = 0, hi_s = a.num_seqs - 1, s = -1;
  while (lo_s <= hi_s) {
    const int mid = (lo_s + hi_s) >> 1;
    if (a.cu_seqlens[mid] <= row) {
      s = mid;
      lo_s = mid + 1;
    } else {
      hi_s = mid - 1;
    }
  }
  if (s < 0 || row >= a.cu_seqlens[s + 1]) return;
  const int pos = row - a.cu_seqlens[s];
  const int c0 = a.comp_offsets[s];
  const int nc = min(a.comp_offsets[s + 1] - c0, a.max_comp_per_seq);
  if (nc <= 0) return;
  const int k_sel = min(a.top_k, nc);
  const int n_valid = pos <= 0 ? 0 : min(nc, (pos + a.m - 1) / a.m);
  const int n_pick = min(k_sel, n_valid);
  const int64_t base = static_cast<int64_t>(a.total_tokens) + c0;
  int32_t* out = a.out + static_cast<int64_t>(row) * a.ld + a.n_win;
  const T* srow = reinterpret_cast<const T*>(a.scores) + static_cast<int64_t>(row) * a.sld;
  if (n_pick > 0) {
    if (n_valid <= 64) it_select_row<T, 2>(srow, n_valid, n_pick, base, out, lane);
    else if (n_valid <= 128) it_select_row<T, 4>(srow, n_valid, n_pick, base, out, lane);
    else if (n_valid <= 256) it_select_row<T, 8>(srow, n_valid, n_pick, base, out, lane);
    else if (n_valid <= 512) it_select_row<T, 16>(srow, n_valid, n_pick, base, out, lane);
    else it_select_row<T, 32>(srow, n_valid, n_pick, base, out, lane);
  }
  // fewer causal slots than k_sel: the masked slots follow in ascending order
  for (int r = n_pick + lane; r < k_sel; r += 32) out[r] = static_cast<int32_t>(base + r);
}

bool csa_select_warp_launch(const IndexerArgs& a, cudaStream_t st) {
  if (!a.cu_seqlens || !a.scores || a.dtype == kF32 || a.max_comp_per_seq > 1024) return false;
  const unsigned grid = static_cast<unsigned>((a.total_tokens + 7) / 8);
  if (a.dtype == kBF16)
    csa_select_warp_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(a);
  else
    csa_select_warp_kernel<__half><<<grid, 256, 0, st>>>(a);
  return true;
}

// Rows of up to 2048 causal slots with few rows (decode): one 512-thread CTA
// per row, thread t holding keys 4t .. 4t+3 of a 2048-key bitonic network.
// Partners closer than 4 keys are in the same thread, closer than 128 one
// shuffle away; only the 10 passes with partners in another warp exchange
// through shared memory (one 16-byte store and load per thread).
template <typename T>
__global__ void __launch_bounds__(512) csa_select_block_kernel(const IndexerArgs a) {
  constexpr int E = 4, N = 512 * E;
  __shared__ uint4 xk[512];
  const int row = blockIdx.x;  // decode: sequence = row
  const int tid = threadIdx.x, lane = tid & 31;
  const int pos = a.context_lens[row];
  const int c0 = a.comp_offsets[row];
  const int nc = min(a.comp_offsets[row + 1] - c0, a.max_comp_per_seq);
  if (nc <= 0) return;
  const int k_sel = min(a.top_k, nc);
  const int n_valid = pos <= 0 ? 0 : min(nc, (pos + a.m - 1) / a.m);
  const int n_pick = min(k_sel, n_valid);
  const int64_t base = static_cast<int64_t>(pos) + c0;
  int32_t* out = a.out + static_cast<int64_t>(row) * a.ld + a.n_win;
  if (n_pick > 0) {
    const T* srow = reinterpret_cast<const T*>(a.scores) + static_cast<int64_t>(row) * a.sld;
    uint32_t k[E];
#pragma unroll
    for (int r = 0; r < E; ++r) {
      const int i = tid * E + r;
      k[r] = i < n_valid ? it_key<T>(srow[i], i) : 0u;
    }
#pragma unroll
    for (int kk = 2; kk <= N; kk <<= 1) {
#pragma unroll
      for (int j = kk >> 1; j > 0; j >>= 1) {
        if (j >= 32 * E) {
          const int tm = j / E;  // partner thread = tid ^ tm (another warp)
          xk[tid] = make_uint4(k[0], k[1], k[2], k[3]);
          __syncthreads();
          const uint4 o4 = xk[tid ^ tm];
          __syncthreads();
          const uint32_t o[E] = {o4.x, o4.y, o4.z, o4.w};
          const bool lower = (tid & tm) == 0;
#pragma unroll
          for (int r = 0; r < E; ++r) {
            const bool desc = ((tid * E + r) & kk) == 0;
            k[r] = (desc == lower) ? max(k[r], o[r]) : min(k[r], o[r]);
          }
        } else if (j >= E) {
          const int lm = j / E;
          const bool lower = (lane & lm) == 0;
#pragma unroll
          for (int r = 0; r < E; ++r) {
            const uint32_t o = __shfl_xor_sync(0xffffffffu, k[r], lm);
            const bool desc = ((tid * E + r) & kk) == 0;
            k[r] = (desc == lower) ? max(k[r], o) : min(k[r], o);
          }
        } else {
#pragma unroll
          for (int r = 0; r < E; ++r) {
            if (r & j) continue;
            const int r2 = r | j;
            const bool desc = ((tid * E + r) & kk) == 0;
            const uint32_t hi = max(k[r], k[r2]), lo = min(k[r], k[r2]);
            k[r] = desc ? hi : lo;
            k[r2] = desc ? lo : hi;
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < E; ++r) {
      const int rank = tid * E + r;
      if (rank < n_pick) out[rank] = static_cast<int32_t>(base + (0xffffu - (k[r] & 0xffffu)));
    }
  }
  for (int r = n_pick + tid; r < k_sel; r += 512) out[r] = static_cast<int32_t>(base + r);
}

bool csa_select_block_launch(const IndexerArgs& a, int rows, cudaStream_t st) {
  if (a.cu_seqlens || !a.scores || a.dtype == kF32 || a.max_comp_per_seq > 2048) return false;
  if (a.dtype == kBF16)
    csa_select_block_kernel<__nv_bfloat16><<<rows, 512, 0, st>>>(a);
  else
    csa_select_block_kernel<__half><<<rows, 512, 0, st>>>(a);
  return true;
}

// 2-D view [rows, cols] of a 16-bit tensor, box {64 columns, 128 rows}, 128-byte swizzle.
static int it_encode(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t row_stride) {
  const uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {static_cast<uint64_t>(row_stride * 2)};
  const uint32_t box[2] = {64, 128};
  const uint32_t es[2] = {1, 1};
  return encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, base, dims, strides, box, es, CU_TENSOR_MAP_SWIZZLE_128B);
}

int64_t csa_scores_ws_bytes(int64_t total_tokens, int max_comp_per_seq, int dtype) {
  const int64_t ld = (static_cast<int64_t>(max_comp_per_seq) + 127) / 128 * 128;
  return total_tokens * ld * (dtype == kF32 ? 4 : 2);
}

// Scores of the prefill rows on the tensor cores into a.ws; true when launched.
bool csa_scores_tc_launch(const IndexerArgs& a, cudaStream_t st, int64_t* ld_out, int* err) {
  *err = 0;
  if (!a.cu_seqlens || a.dtype == kF32 || !a.ws) return false;
  if (a.head_dim % 64 || a.head_dim > 1024) return false;
  if (a.ws_bytes < csa_scores_ws_bytes(a.total_tokens, a.max_comp_per_seq, a.dtype)) return false;
  if (a.sq[2] != 1 || a.sq[1] != a.head_dim || a.sq[0] % 8 || (reinterpret_cast<uintptr_t>(a.q) & 15)) return false;
  if (a.sck[2] != 1 || a.sck[1] != a.head_dim || a.sck[0] % 8 || (reinterpret_cast<uintptr_t>(a.ck) & 15))
    return false;
  if (a.sq[0] < static_cast<int64_t>(a.num_q_heads) * a.head_dim ||
      a.sck[0] < static_cast<int64_t>(a.num_kv_heads) * a.head_dim)
    return false;
  const int64_t ld = (static_cast<int64_t>(a.max_comp_per_seq) + 127) / 128 * 128;
  if ((ld / 128) > 65535) return false;
  CUtensorMap mq, mk;
  // the compressed rows a tile may touch past the last sequence's slots are
  // zero-filled by the tensor map (its row extent is the rows that exist)
  if ((*err = it_encode(&mq, a.q, a.total_tokens, static_cast<int64_t>(a.num_q_heads) * a.head_dim, a.sq[0])))
    return true;
  if ((*err = it_encode(&mk, a.ck, a.comp_rows, static_cast<int64_t>(a.num_kv_heads) * a.head_dim, a.sck[0])))
    return true;
  ScoreParams p{};
  p.cu = a.cu_seqlens;
  p.offs = a.comp_offsets;
  p.num_seqs = a.num_seqs;
  p.total_tokens = a.total_tokens;
  p.m = a.m;
  p.kblocks = a.head_dim / 64;
  p.qcol0 = (a.num_q_heads - 1) * a.head_dim;
  p.kcol0 = (a.num_kv_heads - 1) * a.head_dim;
  p.scores = a.ws;
  p.ld = ld;
  dim3 grid((a.total_tokens + 127) / 128, static_cast<unsigned>(ld / 128));
  if (a.dtype == kBF16) {
    if ((*err = ensure_smem_attr(reinterpret_cast<const void*>(csa_scores_tc_kernel<__nv_bfloat16>), it::kSmem)))
      return true;
    csa_scores_tc_kernel<__nv_bfloat16><<<grid, 192, it::kSmem, st>>>(mq, mk, p);
  } else {
    if ((*err = ensure_smem_attr(reinterpret_cast<const void*>(csa_scores_tc_kernel<__half>), it::kSmem)))
      return true;
    csa_scores_tc_kernel<__half><<<grid, 192, it::kSmem, st>>>(mq, mk, p);
  }
  *ld_out = ld;
  return true;
}

}  // namespace tak

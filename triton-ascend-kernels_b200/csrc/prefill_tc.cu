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
// Warp roles (320 threads):
//   warp 8      TMA producer: both Q tiles once, then K and V blocks of 128
//               rows into 2-stage rings (128-byte swizzle, 64-column boxes).
//   warp 9      TMEM allocator + single-thread tcgen05.mma issuer.  Per K/V
//               block j and tile t: PV_t(j) (TS-MMA: P read from TMEM, V from
//               smem, MN-major), then S_t(j+1) = Q_t K^T (SS-MMA, M=N=128)
//               once PV_t(j) has completed (S_t and P_t share TMEM columns).
//   warps 0-3   softmax of tile A, warps 4-7 softmax of tile B (thread = row =
//               TMEM lane): load S, mask only on boundary blocks, online max
//               with lazy rescaling (O and l rescaled only when the max grows
//               by more than 2^8), P = 2^(s - m) on the MUFU unit, packed to
//               16 bits back into the tile's S columns; epilogue
//               reads O, normalises, stores the row and its LSE.  While one
//               warpgroup runs its softmax the tensor core works on the other
//               tile.
// TMEM: O_A [0,128), O_B [128,256), S/P_A [256,384), S/P_B [384,512); with
// one tile (D = 256), O_A [0,256) and S/P_A [256,384).
#include "prefill_unit.cuh"

namespace tak {

template <typename T, int D>
__global__ void __launch_bounds__(320, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const PrefillTcParams p) {
  using C = pf::Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::BAROFF + pf::NBAR * 8);
  const int warp = threadIdx.x >> 5;
  if (warp == 9) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = *tmem_holder;
  // blockIdx.x = slot * H + h: the heads of one row block are adjacent (they
  // share K/V through L2) and the grid has no 65535 limit on row blocks
  const int h = static_cast<int>(blockIdx.x % static_cast<unsigned>(p.H));
  const int slot = static_cast<int>(blockIdx.x / static_cast<unsigned>(p.H));
  prefill_unit<T, D>(&tmQ, &tmK, &tmV, p, h, slot, smem, reinterpret_cast<uint64_t*>(smem + C::BAROFF), taddr);
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
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

// Tensor maps and parameters of the tensor-core prefill for head dim D.
template <int D>
static int prefill_tc_setup(const PrefillArgs& a, CUtensorMap* mq, CUtensorMap* mk, CUtensorMap* mv,
                            PrefillTcParams* pp) {
  using C = pf::Cfg<D>;
  const int64_t n_aligned = (static_cast<int64_t>(a.total_tokens) + C::ROWS - 1) / C::ROWS;
  if (int r = encode_tnd_map(mq, a.q, a.sq, a.total_tokens, a.num_q_heads, D)) return r;
  if (int r = encode_tnd_map(mk, a.k, a.sk, a.total_tokens, a.num_kv_heads, D)) return r;
  if (int r = encode_tnd_map(mv, a.v, a.sv, a.total_tokens, a.num_kv_heads, D)) return r;
  PrefillTcParams& p = *pp;
  p = PrefillTcParams{};
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
  return 0;
}

template <typename T, int D>
static int launch_prefill_tc(const PrefillArgs& a, cudaStream_t st) {
  using C = pf::Cfg<D>;
  CUtensorMap mq, mk, mv;
  PrefillTcParams p;
  if (int r = prefill_tc_setup<D>(a, &mq, &mk, &mv, &p)) return r;
  // one CTA per (row block, query head); the last row-block slot per head zeroes
  // the rows past the last sequence
  const dim3 grid(static_cast<unsigned>((static_cast<int64_t>(p.n_aligned) + a.num_seqs + 1) * a.num_q_heads));
  auto kern = prefill_tc_kernel<T, D>;
  if (const int r = ensure_smem_attr(reinterpret_cast<const void*>(kern), C::SMEM)) return r;
  kern<<<grid, 320, C::SMEM, st>>>(mq, mk, mv, p);
  note_kernel("prefill_tc");
  return 0;
}

static bool prefill_tc_ok(const PrefillArgs& a) {
  if (a.dtype == kF32 || a.head_dim != a.head_dim_v) return false;
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return false;
  if (!tma_ok(a.q, a.sq) || !tma_ok(a.k, a.sk) || !tma_ok(a.v, a.sv)) return false;
  if (a.so[2] != 1 || (a.so[0] % 8) || (a.so[1] % 8) || (reinterpret_cast<uintptr_t>(a.out) & 15)) return false;
  // the grid's one dimension holds (row blocks + sequences + 1) x heads CTAs
  const int rows = a.head_dim >= 256 ? pf::BM : 2 * pf::BM;
  const int64_t ctas = ((static_cast<int64_t>(a.total_tokens) + rows - 1) / rows + a.num_seqs + 1) * a.num_q_heads;
  return ctas <= 2147483647;
}

int prefill_tc_setup_d128(const PrefillArgs& a, CUtensorMap* mq, CUtensorMap* mk, CUtensorMap* mv,
                          PrefillTcParams* p) {
  if (a.head_dim != 128 || !a.total_tokens || !prefill_tc_ok(a)) return -1;
  return prefill_tc_setup<128>(a, mq, mk, mv, p);
}

int prefill_tc_launch(const PrefillArgs& a, cudaStream_t st, bool* handled) {
  *handled = false;
  if (!prefill_tc_ok(a)) return 0;
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

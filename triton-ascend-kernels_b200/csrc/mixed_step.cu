// A serving step's prefill and decode in ONE persistent launch.
//
// Work: the varlen prefill's (row block, query head) units -- the same
// longest-first order as prefill_tc.cu's grid -- and the paged decode's
// split-KV units, in one device work queue.  A grid of one CTA per SM pulls
// queue positions with an atomic counter.  Decode units are spread evenly
// through the queue (position u is decode iff floor((u + 1) D / N) >
// floor(u D / N) for D decode positions of N), so that while most SMs run the
// tensor-bound prefill a few stream KV pages: the HBM-bound decode overlaps
// the prefill instead of following it.
//
// A CTA has 320 threads and the prefill's shared-memory and TMEM layout
// (prefill_unit.cuh).  A decode position holds two decode units, run side by
// side by the two 160-thread halves of the CTA (warps 0-4 and 5-9), each on
// its own half of shared memory and its own named barriers -- as two decode
// CTAs would share an SM (decode_unit.cuh).  The split combine needs every
// split of a (sequence, KV head chunk): the split that finishes last (an
// arrival counter per pair, zeroed before the launch) merges them.
//
// Shapes: prefill head dim 128 on the tensor-core path, decode head dim 128
// with 64-row chunks (page size a multiple of 64) on the split-KV path, both
// 16-bit of the same type; anything else runs the two kernels back to back.
#include <cstdio>

#include "decode_unit.cuh"
#include "prefill_unit.cuh"

namespace tak {

struct MixedParams {
  int64_t n_pre;      // prefill units
  int64_t n_dec;      // decode positions (two decode units each)
  int64_t dec_units;  // decode units: max_splits x groups x sequences
  unsigned long long* queue;  // next queue position (zero before the launch)
  int* arrive;                // [sequences x groups] finished splits (zero before the launch)
  int max_splits, groups, H;
};

namespace mx {
constexpr int kDecNS = 3;  // ring stages of each decode half
using DS = DecodeSmem<128, 64, kDecNS>;
constexpr int kHalf = (DS::BYTES + 1023) / 1024 * 1024;  // second decode half starts here
constexpr int kDecBytes = kHalf + DS::BYTES;
constexpr int kPreTiles = pf::Cfg<128>::BAROFF;
// the prefill unit's barriers sit past both layouts' data, so a decode unit's
// ring never overlaps them
constexpr int kPreBars = ((kDecBytes > kPreTiles ? kDecBytes : kPreTiles) + 127) / 128 * 128;
constexpr int kSmem = kPreBars + pf::NBAR * 8 + 16 + 1024;
}  // namespace mx

template <typename T>
__global__ void __launch_bounds__(320, 1)
    mixed_step_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmKc,
                      const __grid_constant__ CUtensorMap tmVc, const PrefillTcParams pp, const DecodeParams dp,
                      const MixedParams mp) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t tmem_holder;
  __shared__ long long s_unit;
  __shared__ int s_last[2];
  __shared__ float s_wts[2][16 * 64];
  __shared__ float s_inv[2][16];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5;
  if (warp == 9) {
    tmem_alloc(&tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = tmem_holder;
  const int64_t total = mp.n_pre + mp.n_dec;
  for (;;) {
    if (tid == 0) s_unit = static_cast<long long>(atomicAdd(mp.queue, 1ull));
    __syncthreads();
    const int64_t u = s_unit;
    __syncthreads();
    if (u >= total) break;
    const int64_t k0 = u * mp.n_dec / total, k1 = (u + 1) * mp.n_dec / total;
    if (k1 > k0) {
      // ---------------- two decode units, one per 160-thread half ----------------
      const int half = warp >= 5 ? 1 : 0;
      const int ltid = tid - half * 160;
      const int64_t d = 2 * k0 + half;
      if (d < mp.dec_units) {
        const int split = static_cast<int>(d % mp.max_splits);
        const int64_t sy = d / mp.max_splits;
        const int y = static_cast<int>(sy % mp.groups);
        const int seq = static_cast<int>(sy / mp.groups);
        const int bar_all = 2 + half, bar_cons = 4 + half;
        const bool parts = decode_unit<T, 128, 64, mx::kDecNS>(&tmKc, &tmVc, dp, split, y, seq,
                                                               smem + half * mx::kHalf, ltid, bar_all, bar_cons);
        // the producer warp returns false at once; the 128 consumer threads agree
        if (parts) {
          __threadfence();  // this split's partials are visible before it is counted
          named_bar_sync(bar_cons, 128);
          if (ltid == 0) {
            const int ctx = min(dp.context_lens[seq], dp.max_ctx);
            const int split_tokens = dp.pages_per_split * dp.block_size;
            const int n_splits = (ctx + split_tokens - 1) / split_tokens;
            s_last[half] = atomicAdd(&mp.arrive[static_cast<int64_t>(seq) * mp.groups + y], 1) == n_splits - 1;
          }
          named_bar_sync(bar_cons, 128);
          if (s_last[half]) {
            __threadfence();
            decode_combine<T>(dp, seq, y, ltid, s_wts[half], s_inv[half], bar_cons);
          }
        }
      }
    } else {
      // ---------------- one prefill unit: the whole CTA ----------------
      const int64_t pu = u - k0;
      prefill_unit<T, 128>(&tmQ, &tmK, &tmV, pp, static_cast<int>(pu % mp.H), static_cast<int>(pu / mp.H), smem,
                           reinterpret_cast<uint64_t*>(smem + mx::kPreBars), taddr);
    }
    __syncthreads();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(taddr, 512);
  }
}

// Workspace of the mixed step: the decode's split partials (as
// paged_decode_workspace_bytes), then the queue counter and the split arrival
// counters (zeroed by the launcher before every launch).
size_t mixed_workspace_bytes(const PagedDecodeArgs& d) {
  if (d.num_kv_heads <= 0 || d.num_q_heads <= 0) return 0;
  const size_t part = (paged_decode_workspace_bytes(d) + 255) / 256 * 256;
  const int64_t groups = static_cast<int64_t>(d.num_kv_heads) * ((d.num_q_heads / d.num_kv_heads + 15) / 16);
  return part + 256 + 8 + static_cast<size_t>(d.num_seqs) * groups * 4;
}

int mixed_step_launch(const PrefillArgs& pa, const PagedDecodeArgs& da, cudaStream_t st) {
  CUtensorMap mq, mk, mv, mkc, mvc;
  PrefillTcParams pp;
  DecodeParams dp;
  int max_splits = 0, groups = 0;
  int rp = -1, rd = -1;
  if (pa.dtype == da.dtype && !pa.force_generic) {
    rp = prefill_tc_setup_d128(pa, &mq, &mk, &mv, &pp);
    if (rp > 0) return rp;
    if (rp == 0) {
      rd = decode_fast_setup_d128(da, &mkc, &mvc, &dp, &max_splits, &groups);
      if (rd > 0) return rd;
    }
  }
  if (da.workspace_bytes < mixed_workspace_bytes(da)) return set_error(2, "mixed step: workspace too small");
  if (rp != 0 || rd != 0) {
    // shapes the one-launch kernel does not take: the two kernels back to back
    if (const int r = prefill_launch(pa, st)) return r;
    if (const int r = check_launch("mixed step (prefill)")) return r;
    return paged_decode_launch(da, st);
  }
  uint8_t* counters = static_cast<uint8_t*>(da.workspace) + (paged_decode_workspace_bytes(da) + 255) / 256 * 256;
  counters = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(counters) + 255) & ~uintptr_t(255));
  MixedParams mp{};
  mp.n_pre = (static_cast<int64_t>(pp.n_aligned) + pa.num_seqs + 1) * pa.num_q_heads;
  mp.dec_units = static_cast<int64_t>(max_splits) * groups * da.num_seqs;
  mp.n_dec = (mp.dec_units + 1) / 2;
  mp.queue = reinterpret_cast<unsigned long long*>(counters);
  mp.arrive = reinterpret_cast<int*>(counters + 8);
  mp.max_splits = max_splits;
  mp.groups = groups;
  mp.H = pa.num_q_heads;
  const size_t clear = 8 + static_cast<size_t>(da.num_seqs) * groups * 4;
  if (cudaMemsetAsync(counters, 0, clear, st) != cudaSuccess) return set_error(3, "mixed step: clearing counters failed");
  auto kern = pa.dtype == kBF16 ? mixed_step_kernel<__nv_bfloat16> : mixed_step_kernel<__half>;
  if (const int r = ensure_smem_attr(reinterpret_cast<const void*>(kern), mx::kSmem)) return r;
  kern<<<num_sms(), 320, mx::kSmem, st>>>(mq, mk, mv, mkc, mvc, pp, dp, mp);
  note_kernel("mixed_step");
  return 0;
}

}  // namespace tak

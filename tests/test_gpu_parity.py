"""CUDA path vs the CPU oracle (and vs the reference's golden outputs).

Every test here calls the drop-in modules, which call libtak_b200.so through
its C ABI.  Tolerances: fp16/bf16 outputs max-abs <= 2e-2 of the float64
oracle (the bf16 rounding of an O(1) output is 4e-3), LSE <= 1e-3; fp32
outputs <= 1e-4; index tensors bit-exact.
"""

import json
import math
import os

import numpy as np
import pytest
import torch

import golden_inputs as gi
from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu

import _tak_b200 as T  # noqa: E402
import flash_attention_prefill as FP  # noqa: E402
import paged_attention_decode as PD  # noqa: E402
import sparse_attn_fwd as SA  # noqa: E402
import csa as CSA  # noqa: E402
import hca as HCA  # noqa: E402

DEV = "cuda"
TOL16 = 2e-2
TOL_LSE = 1e-3
TOL32 = 1e-4
HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
GOLD = np.load(os.path.join(HERE, "reference_golden.npz"))
CASES = sorted(json.load(open(os.path.join(HERE, "reference_golden_inputs.json")))["sha256"])


def npy(t):
    return t.detach().float().cpu().numpy()


def cu(x):
    return x.to(DEV) if isinstance(x, torch.Tensor) else x


def close(out, ref, tol):
    out = npy(out) if isinstance(out, torch.Tensor) else out
    err = np.abs(out.astype(np.float64) - ref).max() if out.size else 0.0
    assert err <= tol, f"max abs err {err:.3e} > {tol:.1e}"
    return err


def close_lse(lse, ref):
    lse = npy(lse)
    fin = np.isfinite(ref)
    assert (np.isfinite(lse) == fin).all()
    if fin.any():
        assert np.abs(lse[fin] - ref[fin]).max() <= TOL_LSE


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert T.read_device_error() == 0, "a kernel reported a timed-out wait"


@pytest.fixture(params=[0, 1], ids=["auto", "generic"])
def kernel_path(request):
    old = T.set_kernel_path(request.param)
    yield request.param
    T.set_kernel_path(old)


def assert_topk_match(got, ref, q, ck, base_of_row, n_win, ulp):
    """Index rows equal, except that two slots whose indexer scores differ by
    at most one rounding step of the score dtype may trade places (the CUDA
    kernel accumulates the dot product in fp32, the oracle in float64, so a
    score within one ulp of a rounding boundary can round either way)."""
    np.testing.assert_array_equal(got[:, :n_win], ref[:, :n_win])
    qn, ckn = q[:, -1, :].astype(np.float64), ck[:, -1, :].astype(np.float64)
    for t in np.nonzero((got != ref).any(1))[0]:
        a, b = got[t, n_win:], ref[t, n_win:]
        assert ((a >= 0) == (b >= 0)).all()
        base = base_of_row(t)
        sa = ckn[a[a >= 0] - base] @ qn[t]
        sb = ckn[b[b >= 0] - base] @ qn[t]
        tol = ulp * np.maximum(np.abs(sa), np.abs(sb)) + 1e-6
        assert (np.abs(sa - sb) <= tol).all(), f"row {t}: {a} vs {b}"


# ---------------------------------------------------------------------------
# reference runner configurations (golden fixtures)
# ---------------------------------------------------------------------------

def _golden(case, out):
    rows = GOLD[f"{case}/rows"]
    np.testing.assert_allclose(npy(out)[rows], GOLD[f"{case}/out"].astype(np.float64), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("case", [c for c in CASES if c.startswith("fp_")])
def test_golden_prefill(case, kernel_path):
    inp = {k: cu(v) for k, v in gi.case_inputs(case).items()}
    causal = case.endswith("c1")
    out, lse = FP.flash_attention_prefill(inp["q"], inp["k"], inp["v"], inp["cu_seqlens"], causal=causal,
                                          return_lse=True)
    ref, ref_lse = O.prefill(inp["q"].cpu(), inp["k"].cpu(), inp["v"].cpu(), gi.FP_CU, causal)
    close(out, ref, TOL16)
    close_lse(lse, ref_lse)
    _golden(case, out)


@pytest.mark.parametrize("case", [c for c in CASES if c.startswith("pd_")])
def test_golden_paged_decode(case, kernel_path):
    inp = {k: cu(v) for k, v in gi.case_inputs(case).items()}
    out, lse = PD.paged_attention_decode(inp["q"], inp["k_cache"], inp["v_cache"], inp["block_tables"],
                                         inp["context_lens"], gi.PD_BLOCK, 16, return_lse=True)
    ref, ref_lse = O.paged_decode(*(npy(inp[k]) for k in ("q", "k_cache", "v_cache")),
                                  inp["block_tables"].cpu(), inp["context_lens"].cpu(), gi.PD_BLOCK)
    close(out, ref, TOL16)
    close_lse(lse, ref_lse)
    _golden(case, out)


@pytest.mark.parametrize("case", [c for c in CASES if c.startswith("sap_")])
def test_golden_sparse_prefill(case, kernel_path):
    inp = {k: cu(v) for k, v in gi.case_inputs(case).items()}
    sink = inp.get("attn_sink")
    out, lse = SA.sparse_attn_prefill(inp["q"], inp["k"], inp["v"], inp["topk_idxs"], inp["cu_seqlens"], sink,
                                      return_lse=True)
    ref, ref_lse = O.sparse_prefill(inp["q"].cpu(), inp["k"].cpu(), inp["v"].cpu(), inp["topk_idxs"].cpu(),
                                    None, None if sink is None else sink.cpu())
    close(out, ref, TOL16)
    close_lse(lse, ref_lse)
    _golden(case, out)


@pytest.mark.parametrize("case", [c for c in CASES if c.startswith("sad_")])
def test_golden_sparse_decode(case, kernel_path):
    inp = {k: cu(v) for k, v in gi.case_inputs(case).items()}
    sink = inp.get("attn_sink")
    args = [inp[k] for k in ("q", "k_cache", "v_cache", "compressed_k", "compressed_v", "block_tables",
                             "topk_idxs", "context_lens")]
    out, lse = SA.sparse_attn_decode(*args, num_win=gi.SA_NWIN_D, block_size=gi.SA_BLOCK, attn_sink=sink,
                                     return_lse=True)
    ref, ref_lse = O.sparse_decode(*(a.cpu() for a in args), gi.SA_NWIN_D, gi.SA_BLOCK,
                                   None if sink is None else sink.cpu())
    close(out, ref, TOL16)
    close_lse(lse, ref_lse)
    _golden(case, out)


@pytest.mark.parametrize("case", [c for c in CASES if c.startswith("csap_")])
def test_golden_csa_prefill(case):
    inp = {k: cu(v) for k, v in gi.case_inputs(case).items()}
    q, k, v, cuq = inp["q"], inp["k"], inp["v"], inp["cu_seqlens"]
    ck, cv, offs = CSA.compress_kv_overlap(k, v, cuq, gi.CSA_M)
    np.testing.assert_array_equal(offs.cpu().numpy(), GOLD[f"{case}/comp_offsets"])
    np.testing.assert_allclose(npy(ck), GOLD[f"{case}/ck"].astype(np.float64), atol=2e-3, rtol=2e-3)
    np.testing.assert_allclose(npy(cv), GOLD[f"{case}/cv"].astype(np.float64), atol=2e-3, rtol=2e-3)
    idx = CSA.build_csa_topk_idxs(q, ck, cuq, offs, gi.CSA_NWIN_P, gi.CSA_TOPK, gi.CSA_M)
    mine = O.build_csa_topk_idxs(q.cpu(), npy(ck), gi.SA_CU, offs.cpu(), gi.CSA_NWIN_P, gi.CSA_TOPK, gi.CSA_M,
                                 "float16")
    Tn = q.shape[0]      # entries are Tn + global compressed row
    assert_topk_match(idx.cpu().numpy(), mine, npy(q), npy(ck), lambda t: Tn, gi.CSA_NWIN_P, 2.0 ** -10)
    out = CSA.csa_prefill_forward(q, k, v, cuq, gi.CSA_NWIN_P, gi.CSA_TOPK, gi.CSA_M, inp.get("attn_sink"))
    kf = np.concatenate([npy(k), npy(ck)], 0)
    vf = np.concatenate([npy(v), npy(cv)], 0)
    sink = inp.get("attn_sink")
    ref, _ = O.sparse_prefill(q.cpu(), kf, vf, mine, None, None if sink is None else sink.cpu())
    close(out, ref, TOL16)


@pytest.mark.parametrize("case", [c for c in CASES if c.startswith("hcap_")])
def test_golden_hca_prefill(case):
    inp = {k: cu(v) for k, v in gi.case_inputs(case).items()}
    q, k, v, cuq = inp["q"], inp["k"], inp["v"], inp["cu_seqlens"]
    ck, cv, offs = HCA.compress_kv_simple(k, v, cuq, gi.HCA_M)
    np.testing.assert_allclose(npy(ck), GOLD[f"{case}/ck"].astype(np.float64), atol=2e-3, rtol=2e-3)
    idx = HCA.build_hca_topk_idxs(cuq, offs, q.shape[0], gi.HCA_NWIN, gi.HCA_M)
    np.testing.assert_array_equal(idx.cpu().numpy(), GOLD[f"{case}/topk_idxs"])
    out = HCA.hca_prefill_forward(q, k, v, cuq, gi.HCA_NWIN, gi.HCA_M, inp.get("attn_sink"))
    _golden(case, out)


@pytest.mark.parametrize("case", [c for c in CASES if c.startswith("csad_")])
def test_golden_csa_decode(case):
    inp = {k: cu(v) for k, v in gi.case_inputs(case).items()}
    args = [inp[k] for k in ("q", "k_cache", "v_cache", "block_tables", "context_lens")]
    out = CSA.csa_decode_forward(*args, gi.CSA_NWIN_D, gi.CSA_TOPK, gi.CSA_M, gi.SA_BLOCK, inp.get("attn_sink"))
    _golden(case, out)
    sink = inp.get("attn_sink")
    ref, _, _ = O.csa_decode_forward(*(a.cpu() for a in args), gi.CSA_NWIN_D, gi.CSA_TOPK, gi.CSA_M, gi.SA_BLOCK,
                                     None if sink is None else sink.cpu(), "float16")
    close(out, ref, TOL16)


@pytest.mark.parametrize("case", [c for c in CASES if c.startswith("hcad_")])
def test_golden_hca_decode(case):
    inp = {k: cu(v) for k, v in gi.case_inputs(case).items()}
    args = [inp[k] for k in ("q", "k_cache", "v_cache", "block_tables", "context_lens")]
    out = HCA.hca_decode_forward(*args, gi.HCA_NWIN, gi.HCA_M, gi.SA_BLOCK, inp.get("attn_sink"))
    _golden(case, out)


# ---------------------------------------------------------------------------
# benchmark-shaped configurations and edge cases
# ---------------------------------------------------------------------------

def _cu_t(lens):
    return torch.tensor([0] + np.cumsum(lens).tolist(), dtype=torch.int32, device=DEV)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("causal", [True, False])
def test_prefill_varlen_gqa(dtype, causal, kernel_path):
    """Varlen prefill, lengths {17,128,300,511}, 8 q heads / 2 KV heads, d=128."""
    lens = [17, 128, 300, 511]
    g = torch.Generator().manual_seed(0)
    Tn = sum(lens)
    q = torch.randn(Tn, 8, 128, generator=g).to(DEV, dtype)
    k = torch.randn(Tn, 2, 128, generator=g).to(DEV, dtype)
    v = torch.randn(Tn, 2, 128, generator=g).to(DEV, dtype)
    out, lse = FP.flash_attention_prefill(q, k, v, _cu_t(lens), causal, return_lse=True)
    ref, ref_lse = O.prefill(npy(q), npy(k), npy(v), [0] + np.cumsum(lens).tolist(), causal)
    close(out, ref, TOL32 if dtype == torch.float32 else TOL16)
    close_lse(lse, ref_lse)
    assert out.dtype == dtype


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [True, False])
def test_prefill_edge_lengths(D, causal, kernel_path):
    """Empty sequences, length-1 sequences, a 129-row sequence (one row past a
    128-row tile), sequences starting off the 128-row grid, trailing tokens
    outside every sequence, strided q (last dim contiguous)."""
    lens = [0, 1, 129, 0, 64, 1, 300, 127]
    Tn = sum(lens) + 3
    g = torch.Generator().manual_seed(1)
    qb = torch.randn(Tn, 4, 2, D, generator=g).to(DEV, torch.bfloat16)
    q = qb[:, :, 0, :]                                  # non-contiguous
    k = torch.randn(Tn, 1, D, generator=g).to(DEV, torch.bfloat16)
    v = torch.randn(Tn, 1, D, generator=g).to(DEV, torch.bfloat16)
    cuq = _cu_t(lens)
    out, lse = FP.flash_attention_prefill(q, k, v, cuq, causal, return_lse=True)
    ref, ref_lse = O.prefill(npy(q), npy(k), npy(v), cuq.cpu(), causal)
    close(out, ref, TOL16)
    close_lse(lse, ref_lse)
    assert (npy(out)[-3:] == 0).all()


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_prefill_head_dims_take_tensor_cores(D, causal, dtype):
    """Every power-of-two head dim the tensor-core prefill takes (64, 128,
    256; the reference's HEAD_DIM is a free constexpr, FP:24,49) runs on the
    tcgen05 kernel -- asserted through tak_last_kernel() -- and matches the
    oracle: ragged lengths past several 128- and 256-row blocks, GQA 8/2."""
    lens = [1, 129, 300, 0, 1000, 2100]
    Tn = sum(lens)
    g = torch.Generator().manual_seed(7 + D)
    q = torch.randn(Tn, 8, D, generator=g).to(DEV, dtype)
    k = torch.randn(Tn, 2, D, generator=g).to(DEV, dtype)
    v = torch.randn(Tn, 2, D, generator=g).to(DEV, dtype)
    out, lse = FP.flash_attention_prefill(q, k, v, _cu_t(lens), causal, return_lse=True)
    assert T.last_kernel() == "prefill_tc"
    ref, ref_lse = O.prefill(npy(q), npy(k), npy(v), [0] + np.cumsum(lens).tolist(), causal, acc=np.float32)
    close(out, ref, TOL16)
    close_lse(lse, ref_lse)


def _paged_case(B, H, Hkv, D, P, max_ctx, pool, dtype, seed, ctx=None):
    g = torch.Generator().manual_seed(seed)
    if ctx is None:
        ctx = torch.randint(1, max_ctx + 1, (B,), generator=g)
    ctx = torch.as_tensor(ctx, dtype=torch.int32)
    maxb = (max_ctx + P - 1) // P
    pool = max(pool, int(((ctx + P - 1) // P).sum()) + 3)
    perm = torch.randperm(pool, generator=g).to(torch.int32)
    bt = torch.zeros(B, maxb, dtype=torch.int32)
    i = 0
    for b in range(B):
        for j in range((int(ctx[b]) + P - 1) // P):
            bt[b, j] = perm[i]
            i += 1
    kc = torch.randn(pool, Hkv, P, D, generator=g).to(DEV, dtype)
    vc = torch.randn(pool, Hkv, P, D, generator=g).to(DEV, dtype)
    q = torch.randn(B, H, D, generator=g).to(DEV, dtype)
    return q, kc, vc, bt.to(DEV), ctx.to(DEV)


@pytest.mark.parametrize("P", [16, 64, 128])
@pytest.mark.parametrize("G", [1, 4, 8])
def test_paged_decode_shapes(P, G, kernel_path):
    """Batch 12, 32 query heads, head_dim 128, bf16, contexts up to 1500
    (several splits), including ctx 1, ctx = P and ctx = 0."""
    B, H = 12, 32
    ctx = [1, P, P + 1, 1500, 777, 0, 3 * P, 1024, 5, 1499, 64, 250]
    q, kc, vc, bt, cl = _paged_case(B, H, H // G, 128, P, 1500, 200, torch.bfloat16, 3, ctx)
    out, lse = PD.paged_attention_decode(q, kc, vc, bt, cl, P, min(P, 16), return_lse=True)
    ref, ref_lse = O.paged_decode(npy(q), npy(kc), npy(vc), bt.cpu(), cl.cpu(), P)
    close(out, ref, TOL16)
    close_lse(lse, ref_lse)


@pytest.mark.parametrize("split_pages", [1, 2, 64])
def test_paged_decode_split_invariance(split_pages):
    """The split-KV partition must not change the result beyond rounding."""
    q, kc, vc, bt, cl = _paged_case(8, 32, 8, 128, 128, 4096, 300, torch.bfloat16, 5)
    out = PD.paged_attention_decode(q, kc, vc, bt, cl, 128, 16, split_pages=split_pages)
    ref, _ = O.paged_decode(npy(q), npy(kc), npy(vc), bt.cpu(), cl.cpu(), 128)
    close(out, ref, TOL16)


def test_paged_decode_fp32_and_stale_tail():
    """fp32 cache (generic kernel); and NaN garbage in the unused tail rows of
    the last page must not leak into the bf16 fast path."""
    q, kc, vc, bt, cl = _paged_case(4, 8, 2, 128, 16, 200, 64, torch.float32, 7, [13, 35, 200, 1])
    out = PD.paged_attention_decode(q, kc, vc, bt, cl, 16, 16)
    ref, _ = O.paged_decode(npy(q), npy(kc), npy(vc), bt.cpu(), cl.cpu(), 16)
    close(out, ref, TOL32)
    q, kc, vc, bt, cl = _paged_case(4, 8, 2, 128, 64, 300, 64, torch.bfloat16, 8, [13, 65, 300, 1])
    ref, _ = O.paged_decode(npy(q), npy(kc), npy(vc), bt.cpu(), cl.cpu(), 64)
    for b, c in enumerate(cl.cpu().tolist()):
        last = int(bt[b, (c - 1) // 64])
        kc[last, :, c % 64 or 64:, :] = float("nan")
        vc[last, :, c % 64 or 64:, :] = float("nan")
    out = PD.paged_attention_decode(q, kc, vc, bt, cl, 64, 16)
    close(out, ref, TOL16)


def test_paged_decode_bench_shape_sample():
    """The decode bench shape (batch 64, 32/8 heads, d=128, page 128, pool 5000,
    ctx U[1,8192]) -- checked against the oracle on 6 of the 64 requests."""
    q, kc, vc, bt, cl = _paged_case(64, 32, 8, 128, 128, 8192, 5000, torch.bfloat16, 11)
    out, lse = PD.paged_attention_decode(q, kc, vc, bt, cl, 128, 128, return_lse=True)
    pick = [0, 1, 17, 33, 50, 63]
    idx = torch.tensor(pick, device=DEV)
    ref, ref_lse = O.paged_decode(npy(q[idx]), npy(kc), npy(vc), bt[idx].cpu(), cl[idx].cpu(), 128, acc=np.float32)
    close(out[idx], ref, TOL16)
    close_lse(lse[idx], ref_lse)


def _sparse_case(Tn, H, Hkv, D, Dv, rows, K, dtype, seed, shared_latent=False, pad=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(Tn, H, D, generator=g).to(DEV, dtype)
    k = torch.randn(rows, Hkv, D, generator=g).to(DEV, dtype)
    v = k[..., :Dv] if shared_latent else torch.randn(rows, Hkv, Dv, generator=g).to(DEV, dtype)
    idx = torch.stack([torch.randperm(rows, generator=g)[:K] for _ in range(Tn)]).sort(1).values.to(torch.int32)
    if pad:
        for t in range(0, Tn, 3):
            idx[t, (t * 7) % K:] = -1        # ragged -1 padding, one fully masked row
        idx[1, :] = -1
    sink = torch.randn(H, generator=g).to(DEV)
    return q, k, v, idx.to(DEV), sink


@pytest.mark.parametrize("with_sink", [False, True])
def test_sparse_prefill_mla_shape(with_sink, kernel_path):
    """The sparse bench shape at small size: 64 query heads sharing 1 KV head,
    Dqk 576 (512 latent + 64 rope), Dv 512 with v a view of k's first 512
    dims, 256 indices per token with -1 padding and a fully masked row."""
    q, k, v, idx, sink = _sparse_case(24, 64, 1, 576, 512, 1500, 256, torch.bfloat16, 21, shared_latent=True)
    s = sink if with_sink else None
    out, lse = SA.sparse_attn_prefill(q, k, v, idx, None, s, return_lse=True)
    ref, ref_lse = O.sparse_prefill(npy(q), npy(k), npy(v), idx.cpu(), None, None if s is None else s.cpu())
    close(out, ref, TOL16)
    close_lse(lse, ref_lse)


@pytest.mark.parametrize("H", [64, 128])
def test_sparse_prefill_persistent_units(H):
    """More (token, head group) units than SMs, so every persistent CTA walks
    several units through one K ring (each unit's Q, then its tiles): the
    576/512 latent kernel of the sparse bench with 64 heads (one unit per
    token) and with 128 heads on one KV head (two 64-row units per token).
    160 indices per token (three tiles, the last one ragged), -1 padding and
    a fully masked row."""
    q, k, v, idx, sink = _sparse_case(330, H, 1, 576, 512, 1200, 160, torch.bfloat16, 71 + H, shared_latent=True)
    out, lse = SA.sparse_attn_prefill(q, k, v, idx, None, sink, return_lse=True)
    assert T.last_kernel() == "sparse_tc"
    ref, ref_lse = O.sparse_prefill(npy(q), npy(k), npy(v), idx.cpu(), None, sink.cpu())
    close(out, ref, TOL16)
    close_lse(lse, ref_lse)


@pytest.mark.parametrize("variant", ["576v512_shared", "576v576_shared", "576v576_sep", "576v512_sep",
                                     "512v512_shared", "512v512_sep", "256v256_sep"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_sparse_prefill_tensor_core_variants(variant, dtype):
    """Every K/V head-dim pairing the tensor-core sparse kernel takes --
    V a prefix view of K (the MLA latent: 576/512, 512/512, and V = K itself
    at 576, the call the reference's own shape rule k.shape == v.shape makes,
    SA:279) and V a tensor of its own (576/576, 576/512, 512/512, 256/256) --
    runs on the tcgen05 kernel (tak_last_kernel()) and matches the oracle.
    Ragged -1 padding and a fully masked row; 64 heads on one KV head."""
    dq, dv = (int(x) for x in variant.split("_")[0].split("v"))
    shared = variant.endswith("shared")
    H, Hkv = (64, 1) if dq >= 512 else (16, 2)
    q, k, v, idx, sink = _sparse_case(20, H, Hkv, dq, dv, 900, 200, dtype, 27 + dq + dv, shared_latent=shared)
    out, lse = SA.sparse_attn_prefill(q, k, v, idx, None, sink, return_lse=True)
    assert T.last_kernel() == "sparse_tc"
    ref, ref_lse = O.sparse_prefill(npy(q), npy(k), npy(v), idx.cpu(), None, sink.cpu())
    close(out, ref, TOL16)
    close_lse(lse, ref_lse)


@pytest.mark.parametrize("variant", ["latent576", "sep512", "gqa128"])
def test_sparse_prefill_two_sources(variant, kernel_path):
    """Attention over [K | compressed K] read in place from the two tensors
    (the CSA / HCA forwards' layout, CSA:191-192) equals attention over their
    concatenation: indices on both sides of the boundary, -1 and indices past
    both sources."""
    if variant == "latent576":
        H, Hkv, D, Dv, shared = 64, 1, 576, 512, True
    elif variant == "sep512":
        H, Hkv, D, Dv, shared = 64, 1, 512, 512, False
    else:
        H, Hkv, D, Dv, shared = 16, 2, 128, 128, False
    rows1, rows2 = 700, 300
    q, k, v, idx, sink = _sparse_case(18, H, Hkv, D, Dv, rows1 + rows2, 160, torch.bfloat16, 61, shared_latent=shared)
    idx[4, 7] = rows1 + rows2 + 5     # past both sources: masked
    k1, k2 = k[:rows1], k[rows1:].clone()
    if shared:
        v1, v2 = k1[..., :Dv], k2[..., :Dv]
    else:
        v1, v2 = v[:rows1], v[rows1:].clone()
    out, lse = SA.sparse_attn_prefill_two_sources(q, k1, v1, k2, v2, idx, sink, return_lse=True)
    if kernel_path == 0:
        assert T.last_kernel() == "sparse_tc"
    vfull = torch.cat([v1, v2], 0)
    ref, ref_lse = O.sparse_prefill(npy(q), npy(torch.cat([k1, k2], 0)), npy(vfull), idx.cpu(), None, sink.cpu())
    close(out, ref, TOL16)
    close_lse(lse, ref_lse)


def test_csa_forward_separate_v_on_tensor_cores():
    """csa_prefill_forward with K and V of their own (512-dim, 64 heads): the
    attention over [K | compressed K] and [V | compressed V] runs on the
    tensor-core kernel and matches the oracle's forward."""
    lens = [300, 700]
    Tn = sum(lens)
    g = torch.Generator().manual_seed(62)
    q = torch.randn(Tn, 64, 512, generator=g).to(DEV, torch.bfloat16)
    k = torch.randn(Tn, 1, 512, generator=g).to(DEV, torch.bfloat16)
    v = torch.randn(Tn, 1, 512, generator=g).to(DEV, torch.bfloat16)
    sink = torch.randn(64, generator=g).to(DEV)
    cuq = _cu_t(lens)
    out = CSA.csa_prefill_forward(q, k, v, cuq, 64, 32, 4, sink)
    assert T.last_kernel() == "sparse_tc"
    ref, _, _ = O.csa_prefill_forward(npy(q), npy(k), npy(v), cuq.cpu(), 64, 32, 4, sink.cpu(), "bfloat16")
    close(out, ref, TOL16)


def test_sparse_prefill_wide_index_rows():
    """The sparse bench's index width: 2048 sorted unique indices per token drawn causally
    from a 32768-row latent KV (MQA, 64 heads, 576/512), -1 padding for early
    positions; 16 tokens checked against the oracle."""
    g = torch.Generator().manual_seed(23)
    rows, K, Tn = 32768, 2048, 16
    q = torch.randn(Tn, 64, 576, generator=g).to(DEV, torch.bfloat16)
    k = torch.randn(rows, 1, 576, generator=g).to(DEV, torch.bfloat16)
    pos = torch.tensor([100, 2047, 2048, 5000] + list(range(28000, 28012)))
    idx = torch.full((Tn, K), -1, dtype=torch.int32)
    for t in range(Tn):
        n = min(K, int(pos[t]) + 1)
        idx[t, :n] = torch.randperm(int(pos[t]) + 1, generator=g)[:n].sort().values.to(torch.int32)
    idx = idx.to(DEV)
    sink = torch.randn(64, generator=g).to(DEV)
    out, lse = SA.sparse_attn_prefill(q, k, k[..., :512], idx, None, sink, return_lse=True)
    ref, ref_lse = O.sparse_prefill(npy(q), npy(k), npy(k[..., :512]), idx.cpu(), None, sink.cpu(), acc=np.float32)
    close(out, ref, TOL16)
    close_lse(lse, ref_lse)


def test_sparse_prefill_gqa_fp32_and_oob():
    q, k, v, idx, sink = _sparse_case(40, 8, 2, 128, 128, 300, 64, torch.float32, 22)
    idx[5, 3] = 10_000            # past the last row: masked
    out = SA.sparse_attn_prefill(q, k, v, idx, None, sink)
    ref, _ = O.sparse_prefill(npy(q), npy(k), npy(v), idx.cpu(), None, sink.cpu())
    close(out, ref, TOL32)


def _sparse_decode_case(ctx, H, Hkv, D, Dv, P, n_win, n_comp_slots, ncomp, dtype, seed, shared_latent=False):
    """Paged window + compressed rows for sparse decode, with index rows that
    exercise the slot-position rule: window slots hold the last n_win logical
    positions (negative ones masked) plus one position == ctx (masked) and one
    -1; compressed slots hold ctx + row for sorted random rows, plus one index
    below ctx (masked in a compressed slot), one past the last compressed row
    and -1 padding."""
    g = torch.Generator().manual_seed(seed)
    B = len(ctx)
    maxb = max((max(ctx) + P - 1) // P, 1)
    pool = sum((c + P - 1) // P for c in ctx) + 5
    perm = torch.randperm(pool, generator=g).to(torch.int32)
    bt = torch.zeros(B, maxb, dtype=torch.int32)
    i = 0
    for b, c in enumerate(ctx):
        for j in range((c + P - 1) // P):
            bt[b, j] = perm[i]
            i += 1
    kc = torch.randn(pool, Hkv, P, D, generator=g).to(DEV, dtype)
    ck = torch.randn(ncomp, Hkv, D, generator=g).to(DEV, dtype)
    if shared_latent:
        vc, cv = kc[..., :Dv], ck[..., :Dv]
    else:
        vc = torch.randn(pool, Hkv, P, Dv, generator=g).to(DEV, dtype)
        cv = torch.randn(ncomp, Hkv, Dv, generator=g).to(DEV, dtype)
    q = torch.randn(B, H, D, generator=g).to(DEV, dtype)
    idx = torch.full((B, n_win + n_comp_slots), -1, dtype=torch.int32)
    for b, c in enumerate(ctx):
        idx[b, :n_win] = torch.arange(c - n_win, c, dtype=torch.int32)
        if b % 3 == 1:
            idx[b, n_win // 2] = c          # position == ctx: masked
            idx[b, n_win // 3] = -1
        n_here = (b * 37) % (n_comp_slots + 1)
        rows = torch.randperm(ncomp, generator=g)[:n_here].sort().values.to(torch.int32)
        idx[b, n_win:n_win + rows.numel()] = c + rows
        if b % 4 == 2 and n_here > 2:
            idx[b, n_win] = c - 1            # below ctx in a compressed slot: masked
            idx[b, n_win + n_here - 1] = c + ncomp  # past the compressed rows: masked
    sink = torch.randn(H, generator=g).to(DEV)
    cl = torch.tensor(ctx, dtype=torch.int32)
    return q, kc, vc, ck, cv, bt.to(DEV), idx.to(DEV), cl.to(DEV), sink


@pytest.mark.parametrize("shape", ["latent576", "latent512", "gqa128", "gqa64", "sep512", "latent576v576"])
@pytest.mark.parametrize("with_sink", [False, True])
def test_sparse_decode_paged_and_compressed(shape, with_sink, kernel_path):
    """Sparse decode over a paged window plus compressed rows: 64 heads sharing
    one latent KV head (Dqk 576 or 512, V a view of K), and GQA with 128- and
    64-dim heads; ragged index rows (slot counts not a multiple of 64), empty
    and short contexts, and every masking case of the slot-position rule."""
    ctx = [0, 1, 5, 127, 128, 3 * 64 + 7, 9 * 64, 1000, 33, 2]
    if shape == "latent576v576":      # V = K itself (the reference's k.shape == v.shape call)
        case = _sparse_decode_case(ctx, 64, 1, 576, 576, 64, 128, 200, 700, torch.bfloat16, 54, shared_latent=True)
        n_win = 128
    elif shape == "sep512":           # compressed K and V of their own (pooled separately)
        case = _sparse_decode_case(ctx, 64, 1, 512, 512, 64, 128, 200, 700, torch.bfloat16, 55)
        n_win = 128
    elif shape.startswith("latent"):
        D = int(shape[6:])
        case = _sparse_decode_case(ctx, 64, 1, D, 512, 64, 128, 200, 700, torch.bfloat16, 51, shared_latent=True)
        n_win = 128
    elif shape == "gqa128":
        case = _sparse_decode_case(ctx, 16, 4, 128, 128, 16, 40, 90, 300, torch.float16, 52)
        n_win = 40
    else:
        case = _sparse_decode_case(ctx, 8, 2, 64, 64, 32, 70, 30, 120, torch.bfloat16, 53)
        n_win = 70
    q, kc, vc, ck, cv, bt, idx, cl, sink = case
    P = kc.shape[2]
    s = sink if with_sink else None
    out, lse = SA.sparse_attn_decode(q, kc, vc, ck, cv, bt, idx, cl, n_win, P, s, return_lse=True)
    if kernel_path == 0:
        assert T.last_kernel() == "sparse_tc"
    ref, ref_lse = O.sparse_decode(npy(q), npy(kc), npy(vc), npy(ck), npy(cv), bt.cpu(), idx.cpu(), cl.cpu(),
                                   n_win, P, None if s is None else s.cpu())
    close(out, ref, TOL16)
    close_lse(lse, ref_lse)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("gated", [False, True])
def test_compress_csa_hca(dtype, gated):
    lens = [0, 3, 4, 5, 130, 257, 1]
    Tn = sum(lens)
    g = torch.Generator().manual_seed(31)
    k = torch.randn(Tn, 2, 128, generator=g).to(DEV, dtype)
    v = torch.randn(Tn, 2, 128, generator=g).to(DEV, dtype)
    gate = torch.randn(Tn, generator=g).to(DEV) if gated else None
    cuq = _cu_t(lens)
    for fn, stride, window in ((CSA.compress_kv_overlap, 4, 8), (HCA.compress_kv_simple, 128, 128)):
        ck, cv, offs = fn(k, v, cuq, stride, gate=gate)
        rk, rv, roffs = O.compress_kv(npy(k), npy(v), cuq.cpu(), stride, window,
                                      None if gate is None else gate.cpu())
        np.testing.assert_array_equal(offs.cpu().numpy(), roffs)
        close(ck, rk, 1e-2)
        close(cv, rv, 1e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("gated", [False, True])
@pytest.mark.parametrize("shape", ["ragged", "latent512", "heads2x256", "strided", "m3"])
def test_compress_csa_hca_one_pass(dtype, gated, shape):
    """CSA + HCA pooling of the same K/V in one launch vs the oracle's two
    separate poolings: ragged lengths (empty, shorter than m, chunk-straddling
    tails), 512-dim latent rows, two KV heads of 256-dim K and V (1 KB rows:
    the block-pair path of the bulk kernel on a multi-head grid), a strided
    K/V view, and m = 3 (m' = 128 not a multiple of m: the two-pass path)."""
    g = torch.Generator().manual_seed(71)
    m, mp, hkv, D, Dv = 4, 128, 2, 128, 256
    if shape == "latent512":
        lens, hkv, D, Dv = [4096, 77, 4096], 1, 512, 512
    elif shape == "heads2x256":
        lens, hkv, D, Dv = [300, 0, 1, 1030, 129], 2, 256, 256
    else:
        lens = [0, 3, 4, 5, 130, 257, 1, 0, 132]
    if shape == "m3":
        m = 3
    Tn = sum(lens)
    if shape == "strided":
        big = torch.randn(Tn, hkv, 2 * D + Dv, generator=g).to(DEV, dtype)
        k, v = big[:, :, :D], big[:, :, 2 * D:]
    else:
        k = torch.randn(Tn, hkv, D, generator=g).to(DEV, dtype)
        v = torch.randn(Tn, hkv, Dv, generator=g).to(DEV, dtype)
    gate = torch.randn(Tn, generator=g).to(DEV) if gated else None
    cuq = _cu_t(lens)
    (ck, cv, co), (hk, hv, ho) = CSA.compress_kv_csa_hca(k, v, cuq, m, mp, gate=gate)
    if dtype != torch.float32 and shape != "m3":
        # 16-bit rows with m' a multiple of m take the one-pass bulk-copy kernel
        assert T.last_kernel() == "compress_dual"
    gnp = None if gate is None else gate.cpu()
    for (gk, gv, go), (stride, window) in (((ck, cv, co), (m, 2 * m)), ((hk, hv, ho), (mp, mp))):
        rk, rv, roffs = O.compress_kv(npy(k), npy(v), cuq.cpu(), stride, window, gnp)
        np.testing.assert_array_equal(go.cpu().numpy(), roffs)
        close(gk, rk, 1e-2)
        close(gv, rv, 1e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("one_pass", [True, False])
def test_compress_masked_gates(dtype, one_pass):
    """Gate logits of -inf mask their rows: a partly masked window pools its
    other rows, a window (here also a whole HCA slot and a whole short
    sequence) with every row masked pools to zeros -- in the one-pass
    compressor, in the separate CSA and HCA compressors and in the oracle."""
    lens = [300, 9, 256, 131]
    Tn = sum(lens)
    g = torch.Generator().manual_seed(91)
    k = torch.randn(Tn, 1, 512, generator=g).to(DEV, dtype)
    v = torch.randn(Tn, 1, 512, generator=g).to(DEV, dtype)
    gate = torch.randn(Tn, generator=g)
    ninf = float("-inf")
    gate[0:8] = ninf               # the first CSA window of sequence 0, entirely
    gate[20] = ninf                # single rows
    gate[50:53] = ninf
    gate[300:309] = ninf           # all of sequence 1
    gate[309:309 + 128] = ninf     # the first HCA slot of sequence 2
    gate[Tn - 1] = ninf
    gate = gate.to(DEV)
    cuq = _cu_t(lens)
    if one_pass:
        (ck, cv, co), (hk, hv, ho) = CSA.compress_kv_csa_hca(k, v, cuq, 4, 128, gate=gate)
    else:
        ck, cv, co = CSA.compress_kv_overlap(k, v, cuq, 4, gate=gate)
        hk, hv, ho = HCA.compress_kv_simple(k, v, cuq, 128, gate=gate)
    tol = TOL32 if dtype == torch.float32 else 1e-2
    for (gk, gv, go), (stride, window) in (((ck, cv, co), (4, 8)), ((hk, hv, ho), (128, 128))):
        rk, rv, roffs = O.compress_kv(npy(k), npy(v), cuq.cpu(), stride, window, gate.cpu())
        np.testing.assert_array_equal(go.cpu().numpy(), roffs)
        assert torch.isfinite(gk).all() and torch.isfinite(gv).all()
        close(gk, rk, tol)
        close(gv, rv, tol)
    assert float(ck[0].abs().max()) == 0.0 and float(hk[3].abs().max()) == 0.0  # all-masked windows


def test_compress_paged_matches_tnd():
    q, kc, vc, bt, cl = _paged_case(5, 8, 2, 128, 16, 300, 120, torch.bfloat16, 33, [0, 17, 300, 64, 1])
    ck, cv, offs, lens, _ = T.compress_paged(kc, vc, bt, cl, 16, 4, 8)
    kt, cut = O.gather_paged_to_tnd(npy(kc), bt.cpu(), cl.cpu(), 16)
    vt, _ = O.gather_paged_to_tnd(npy(vc), bt.cpu(), cl.cpu(), 16)
    rk, rv, roffs = O.compress_kv(kt, vt, cut, 4, 8)
    np.testing.assert_array_equal(offs.cpu().numpy(), roffs)
    close(ck, rk, 1e-2)
    close(cv, rv, 1e-2)


def test_index_builders_bit_exact():
    lens = [0, 1, 37, 300, 0, 129]
    Tn = sum(lens)
    cuq = _cu_t(lens)
    assert SA.build_token_to_seq(cuq, Tn + 2, DEV).cpu().tolist() == O.build_token_to_seq(cuq.cpu(), Tn + 2).tolist()
    offs = torch.tensor(O.comp_offsets_for(lens, 128), dtype=torch.int32, device=DEV)
    got = HCA.build_hca_topk_idxs(cuq, offs, Tn, 16, 128)
    np.testing.assert_array_equal(got.cpu().numpy(), O.build_hca_topk_idxs(cuq.cpu(), offs.cpu(), Tn, 16, 128))


def _indexer_on_cores(q, ck, cuq, offs, n_win, top_k, m):
    """build_csa_topk_idxs with the dot products on CUDA cores: the C entry
    point without a score workspace."""
    Tn, H, D = q.shape
    K = n_win + top_k
    out = torch.full((Tn, K), -1, dtype=torch.int32, device=DEV)
    L = T.lib()
    st = T.stream_of(q)
    T.check(L.tak_build_window_idxs(T.ptr(cuq), cuq.numel() - 1, Tn, n_win, T.ptr(out), K, st))
    mc = int((offs[1:] - offs[:-1]).max())
    T.check(L.tak_csa_indexer_topk(T.ptr(q), T.strides(q), T.ptr(ck), T.strides(ck), T.ptr(cuq), None, T.ptr(offs),
                                   cuq.numel() - 1, Tn, H, ck.shape[1], D, n_win, top_k, m, mc, T.ptr(out), K,
                                   T.dtype_code(q), None, 0, ck.shape[0], st))
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("top_k", [16, 48, 300])
@pytest.mark.parametrize("rows", ["many", "few", "many-cores", "long"])
def test_csa_indexer_bit_exact(dtype, top_k, rows):
    """Lightning indexer on 512-dim compressed keys; ties and fewer-than-k
    causal slots included (short sequences).  top_k 16 takes the
    repeated-argmax selection, 48 and 300 the sorted one (up to 525 slots).
    "many" (2856 query rows) and "few" (271 rows: the 512-thread selection)
    score on the tensor cores; "many-cores" scores each row on CUDA cores;
    "long" has a 6000-token sequence (1500 slots: past the one-warp-per-row
    selection, so the tensor-core scores go to the shared-memory sort)."""
    lens = {"few": [3, 8, 260], "long": [6000, 37]}.get(rows, [3, 40, 200, 513, 2100])
    Tn = sum(lens)
    g = torch.Generator().manual_seed(41)
    q = torch.randn(Tn, 4, 512, generator=g).to(DEV, dtype)
    k = torch.randn(Tn, 1, 512, generator=g).to(DEV, dtype)
    cuq = _cu_t(lens)
    ck, cv, offs = CSA.compress_kv_overlap(k, k, cuq, 4)
    if rows == "many-cores":
        got = _indexer_on_cores(q, ck, cuq, offs, 8, top_k, 4)
    else:
        got = CSA.build_csa_topk_idxs(q, ck, cuq, offs, 8, top_k, 4)
    name = "bfloat16" if dtype == torch.bfloat16 else "float16"
    ref = O.build_csa_topk_idxs(npy(q), npy(ck), cuq.cpu(), offs.cpu(), 8, top_k, 4, name)
    assert_topk_match(got.cpu().numpy(), ref, npy(q), npy(ck), lambda t: Tn, 8,
                      2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_csa_hca_forward_latent512(dtype):
    """MLA-style: one 512-dim latent tensor passed as both K and V, 64 query
    heads on one KV head (the shared-latent 512/512 tensor-core path), ragged
    sequences longer than the window and top-k."""
    lens = [300, 1030, 7]
    Tn = sum(lens)
    g = torch.Generator().manual_seed(57)
    q = torch.randn(Tn, 64, 512, generator=g).to(DEV, dtype)
    kv = torch.randn(Tn, 1, 512, generator=g).to(DEV, dtype)
    sink = torch.randn(64, generator=g).to(DEV)
    cuq = _cu_t(lens)
    name = "bfloat16" if dtype == torch.bfloat16 else "float16"
    out = CSA.csa_prefill_forward(q, kv, kv, cuq, 64, 32, 4, sink)
    ref, _, _ = O.csa_prefill_forward(npy(q), npy(kv), npy(kv), cuq.cpu(), 64, 32, 4, sink.cpu(), name)
    close(out, ref, TOL16)
    out = HCA.hca_prefill_forward(q, kv, kv, cuq, 64, 128, sink)
    ref, _, _ = O.hca_prefill_forward(npy(q), npy(kv), npy(kv), cuq.cpu(), 64, 128, sink.cpu(), name)
    close(out, ref, TOL16)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_csa_decode_indexer_split_scores(dtype):
    """Decode index rows with the scores split over CTAs (score workspace) equal
    the rows of one CTA per request scoring on its own (no workspace), bit for
    bit (same dot-product order), and match the oracle's csa_decode_idxs (up to
    one-rounding-step swaps); contexts up to 4000 tokens (1000 slots), empty and
    short ones included."""
    ctx = [4000, 0, 1, 7, 2049, 3333, 512, 90]
    P, m, n_win, top_k = 64, 4, 16, 300
    _, kc, _, _, _, bt, _, cl, _ = _sparse_decode_case(ctx, 8, 1, 512, 512, P, 1, 1, 1, dtype, 73,
                                                       shared_latent=True)
    g = torch.Generator().manual_seed(74)
    q = torch.randn(len(ctx), 8, 512, generator=g).to(DEV, dtype)
    ck, _, offs, lens, offs_h = T.compress_paged(kc, kc, bt, cl, P, m, 2 * m)
    B, K = len(ctx), n_win + top_k
    mc = max(offs_h[i + 1] - offs_h[i] for i in range(B))
    L = T.lib()
    st = T.stream_of(q)
    rows = []
    for with_ws in (True, False):
        idx = torch.empty((B, K), dtype=torch.int32, device=DEV)
        T.check(L.tak_build_decode_topk_idxs(T.ptr(cl), T.ptr(offs), B, n_win, top_k, 0, T.ptr(idx), K, st))
        nb = L.tak_csa_indexer_workspace_size(B, mc, T.dtype_code(q)) if with_ws else 0
        ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=DEV)
        T.check(L.tak_csa_indexer_topk(T.ptr(q), T.strides(q), T.ptr(ck), T.strides(ck), None, T.ptr(cl),
                                       T.ptr(offs), B, B, 8, 1, 512, n_win, top_k, m, mc, T.ptr(idx), K,
                                       T.dtype_code(q), T.ptr(ws) if with_ws else None, nb, ck.shape[0], st))
        rows.append(idx.cpu().numpy())
    np.testing.assert_array_equal(rows[0], rows[1])
    name = "bfloat16" if dtype == torch.bfloat16 else "float16"
    ref = O.csa_decode_idxs(npy(q), npy(ck), cl.cpu(), offs.cpu(), n_win, top_k, m, name)
    assert_topk_match(rows[0], ref, npy(q), npy(ck), lambda b: int(cl[b]), n_win,
                      2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_csa_hca_decode_latent512(dtype):
    """MLA-style decode: one paged 512-dim latent cache passed as both K and V
    (pooled once, compressed V a view of compressed K, the shared-latent
    tensor-core sparse path), 64 query heads, ragged contexts across pages."""
    ctx = [300, 1030, 7, 129, 64]
    g = torch.Generator().manual_seed(59)
    P = 64
    _, kc, _, _, _, bt, _, cl, sink = _sparse_decode_case(ctx, 64, 1, 512, 512, P, 1, 1, 1, dtype, 59,
                                                          shared_latent=True)
    q = torch.randn(len(ctx), 64, 512, generator=g).to(DEV, dtype)
    name = "bfloat16" if dtype == torch.bfloat16 else "float16"
    out = CSA.csa_decode_forward(q, kc, kc, bt, cl, 64, 32, 4, P, sink)
    ref, _, _ = O.csa_decode_forward(npy(q), npy(kc), npy(kc), bt.cpu(), cl.cpu(), 64, 32, 4, P, sink.cpu(), name)
    close(out, ref, TOL16)
    out = HCA.hca_decode_forward(q, kc, kc, bt, cl, 64, 128, P, sink)
    ref, _, _ = O.hca_decode_forward(npy(q), npy(kc), npy(kc), bt.cpu(), cl.cpu(), 64, 128, P, sink.cpu(), name)
    close(out, ref, TOL16)


@pytest.mark.parametrize("kind", ["csa", "hca"])
def test_decode_wrappers_graph_capture(kind):
    """csa/hca_decode_forward with max_compressed read nothing on the host, so
    one call is captured in a CUDA graph; replays after the context lengths
    and queries change in place (within the block tables' reach) equal the
    oracle each time."""
    ctx0 = [300, 1030, 7, 129, 64]
    P, n_win = 64, 64
    _, kc, _, _, _, bt, _, cl, sink = _sparse_decode_case(ctx0, 64, 1, 512, 512, P, 1, 1, 1, torch.bfloat16, 67,
                                                          shared_latent=True)
    g = torch.Generator().manual_seed(68)
    q = torch.randn(len(ctx0), 64, 512, generator=g).to(DEV, torch.bfloat16)
    stride = 4 if kind == "csa" else 128
    cap = sum(max(1, -(-c // stride)) for c in (1030,) * len(ctx0))  # every request at the longest context

    def run():
        if kind == "csa":
            return CSA.csa_decode_forward(q, kc, kc, bt, cl, n_win, 32, 4, P, sink, max_compressed=cap)
        return HCA.hca_decode_forward(q, kc, kc, bt, cl, n_win, 128, P, sink, max_compressed=cap)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        run()  # warm-up outside the capture (kernel attributes, library load)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = run()
    for new_ctx in (ctx0, [5, 1000, 64, 0, 1], [299, 1, 7, 128, 63]):
        cl.copy_(torch.tensor(new_ctx, dtype=torch.int32))
        q.copy_(torch.randn(len(ctx0), 64, 512, generator=g))
        graph.replay()
        torch.cuda.synchronize()
        if kind == "csa":
            ref, _, _ = O.csa_decode_forward(npy(q), npy(kc), npy(kc), bt.cpu(), cl.cpu(), n_win, 32, 4, P,
                                             sink.cpu(), "bfloat16")
        else:
            ref, _, _ = O.hca_decode_forward(npy(q), npy(kc), npy(kc), bt.cpu(), cl.cpu(), n_win, 128, P,
                                             sink.cpu(), "bfloat16")
        close(out, ref, TOL16)
    del graph


@pytest.mark.parametrize("stride,window", [(4, 8), (128, 128), (3, 6)])
def test_compress_paged_k_only_latent(stride, window):
    """Paged pooling with V a prefix view of K (576-dim latent + rope rows, V =
    the first 512 columns): K is pooled once and compressed V is the same view
    of compressed K, equal to pooling V on its own."""
    ctx = [0, 1, 5, 300, 1030, 129, 64, 2]
    _, kc, vc, _, _, bt, _, cl, _ = _sparse_decode_case(ctx, 8, 1, 576, 512, 64, 1, 1, 1, torch.bfloat16, 61,
                                                        shared_latent=True)
    ck, cv, offs, lens, _ = T.compress_paged(kc, vc, bt, cl, 64, stride, window)
    assert T.last_kernel() == "compress_bulk"  # plain-mean 16-bit pooling straight from the pages
    assert cv.data_ptr() == ck.data_ptr() and cv.shape[-1] == 512
    kt, cut = O.gather_paged_to_tnd(npy(kc), bt.cpu(), cl.cpu(), 64)
    rk, _, roffs = O.compress_kv(kt, kt[..., :512], cut, stride, window)
    np.testing.assert_array_equal(offs.cpu().numpy(), roffs)
    close(ck, rk, 1e-2)
    close(cv, rk[..., :512], 1e-2)


def test_csa_hca_forward_bf16():
    lens = [50, 200]
    Tn = sum(lens)
    g = torch.Generator().manual_seed(51)
    q = torch.randn(Tn, 8, 128, generator=g).to(DEV, torch.bfloat16)
    k = torch.randn(Tn, 2, 128, generator=g).to(DEV, torch.bfloat16)
    v = torch.randn(Tn, 2, 128, generator=g).to(DEV, torch.bfloat16)
    sink = torch.randn(8, generator=g).to(DEV)
    cuq = _cu_t(lens)
    out = CSA.csa_prefill_forward(q, k, v, cuq, 16, 8, 4, sink)
    ref, _, _ = O.csa_prefill_forward(npy(q), npy(k), npy(v), cuq.cpu(), 16, 8, 4, sink.cpu(), "bfloat16")
    close(out, ref, TOL16)
    out = HCA.hca_prefill_forward(q, k, v, cuq, 16, 32, sink)
    ref, _, _ = O.hca_prefill_forward(npy(q), npy(k), npy(v), cuq.cpu(), 16, 32, sink.cpu(), "bfloat16")
    close(out, ref, TOL16)

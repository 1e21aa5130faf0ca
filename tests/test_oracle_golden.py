"""Pin the CPU oracle to the reference: golden vectors made by the reference's
own torch functions on its own runner configurations (tests/golden)."""

import json
import os

import numpy as np
import pytest
import torch

import golden_inputs as gi
from oracle import attention_oracle as O

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
GOLD = np.load(os.path.join(HERE, "reference_golden.npz"))
SHA = json.load(open(os.path.join(HERE, "reference_golden_inputs.json")))["sha256"]
CASES = sorted(SHA)

# The reference's runners compare with allclose(atol=1e-2, rtol=1e-2)
# (FP:276, PD:256, SA:571, CSA:514, HCA:459); the reference computes in fp16
# with fp16-rounded softmax weights, the oracle in float64.
ATOL = RTOL = 1e-2


def _sha(t):
    import hashlib
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def _check_out(case, out):
    rows = GOLD[f"{case}/rows"]
    ref = GOLD[f"{case}/out"].astype(np.float64)
    np.testing.assert_allclose(out[rows], ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("case", CASES)
def test_inputs_regenerate_bit_exact(case):
    inp = gi.case_inputs(case)
    for name, h in SHA[case].items():
        assert _sha(inp[name]) == h, f"{case}:{name} differs from the fixture's inputs"


@pytest.mark.parametrize("case", [c for c in CASES if c.startswith("fp_")])
def test_prefill(case):
    inp = gi.case_inputs(case)
    out, lse = O.prefill(inp["q"], inp["k"], inp["v"], inp["cu_seqlens"], causal=case.endswith("c1"))
    _check_out(case, out)
    assert np.isfinite(lse).all()


@pytest.mark.parametrize("case", [c for c in CASES if c.startswith("pd_")])
def test_paged_decode(case):
    inp = gi.case_inputs(case)
    out, _ = O.paged_decode(inp["q"], inp["k_cache"], inp["v_cache"], inp["block_tables"],
                            inp["context_lens"], gi.PD_BLOCK)
    _check_out(case, out)


@pytest.mark.parametrize("case", [c for c in CASES if c.startswith("sap_")])
def test_sparse_prefill(case):
    inp = gi.case_inputs(case)
    out, _ = O.sparse_prefill(inp["q"], inp["k"], inp["v"], inp["topk_idxs"], inp["cu_seqlens"],
                              inp.get("attn_sink"))
    _check_out(case, out)


@pytest.mark.parametrize("case", [c for c in CASES if c.startswith("sad_")])
def test_sparse_decode(case):
    inp = gi.case_inputs(case)
    out, _ = O.sparse_decode(inp["q"], inp["k_cache"], inp["v_cache"], inp["compressed_k"],
                             inp["compressed_v"], inp["block_tables"], inp["topk_idxs"],
                             inp["context_lens"], gi.SA_NWIN_D, gi.SA_BLOCK, inp.get("attn_sink"))
    _check_out(case, out)


def _check_compress(case, k, v, cu, stride, window):
    ck, cv, offs = O.compress_kv(k, v, cu, stride, window)
    np.testing.assert_array_equal(offs, GOLD[f"{case}/comp_offsets"])
    # the reference averages fp16 values and stores fp16: one fp16 rounding
    np.testing.assert_allclose(ck, GOLD[f"{case}/ck"].astype(np.float64), atol=2e-3, rtol=2e-3)
    np.testing.assert_allclose(cv, GOLD[f"{case}/cv"].astype(np.float64), atol=2e-3, rtol=2e-3)


def assert_topk_equivalent(mine, ref, n_win, causal_count, score_of):
    """Window part bit-exact.  Compressed part: wherever the reference picked a
    causal slot, both rows must pick slots of identical indexer score in the
    same order (bit-exact unless scores tie exactly: torch.topk orders equal
    values in a backend-defined way, this repository by lower slot index).
    Where fewer than top_k slots are causal, the reference's remaining picks
    are -inf ties; there only the count of picks must agree."""
    np.testing.assert_array_equal(mine[:, :n_win], ref[:, :n_win])
    for t in range(ref.shape[0]):
        c = causal_count[t]
        a, b = mine[t, n_win:n_win + c], ref[t, n_win:n_win + c]
        assert len(set(a.tolist())) == c
        np.testing.assert_array_equal(score_of(t, a), score_of(t, b), err_msg=f"token {t}")
        assert (mine[t, n_win + c:] >= 0).sum() == (ref[t, n_win + c:] >= 0).sum()


@pytest.mark.parametrize("case", [c for c in CASES if c.startswith("csap_")])
def test_csa_prefill(case):
    inp = gi.case_inputs(case)
    q, k, v, cu = inp["q"], inp["k"], inp["v"], inp["cu_seqlens"]
    _check_compress(case, k, v, cu, gi.CSA_M, 2 * gi.CSA_M)
    ck16 = GOLD[f"{case}/ck"]
    offs = GOLD[f"{case}/comp_offsets"]
    ref_idx = GOLD[f"{case}/topk_idxs"]
    mine = O.build_csa_topk_idxs(q, ck16.astype(np.float64), cu, offs, gi.CSA_NWIN_P, gi.CSA_TOPK, gi.CSA_M,
                                 "float16")
    T = q.shape[0]
    causal = np.zeros(T, np.int64)
    for s in range(len(gi.SA_CU) - 1):
        nc = offs[s + 1] - offs[s]
        for p in range(gi.SA_CU[s + 1] - gi.SA_CU[s]):
            causal[gi.SA_CU[s] + p] = min(gi.CSA_TOPK, int((np.arange(nc) * gi.CSA_M < p).sum()))
    # the reference's indexer scores: fp16 matmul of the last head (CSA:144)
    qlast = q[:, -1, :]
    kf16 = torch.from_numpy(ck16[:, -1, :])

    def score_of(t, idxs):
        return torch.matmul(kf16[torch.from_numpy(idxs - T).long()], qlast[t]).numpy()

    assert_topk_equivalent(mine, ref_idx, gi.CSA_NWIN_P, causal, score_of)
    # attention over the reference's own index rows and compressed K/V
    kf = np.concatenate([k.float().numpy(), ck16.astype(np.float32)], 0)
    vf = np.concatenate([v.float().numpy(), GOLD[f"{case}/cv"].astype(np.float32)], 0)
    out, _ = O.sparse_prefill(q, kf, vf, ref_idx, cu, inp.get("attn_sink"))
    _check_out(case, out)


@pytest.mark.parametrize("case", [c for c in CASES if c.startswith("hcap_")])
def test_hca_prefill(case):
    inp = gi.case_inputs(case)
    q, k, v, cu = inp["q"], inp["k"], inp["v"], inp["cu_seqlens"]
    _check_compress(case, k, v, cu, gi.HCA_M, gi.HCA_M)
    out, _, idx = O.hca_prefill_forward(q, k, v, cu, gi.HCA_NWIN, gi.HCA_M, inp.get("attn_sink"), "float16")
    np.testing.assert_array_equal(idx, GOLD[f"{case}/topk_idxs"])
    _check_out(case, out)


@pytest.mark.parametrize("case", [c for c in CASES if c.startswith("csad_")])
def test_csa_decode(case):
    inp = gi.case_inputs(case)
    out, _, _ = O.csa_decode_forward(inp["q"], inp["k_cache"], inp["v_cache"], inp["block_tables"],
                                     inp["context_lens"], gi.CSA_NWIN_D, gi.CSA_TOPK, gi.CSA_M, gi.SA_BLOCK,
                                     inp.get("attn_sink"), "float16")
    _check_out(case, out)


@pytest.mark.parametrize("case", [c for c in CASES if c.startswith("hcad_")])
def test_hca_decode(case):
    inp = gi.case_inputs(case)
    out, _, _ = O.hca_decode_forward(inp["q"], inp["k_cache"], inp["v_cache"], inp["block_tables"],
                                     inp["context_lens"], gi.HCA_NWIN, gi.HCA_M, gi.SA_BLOCK,
                                     inp.get("attn_sink"), "float16")
    _check_out(case, out)


def test_window_and_token_to_seq_edge_cases():
    cu = [0, 0, 3, 3, 7]                       # empty sequences interleaved
    w = O.build_window_idxs(cu, 7, 4)
    assert w[0].tolist() == [-1, -1, -1, 0]
    assert w[2].tolist() == [-1, 0, 1, 2]
    assert w[3].tolist() == [-1, -1, -1, 3]
    assert O.build_token_to_seq(cu, 8).tolist() == [1, 1, 1, 3, 3, 3, 3, 0]
    assert O.comp_offsets_for([0, 3, 0, 4], 4).tolist() == [0, 0, 1, 1, 2]

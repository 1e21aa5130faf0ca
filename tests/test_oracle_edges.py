"""Pin the oracle's integer index builders and mean compressors to the
reference on edge configurations (tests/golden/reference_edges.npz, made by
tests/golden/make_golden.py from the reference's own functions).

Sequence lengths 0, 1, 2, 3, 4, 5, 7, 8, 9, 127, 128, 129 and 300; CSA strides
1, 3 and 4 (attention/csa.py:9-69); HCA strides 1, 5, 16 and 128
(attention/hca.py:9-69); windows of 1, 4 and 130 tokens, the last longer than
most sequences (attention/hca.py:76-146); CSA top-k above the slot count
(attention/csa.py:76-164).  Offsets and HCA index rows must match bit for bit;
compressed rows within one fp16 rounding.

The same fixture holds the reference's torch attention functions on edge
lengths: 0 / 1 / 2 / 63-65 / 129-token sequences in prefill, contexts of 1,
P - 1, P, P + 1 and whole tables in paged decode, -1 padding and an all -1
row with and without sinks in sparse prefill, contexts shorter than the
window in sparse decode.
"""
import os

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O
from test_oracle_golden import assert_topk_equivalent

EDGE = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_edges.npz"))
CU = EDGE["cu_seqlens"]
LENS = np.diff(CU)
T = int(CU[-1])
K, V, Q = EDGE["k"], EDGE["v"], EDGE["q"]


def test_edge_lengths_cover_the_corners():
    assert 0 in LENS and 1 in LENS and 300 in LENS and T == LENS.sum()


@pytest.mark.parametrize("kind,stride,window", [("csa", 1, 2), ("csa", 3, 6), ("csa", 4, 8), ("hca", 1, 1),
                                                ("hca", 5, 5), ("hca", 16, 16), ("hca", 128, 128)])
def test_compress_edges(kind, stride, window):
    ck, cv, offs = O.compress_kv(K, V, CU, stride, window)
    case = f"{kind}_m{stride}"
    np.testing.assert_array_equal(offs, EDGE[f"{case}/comp_offsets"])
    # the reference averages fp16 rows and stores fp16: one fp16 rounding
    np.testing.assert_allclose(ck, EDGE[f"{case}/ck"].astype(np.float64), atol=2e-3, rtol=2e-3)
    np.testing.assert_allclose(cv, EDGE[f"{case}/cv"].astype(np.float64), atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize("m_prime", [5, 16, 128])
@pytest.mark.parametrize("n_win", [1, 4, 130])
def test_hca_index_rows_edges(m_prime, n_win):
    offs = EDGE[f"hca_m{m_prime}/comp_offsets"]
    mine = O.build_hca_topk_idxs(CU, offs, T, n_win, m_prime)
    np.testing.assert_array_equal(mine, EDGE[f"hca_m{m_prime}/topk_idxs_w{n_win}"])


@pytest.mark.parametrize("m,n_win,top_k", [(4, 4, 6), (4, 1, 64), (3, 130, 16)])
def test_csa_index_rows_edges(m, n_win, top_k):
    ck16 = EDGE[f"csa_m{m}/ck"]
    offs = EDGE[f"csa_m{m}/comp_offsets"]
    ref = EDGE[f"csa_idx_m{m}_w{n_win}_k{top_k}"]
    mine = O.build_csa_topk_idxs(Q, ck16.astype(np.float64), CU, offs, n_win, top_k, m, "float16")
    assert mine.shape == ref.shape
    causal = np.zeros(T, np.int64)
    for s in range(len(LENS)):
        nc = int(offs[s + 1] - offs[s])
        for p in range(int(LENS[s])):
            causal[CU[s] + p] = min(top_k, int((np.arange(nc) * m < p).sum()))
    qlast = torch.from_numpy(Q[:, -1, :])
    kf16 = torch.from_numpy(ck16[:, -1, :])

    def score_of(t, idxs):   # the reference's indexer score: fp16 product of the last head (csa.py:144)
        return torch.matmul(kf16[torch.from_numpy(idxs - T).long()], qlast[t]).numpy()

    assert_topk_equivalent(mine, ref, n_win, causal, score_of)


# ---------------------------------------------------------------------------
# attention on edge lengths: the reference's torch functions
# (flash_attention_prefill.py:177-229, paged_attention_decode.py:157-202,
# sparse_attn_fwd.py:389-470), fp16; the reference's runner tolerance
# ---------------------------------------------------------------------------

ATOL = RTOL = 1e-2


def _e(name):
    return EDGE[name].astype(np.float64) if EDGE[name].dtype == np.float16 else EDGE[name]


@pytest.mark.parametrize("causal", [True, False])
def test_prefill_edge_lengths(causal):
    cu = EDGE["fp/cu_seqlens"]
    assert 0 in np.diff(cu) and 1 in np.diff(cu) and 129 in np.diff(cu)
    out, lse = O.prefill(_e("fp/q"), _e("fp/k"), _e("fp/v"), cu, causal)
    np.testing.assert_allclose(out, _e(f"fp/out_c{int(causal)}"), atol=ATOL, rtol=RTOL)
    assert np.isfinite(lse).all()


def test_paged_decode_edge_contexts():
    out, _ = O.paged_decode(_e("pd/q"), _e("pd/k_cache"), _e("pd/v_cache"), EDGE["pd/block_tables"],
                            EDGE["pd/context_lens"], 16)
    np.testing.assert_allclose(out, _e("pd/out"), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("with_sink", [False, True])
def test_sparse_prefill_padding_and_empty_rows(with_sink):
    k = _e("sap/k")
    sink = _e("sap/attn_sink") if with_sink else None
    out, lse = O.sparse_prefill(_e("sap/q"), k, k, EDGE["sap/topk_idxs"], None, sink)
    np.testing.assert_allclose(out, _e(f"sap/out_s{int(with_sink)}"), atol=ATOL, rtol=RTOL)
    assert np.all(out[2] == 0)                 # an all -1 row: zeros, as the reference's l_safe gives
    assert np.isneginf(lse[2]).all() != with_sink


@pytest.mark.parametrize("with_sink", [False, True])
def test_sparse_decode_short_contexts(with_sink):
    sink = _e("sad/attn_sink") if with_sink else None
    out, _ = O.sparse_decode(_e("sad/q"), _e("sad/k_cache"), _e("sad/v_cache"), _e("sad/compressed_k"),
                             _e("sad/compressed_v"), EDGE["sad/block_tables"], EDGE["sad/topk_idxs"],
                             EDGE["sad/context_lens"], 4, 16, sink)
    np.testing.assert_allclose(out, _e(f"sad/out_s{int(with_sink)}"), atol=ATOL, rtol=RTOL)

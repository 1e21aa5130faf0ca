"""Pin the oracle's integer index builders and mean compressors to the
reference on edge configurations (tests/golden/reference_edges.npz, made by
tests/golden/make_golden.py from the reference's own functions).

Sequence lengths 0, 1, 2, 3, 4, 5, 7, 8, 9, 127, 128, 129 and 300; CSA strides
1, 3 and 4 (attention/csa.py:9-69); HCA strides 1, 5, 16 and 128
(attention/hca.py:9-69); windows of 1, 4 and 130 tokens, the last longer than
most sequences (attention/hca.py:76-146); CSA top-k above the slot count
(attention/csa.py:76-164).  Offsets and HCA index rows must match bit for bit;
compressed rows within one fp16 rounding.
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

"""Properties of the oracle's gated window pooling (CPU).

The gate (softmax of per-row logits over each window) is an addition with no
counterpart in the reference, so no golden vector pins it.  These properties
do: equal logits give the reference's plain mean (compress_kv_overlap,
attention/csa.py:45-55; compress_kv_simple, attention/hca.py:45-55), the
softmax ignores a constant shift, a -inf logit removes its row, an all-masked
window pools to zeros and large logits do not overflow.
"""
import numpy as np
import pytest

from oracle import attention_oracle as O


def _case(seed, lens=(37, 64, 5), H=2, D=16, Dv=8):
    rng = np.random.default_rng(seed)
    T = sum(lens)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    k = rng.standard_normal((T, H, D))
    v = rng.standard_normal((T, H, Dv))
    g = rng.standard_normal(T)
    return k, v, g, cu


@pytest.mark.parametrize("stride,window", [(4, 8), (16, 16), (3, 6)])
def test_equal_logits_give_the_plain_mean(stride, window):
    k, v, _, cu = _case(1)
    ck0, cv0, o0 = O.compress_kv(k, v, cu, stride, window)
    ck1, cv1, o1 = O.compress_kv(k, v, cu, stride, window, gate=np.zeros(k.shape[0]))
    np.testing.assert_array_equal(o0, o1)
    np.testing.assert_allclose(ck1, ck0, rtol=0, atol=1e-12)
    np.testing.assert_allclose(cv1, cv0, rtol=0, atol=1e-12)


def test_constant_shift_and_large_logits():
    k, v, g, cu = _case(2)
    ck0, cv0, _ = O.compress_kv(k, v, cu, 4, 8, gate=g)
    for c in (-30.0, 7.5, 1000.0):
        ck1, cv1, _ = O.compress_kv(k, v, cu, 4, 8, gate=g + c)
        assert np.isfinite(ck1).all() and np.isfinite(cv1).all()
        np.testing.assert_allclose(ck1, ck0, rtol=0, atol=1e-12)
        np.testing.assert_allclose(cv1, cv0, rtol=0, atol=1e-12)


def test_masked_rows_and_all_masked_windows():
    k, v, g, cu = _case(3, lens=(24,))
    g = g.copy()
    g[5] = -np.inf                      # one masked row inside slots 0 and 1 (rows 0-7, 4-11)
    g[16:24] = -np.inf                  # slots 4 (rows 16-23) and 5 (rows 20-23): every row masked
    ck, cv, offs = O.compress_kv(k, v, cu, 4, 8, gate=g)
    assert offs.tolist() == [0, 6]
    # slot 1 = softmax over rows 4-11 without row 5
    rows = [4, 6, 7, 8, 9, 10, 11]
    w = np.exp(g[rows] - g[rows].max())
    w /= w.sum()
    np.testing.assert_allclose(ck[1], np.tensordot(w, k[rows], 1), rtol=0, atol=1e-12)
    np.testing.assert_allclose(cv[1], np.tensordot(w, v[rows], 1), rtol=0, atol=1e-12)
    # slot 3 (rows 12-19): rows 16-19 masked, the softmax is over rows 12-15
    rows = [12, 13, 14, 15]
    w = np.exp(g[rows] - g[rows].max())
    w /= w.sum()
    np.testing.assert_allclose(ck[3], np.tensordot(w, k[rows], 1), rtol=0, atol=1e-12)
    for slot in (4, 5):
        assert not ck[slot].any() and not cv[slot].any()

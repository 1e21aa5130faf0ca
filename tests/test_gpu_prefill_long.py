"""Varlen prefill at the lengths the prefill benchmark and the box-scale mixed
step run (hundreds to tens of thousands of tokens per sequence), against the
CPU oracle on sampled rows.

The reference's kernel (attention/flash_attention_prefill.py:11-102) is checked
by its runner at lengths up to 511; the B200 kernel's schedule has paths that
only long sequences reach: many 256-row blocks per sequence issued longest
first, the per-sequence head piece before the first 256-row boundary, the K/V
ring wrapping over up to 256 blocks, and the lazy O rescale (taken only when a
row's running max grows by more than 2^8).  Rows are sampled (first, last,
around every 128/256-row boundary, every 1024th) so that the float64 oracle
finishes in seconds.  Tolerances: bf16 outputs max-abs <= 2e-2, LSE <= 1e-3.
"""

import math

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu

import _tak_b200 as T  # noqa: E402
import flash_attention_prefill as FP  # noqa: E402

DEV = "cuda"
TOL16 = 2e-2
TOL_LSE = 1e-3
ROWS = 256  # the kernel's row-block size (two 128-row tiles)


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert T.read_device_error() == 0, "a kernel reported a timed-out wait"


def _sample_rows(lens):
    """Global rows to check: per sequence its first rows, last rows, the rows
    around each 128-row tile edge of its first blocks, the rows around the
    first 256-aligned global boundary (end of the head piece) and every
    1024th row."""
    cu = np.concatenate([[0], np.cumsum(lens)])
    rows = set()
    for s, L in enumerate(lens):
        st = int(cu[s])
        if L == 0:
            continue
        pos = {0, 1, 127, 128, 129, 254, 255, 256, 257, L - 2, L - 1}
        pos |= set(range(0, L, 1024))
        b0 = -(-st // ROWS) * ROWS - st          # first aligned boundary, as a position
        pos |= {b0 - 1, b0, b0 + 1, b0 + 127, b0 + 128, b0 + 255, b0 + 256}
        rows |= {st + p for p in pos if 0 <= p < L}
    return np.array(sorted(rows), dtype=np.int64)


def _check(q, k, v, lens, causal):
    cu = torch.tensor([0] + np.cumsum(lens).tolist(), dtype=torch.int32, device=DEV)
    out, lse = FP.flash_attention_prefill(q, k, v, cu, causal, return_lse=True)
    torch.cuda.synchronize()
    rows = _sample_rows(lens)
    ridx = torch.from_numpy(rows).to(DEV)
    qn = q[ridx].float().cpu().numpy()
    kn, vn = k.float().cpu().numpy(), v.float().cpu().numpy()
    ref, ref_lse = _oracle_rows(qn, kn, vn, cu.cpu().numpy(), rows, causal)
    got = out[ridx].float().cpu().numpy()
    got_lse = lse[ridx].cpu().numpy()
    err = np.abs(got.astype(np.float64) - ref).max()
    assert err <= TOL16, f"max abs err {err:.3e} over {rows.size} sampled rows"
    assert np.isfinite(got_lse).all() and np.isfinite(ref_lse).all()
    lerr = np.abs(got_lse.astype(np.float64) - ref_lse).max()
    assert lerr <= TOL_LSE, f"lse max abs err {lerr:.3e}"
    return err, lerr


def _oracle_rows(q_rows, k, v, cu, rows, causal):
    """O.prefill_rows with q given only at the sampled rows (q_rows[i] is row rows[i])."""

    class _RowView:
        shape = (int(cu[-1]), q_rows.shape[1], q_rows.shape[2])

        def __getitem__(self, idx):
            pos = np.searchsorted(rows, idx)
            assert (rows[pos] == idx).all()
            return q_rows[pos]

    return O.prefill_rows(_RowView(), k, v, cu, rows, causal)


@pytest.mark.parametrize("causal", [True, False])
def test_prefill_long_sequences(causal):
    """Lengths 300, 512, 1000, 4097 and 32768 (64 query heads / 8 KV heads,
    d 128, bf16): the 300-token sequence puts every later sequence off the
    256-row grid, so each has a head piece and then full aligned blocks; the
    32768-token sequence runs 128 row blocks and 256 K/V blocks per tile."""
    lens = [300, 512, 1000, 4097, 32768]
    Tn = sum(lens)
    g = torch.Generator(device=DEV).manual_seed(101 if causal else 102)
    q = torch.randn(Tn, 64, 128, device=DEV, generator=g).to(torch.bfloat16)
    k = torch.randn(Tn, 8, 128, device=DEV, generator=g).to(torch.bfloat16)
    v = torch.randn(Tn, 8, 128, device=DEV, generator=g).to(torch.bfloat16)
    _check(q, k, v, lens, causal)


@pytest.mark.parametrize("causal", [True, False])
def test_prefill_rising_scores_rescale(causal):
    """Scores that rise along the key axis: every query carries 4 u and key j
    carries 0.15 j u (u a unit vector), so each 128-key block raises a row's
    running max by about 9.8 in log2 units -- more than the 2^8 lazy-rescale
    threshold -- and O and l are rescaled at almost every block, 16 times per
    2048-token row.  Two such sequences plus a short one ahead of them (off
    the 256-row grid)."""
    lens = [77, 2048, 2048]
    Tn = sum(lens)
    H, Hkv, D = 64, 8, 128
    g = torch.Generator().manual_seed(103)
    u = torch.ones(D) / math.sqrt(D)
    q = torch.randn(Tn, H, D, generator=g) + 4.0 * u
    k = torch.randn(Tn, Hkv, D, generator=g)
    v = torch.randn(Tn, Hkv, D, generator=g)
    cu = np.concatenate([[0], np.cumsum(lens)])
    for s in range(len(lens)):
        j = torch.arange(lens[s], dtype=torch.float32)
        k[cu[s]:cu[s + 1]] += (0.15 * j)[:, None, None] * u
    q, k, v = (t.to(DEV, torch.bfloat16) for t in (q, k, v))
    _check(q, k, v, lens, causal)

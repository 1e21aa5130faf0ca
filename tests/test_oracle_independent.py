"""The oracle against a second, independent formulation of the same math (CPU).

The golden vectors pin the oracle where the reference itself runs: fp16 inputs,
V with the head dim of K, output only.  The kernels also return the log-sum-exp
(the reference computes none), take fp32/bf16 inputs and a V head dim of its
own (MLA latent: 576 / 512).  Those parts of the oracle are checked here
against torch float64 code written a different way:

* attention as one dense masked score matrix over all packed rows
  (block-diagonal for varlen, a scatter of the index lists for sparse), with
  ``torch.logsumexp`` for the LSE;
* the sink as one extra logit column whose value row is zero -- the
  definition behind the kernels' fold ``m' = max(m, sink)``,
  ``l = l * e^(m - m') + e^(sink - m')`` (attention/sparse_attn_fwd.py:86-92);
* paged rows addressed by a vectorised block-table lookup
  (attention/paged_attention_decode.py:49-58) rather than by concatenating pages;
* window pooling through prefix sums (plain mean: attention/csa.py:45-55,
  attention/hca.py:45-55) and an explicit per-window softmax (gated).
"""
import math

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O

TOL = dict(rtol=1e-10, atol=1e-10)


def _t(x):
    return torch.as_tensor(np.asarray(x), dtype=torch.float64)


def _dense_attention(q, k, v, allowed, sink=None):
    """q [T,H,D], k [N,H,D], v [N,H,Dv] (heads already expanded), allowed [T,N]
    or [T,H,N] bool; sink [H] or None.  Returns out [T,H,Dv], lse [T,H]."""
    scale = 1.0 / math.sqrt(q.shape[-1])
    s = torch.einsum("thd,nhd->thn", q, k) * scale
    if allowed.dim() == 2:
        allowed = allowed[:, None, :].expand_as(s)
    s = s.masked_fill(~allowed, float("-inf"))
    vals = v
    if sink is not None:
        s = torch.cat([s, sink[None, :, None].expand(s.shape[0], -1, 1)], dim=-1)
        vals = torch.cat([v, torch.zeros_like(v[:1])], dim=0)
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - torch.where(torch.isfinite(lse), lse, torch.zeros_like(lse))[..., None])
    p = torch.where(torch.isfinite(lse)[..., None], p, torch.zeros_like(p))
    out = torch.einsum("thn,nhd->thd", p, vals)
    return out, lse


def _expand(x, H):
    """[N,H_kv,D] -> [N,H,D] with kv_head = h // (H // H_kv)."""
    return x.repeat_interleave(H // x.shape[1], dim=1)


def _close(a, b, **kw):
    np.testing.assert_allclose(np.asarray(a, np.float64), np.asarray(b, np.float64), **(kw or TOL))


# ---------------------------------------------------------------------------
# varlen prefill (attention/flash_attention_prefill.py:11-102)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("heads,dv", [((4, 4), 16), ((8, 2), 16), ((6, 1), 24)])
def test_prefill_dense_mask_form(causal, heads, dv):
    rng = np.random.default_rng(11)
    H, Hkv = heads
    lens = [1, 9, 0, 23, 4]
    T = sum(lens) + 3                       # three tokens outside every sequence
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    q = rng.standard_normal((T, H, 16)).astype(np.float32)
    k = rng.standard_normal((T, Hkv, 16)).astype(np.float32)
    v = rng.standard_normal((T, Hkv, dv)).astype(np.float32)
    out, lse = O.prefill(q, k, v, cu, causal)

    seq = np.full(T, -1)
    pos = np.zeros(T, np.int64)
    for i in range(len(lens)):
        seq[cu[i]:cu[i + 1]] = i
        pos[cu[i]:cu[i + 1]] = np.arange(lens[i])
    seq_t, pos_t = torch.as_tensor(seq), torch.as_tensor(pos)
    allowed = (seq_t[:, None] == seq_t[None, :]) & (seq_t[:, None] >= 0)
    if causal:
        allowed &= pos_t[None, :] <= pos_t[:, None]
    ro, rl = _dense_attention(_t(q), _expand(_t(k), H), _expand(_t(v), H), allowed)
    _close(out, ro)
    _close(lse, rl)
    outside = seq < 0
    assert np.all(out[outside] == 0) and np.all(np.isneginf(lse[outside]))


def test_prefill_lse_is_log_of_row_sums():
    """lse[t,h] = ln sum_j exp(scale q_t.k_j) over the causal keys, written out
    as a plain sum for one short sequence."""
    rng = np.random.default_rng(3)
    L, D = 7, 8
    q = rng.standard_normal((L, 1, D))
    k = rng.standard_normal((L, 1, D))
    v = rng.standard_normal((L, 1, D))
    _, lse = O.prefill(q, k, v, [0, L], True)
    for i in range(L):
        s = [float(q[i, 0] @ k[j, 0]) / math.sqrt(D) for j in range(i + 1)]
        assert abs(lse[i, 0] - math.log(sum(math.exp(x) for x in s))) < 1e-12


@pytest.mark.parametrize("causal", [True, False])
def test_prefill_rows_equals_full_prefill(causal):
    """The row-sampled prefill (used to check sequences too long for the full
    score matrix) gives exactly the full oracle's rows, including rows of
    empty sequences' neighbours and rows outside every sequence."""
    rng = np.random.default_rng(12)
    lens = [5, 0, 300, 1, 77]
    T = sum(lens) + 2
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    q = rng.standard_normal((T, 8, 32)).astype(np.float32)
    k = rng.standard_normal((T, 2, 32)).astype(np.float32)
    v = rng.standard_normal((T, 2, 24)).astype(np.float32)
    out, lse = O.prefill(q, k, v, cu, causal)
    rows = np.array([0, 4, 5, 6, 100, 255, 256, 257, 304, 305, 306, 350, T - 2, T - 1])
    ro, rl = O.prefill_rows(q, k, v, cu, rows, causal)
    _close(ro, out[rows])
    _close(rl, lse[rows])


# ---------------------------------------------------------------------------
# paged decode (attention/paged_attention_decode.py:11-98)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("P", [4, 16])
@pytest.mark.parametrize("heads", [(4, 4), (8, 2)])
def test_paged_decode_table_lookup_form(P, heads):
    rng = np.random.default_rng(5)
    H, Hkv = heads
    D, Dv, pool, maxb = 16, 12, 40, 6
    ctx = np.array([0, 1, P, P + 1, maxb * P - 3, 5], np.int32)
    B = len(ctx)
    kc = rng.standard_normal((pool, Hkv, P, D)).astype(np.float32)
    vc = rng.standard_normal((pool, Hkv, P, Dv)).astype(np.float32)
    bt = rng.permutation(pool)[:B * maxb].reshape(B, maxb).astype(np.int32)
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    out, lse = O.paged_decode(q, kc, vc, bt, ctx, P)

    for b in range(B):
        r = torch.arange(maxb * P)
        page = torch.as_tensor(bt[b]).long()[r // P]
        kr = _t(kc)[page, :, r % P, :]                 # [maxb*P, Hkv, D]
        vr = _t(vc)[page, :, r % P, :]
        allowed = (r < int(ctx[b]))[None, :]
        ro, rl = _dense_attention(_t(q[b:b + 1]), _expand(kr, H), _expand(vr, H), allowed)
        _close(out[b], ro[0])
        _close(lse[b], rl[0])
    assert np.all(out[0] == 0) and np.all(np.isneginf(lse[0]))


# ---------------------------------------------------------------------------
# top-k sparse attention with sinks (attention/sparse_attn_fwd.py:10-98)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("with_sink", [False, True])
@pytest.mark.parametrize("shape", ["latent", "gqa"])
def test_sparse_prefill_extra_logit_form(with_sink, shape):
    rng = np.random.default_rng(7)
    if shape == "latent":          # MQA over a latent: Dqk = 40 = 32 + 8 rope, V = K[..., :32]
        H, Hkv, D, Dv = 8, 1, 40, 32
    else:
        H, Hkv, D, Dv = 8, 2, 16, 16
    T, rows, K = 9, 50, 12
    q = rng.standard_normal((T, H, D)).astype(np.float32)
    k = rng.standard_normal((rows, Hkv, D)).astype(np.float32)
    v = k[..., :Dv] if shape == "latent" else rng.standard_normal((rows, Hkv, Dv)).astype(np.float32)
    idx = np.stack([np.sort(rng.choice(rows, K, replace=False)) for _ in range(T)]).astype(np.int32)
    idx[1, 5:] = -1                      # -1 padding
    idx[2, :] = -1                       # nothing to attend to: the sink alone
    idx[3, -2:] = [rows, rows + 7]       # past the rows: masked
    sink = rng.standard_normal(H).astype(np.float32) if with_sink else None
    out, lse = O.sparse_prefill(q, k, v, idx, None, sink)

    allowed = torch.zeros(T, rows, dtype=torch.bool)
    for t in range(T):
        sel = idx[t][(idx[t] >= 0) & (idx[t] < rows)]
        allowed[t, torch.as_tensor(sel).long()] = True
    ro, rl = _dense_attention(_t(q), _expand(_t(k), H), _expand(_t(v), H), allowed,
                              None if sink is None else _t(sink))
    _close(out, ro)
    _close(lse, rl)
    assert np.all(out[2] == 0)
    if with_sink:
        _close(lse[2], sink)             # only the sink term: ln e^sink
    else:
        assert np.all(np.isneginf(lse[2]))


def test_sink_lowers_weights_by_one_shared_factor():
    """With a sink every weight is the sink-free weight times
    l / (l + e^sink), so out_sink = out * (1 - e^(sink - lse_sink))."""
    rng = np.random.default_rng(8)
    T, H, D, rows, K = 5, 4, 16, 30, 10
    q = rng.standard_normal((T, H, D))
    k = rng.standard_normal((rows, 1, D))
    idx = np.stack([rng.choice(rows, K, replace=False) for _ in range(T)]).astype(np.int32)
    sink = rng.standard_normal(H) * 3
    o0, l0 = O.sparse_prefill(q, k, k, idx)
    o1, l1 = O.sparse_prefill(q, k, k, idx, None, sink)
    _close(l1, np.logaddexp(l0, sink[None, :]))
    _close(o1, o0 * (1.0 - np.exp(sink[None, :] - l1))[..., None])


@pytest.mark.parametrize("with_sink", [False, True])
def test_sparse_decode_virtual_row_form(with_sink):
    """Decode slots by position (attention/sparse_attn_fwd.py:151-210): window
    slots are logical positions < ctx read through the block table, later
    slots are compressed rows idx - ctx (idx >= ctx)."""
    rng = np.random.default_rng(9)
    H, Hkv, D, Dv, P, pool, maxb = 8, 1, 24, 16, 4, 30, 5
    ctx = np.array([0, 3, 17, 20], np.int32)
    B, nc, nwin, K = len(ctx), 7, 4, 9
    kc = rng.standard_normal((pool, Hkv, P, D))
    vc = kc[..., :Dv]
    ck = rng.standard_normal((nc, Hkv, D))
    cv = ck[..., :Dv]
    bt = rng.permutation(pool)[:B * maxb].reshape(B, maxb).astype(np.int32)
    q = rng.standard_normal((B, H, D))
    idx = np.full((B, K), -1, np.int32)
    for b in range(B):
        c = int(ctx[b])
        idx[b, :nwin] = [c - nwin + i if c - nwin + i >= 0 else -1 for i in range(nwin)]
        comp = rng.choice(nc, K - nwin - 1, replace=False) + c
        idx[b, nwin:K - 1] = comp
    idx[2, 0] = 17          # a window slot at ctx: invalid
    idx[3, nwin] = 4        # a compressed slot below ctx: invalid
    idx[3, -1] = 20 + nc    # past the compressed rows: invalid
    sink = rng.standard_normal(H) if with_sink else None
    out, lse = O.sparse_decode(q, kc, vc, ck, cv, bt, idx, ctx, nwin, P, sink)

    for b in range(B):
        c = int(ctx[b])
        r = torch.arange(maxb * P)
        page = torch.as_tensor(bt[b]).long()[r // P]
        kr = torch.cat([_t(kc)[page, :, r % P, :], _t(ck)])          # virtual rows: positions, then compressed
        vr = torch.cat([_t(vc)[page, :, r % P, :], _t(cv)])
        allowed = torch.zeros(1, kr.shape[0], dtype=torch.bool)
        for j, x in enumerate(idx[b]):
            x = int(x)
            if j < nwin and 0 <= x < c:
                allowed[0, x] = True
            elif j >= nwin and x >= c and x - c < nc:
                allowed[0, maxb * P + x - c] = True
        ro, rl = _dense_attention(_t(q[b:b + 1]), _expand(kr, H), _expand(vr, H), allowed,
                                  None if sink is None else _t(sink))
        _close(out[b], ro[0])
        _close(lse[b], rl[0])


# ---------------------------------------------------------------------------
# window pooling (attention/csa.py:9-69, attention/hca.py:9-69)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("stride,window", [(4, 8), (128, 128), (3, 6), (5, 5)])
def test_mean_pooling_prefix_sum_form(stride, window):
    rng = np.random.default_rng(13)
    lens = [1, 3, 4, 9, 0, 130, 257]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    k = rng.standard_normal((T, 2, 8))
    v = rng.standard_normal((T, 2, 5))
    ck, cv, offs = O.compress_kv(k, v, cu, stride, window)
    for x, cx in ((k, ck), (v, cv)):
        pre = torch.cat([torch.zeros(1, *x.shape[1:], dtype=torch.float64), torch.cumsum(_t(x), 0)])
        for s in range(len(lens)):
            L, s0 = lens[s], int(cu[s])
            n = int(offs[s + 1] - offs[s])
            assert n == (max(1, -(-L // stride)) if L else 0)
            for i in range(n):
                a, b = s0 + i * stride, s0 + min(i * stride + window, L)
                _close(cx[offs[s] + i], (pre[b] - pre[a]) / (b - a))


def test_gated_pooling_explicit_softmax():
    rng = np.random.default_rng(17)
    lens = [11, 6]
    cu = np.array([0, 11, 17], np.int32)
    k = rng.standard_normal((17, 1, 6))
    v = rng.standard_normal((17, 1, 4))
    g = rng.standard_normal(17) * 4
    ck, cv, offs = O.compress_kv(k, v, cu, 4, 8, gate=g)
    for s in range(2):
        for i in range(int(offs[s + 1] - offs[s])):
            a = int(cu[s]) + 4 * i
            b = int(cu[s]) + min(4 * i + 8, lens[s])
            w = torch.softmax(_t(g[a:b]), 0)
            _close(ck[offs[s] + i], torch.einsum("r,rhd->hd", w, _t(k[a:b])))
            _close(cv[offs[s] + i], torch.einsum("r,rhd->hd", w, _t(v[a:b])))

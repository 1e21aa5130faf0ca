"""CPU oracle for the attention hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the math of suluner/triton-ascend-kernels'
``attention/*.py`` so that the CUDA kernels of this repository can be checked
against it.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg may import it; the product path (``attention/*.py`` modules of the
package) never calls into it and fails loudly when its CUDA library is missing.

Pinning: every function below is checked against golden vectors produced by the
reference's own ``torch_*_reference`` functions (fp16, on CPU) for the
reference's runner configurations; see ``tests/golden/make_golden.py`` and
``tests/test_oracle_golden.py``.

Conventions shared by every function (same as the reference):
  * ``scale = 1/sqrt(q.shape[-1])``                      (FP:136, PD:132, SA:295)
  * GQA head map ``kv_head = h // (H // H_kv)``           (FP:34, PD:34, SA:34)
  * results are returned as float arrays of the accumulation dtype
    (``acc``, float64 by default); the log-sum-exp ``lse[t, h]`` is the natural
    log of the softmax denominator (sink term included), ``-inf`` when the
    denominator is zero.  The reference computes no LSE; it is an addition.

Citations use the reference file names: FP = flash_attention_prefill.py,
PD = paged_attention_decode.py, SA = sparse_attn_fwd.py, CSA = csa.py,
HCA = hca.py (all under ``attention/``).
"""

from __future__ import annotations

import math

import numpy as np

NEG_INF = -np.inf


def _np(x, dtype=None):
    """Accept numpy arrays or torch tensors (CPU) and return a numpy array."""
    if hasattr(x, "detach"):
        x = x.detach().cpu()
        if str(x.dtype) == "torch.bfloat16":
            x = x.float()
        x = x.numpy()
    x = np.asarray(x)
    return x.astype(dtype) if dtype is not None else x


def _bounds(cu_seqlens):
    cu = _np(cu_seqlens).astype(np.int64)
    return [(int(cu[i]), int(cu[i + 1])) for i in range(cu.shape[0] - 1)]


def _softmax_rows(scores, sink=None):
    """Row softmax of ``scores [..., N]`` with an optional extra logit ``sink``
    that enters only the denominator (SA:86-95, SA:421-423).

    Returns (p, l, m): unnormalised weights, denominator, row max (the sink
    counts towards the max).  Rows with no finite entry and no sink get l = 0.
    """
    m = np.max(scores, axis=-1, initial=NEG_INF) if scores.shape[-1] else np.full(scores.shape[:-1], NEG_INF)
    if sink is not None:
        m = np.maximum(m, sink)
    m_safe = np.where(np.isfinite(m), m, 0.0)
    p = np.exp(scores - m_safe[..., None])
    l = p.sum(axis=-1)
    if sink is not None:
        l = l + np.exp(sink - m_safe)
    return p, l, m_safe


def _finish(p, l, m, vals):
    """out = p @ vals / l (0 where l == 0, SA:94-95); lse = m + ln l."""
    l_safe = np.where(l > 0, l, 1.0)
    out = (p @ vals) / l_safe[..., None]
    with np.errstate(divide="ignore"):
        lse = np.where(l > 0, m + np.log(np.where(l > 0, l, 1.0)), NEG_INF)
    return out, lse


# ---------------------------------------------------------------------------
# Dense varlen prefill  (FP:177-229; kernel FP:11-102)
# ---------------------------------------------------------------------------

def prefill(q, k, v, cu_seqlens, causal=True, acc=np.float64):
    """Varlen flash prefill over TND-packed sequences.

    q [T,H,D], k/v [T,H_kv,D(v)], cu_seqlens [S+1].  Row i of a sequence sees
    keys j <= i when causal (``triu`` mask, FP:218).  Tokens outside every
    sequence keep out = 0, lse = -inf (FP:189 zero init).
    """
    q, k, v = _np(q, acc), _np(k, acc), _np(v, acc)
    T, H, D = q.shape
    Hkv, Dv = k.shape[1], v.shape[2]
    G = H // Hkv
    scale = 1.0 / math.sqrt(D)
    out = np.zeros((T, H, Dv), acc)
    lse = np.full((T, H), NEG_INF, acc)
    for start, end in _bounds(cu_seqlens):
        L = end - start
        if L <= 0:
            continue
        for g in range(Hkv):
            qg = q[start:end, g * G:(g + 1) * G, :].transpose(1, 0, 2)  # [G,L,D]
            kg = k[start:end, g, :]
            vg = v[start:end, g, :]
            s = (qg @ kg.T) * scale                                      # [G,L,L]
            if causal:
                s = np.where(np.triu(np.ones((L, L), bool), 1)[None], NEG_INF, s)
            p, l, m = _softmax_rows(s)
            o, ls = _finish(p, l, m, vg)
            out[start:end, g * G:(g + 1) * G, :] = o.transpose(1, 0, 2)
            lse[start:end, g * G:(g + 1) * G] = ls.T
    return out, lse


def prefill_rows(q, k, v, cu_seqlens, rows, causal=True, acc=np.float64):
    """The rows ``rows`` (global token indices) of :func:`prefill`, computed
    without the full [L, L] score matrix -- the same math (FP:177-229: scores
    ``scale * q k^T``, causal ``triu`` mask FP:218, softmax, ``@ v``), so that
    sequences of tens of thousands of tokens can be checked row by row.

    Returns (out [len(rows), H, Dv], lse [len(rows), H]); a row outside every
    sequence gives out = 0, lse = -inf (FP:189).
    """
    rows = np.asarray(rows, dtype=np.int64)
    T, H, D = q.shape
    Hkv, Dv = k.shape[1], v.shape[2]
    G = H // Hkv
    scale = 1.0 / math.sqrt(D)
    bounds = _bounds(cu_seqlens)
    out = np.zeros((rows.shape[0], H, Dv), acc)
    lse = np.full((rows.shape[0], H), NEG_INF, acc)
    for start, end in bounds:
        sel = np.nonzero((rows >= start) & (rows < end))[0]
        if sel.size == 0:
            continue
        pos = rows[sel] - start                                           # position in the sequence
        kl = end if not causal else start + int(pos.max()) + 1            # keys any selected row sees
        qs = _np(q[rows[sel]], acc)                                       # [n, H, D]
        ks = _np(k[start:kl], acc)                                        # [Lk, Hkv, D]
        vs = _np(v[start:kl], acc)
        for g in range(Hkv):
            qg = qs[:, g * G:(g + 1) * G, :].transpose(1, 0, 2)           # [G, n, D]
            s = (qg @ ks[:, g, :].T) * scale                              # [G, n, Lk]
            if causal:
                s = np.where(np.arange(kl - start)[None, None, :] > pos[None, :, None], NEG_INF, s)
            p, l, m = _softmax_rows(s)
            o, ls = _finish(p, l, m, vs[:, g, :])
            out[sel, g * G:(g + 1) * G, :] = o.transpose(1, 0, 2)
            lse[sel, g * G:(g + 1) * G] = ls.T
    return out, lse


# ---------------------------------------------------------------------------
# Paged decode  (PD:157-202; kernel PD:11-98)
# ---------------------------------------------------------------------------

def gather_pages(cache, table_row, ctx, block_size):
    """Logical rows [0, ctx) of one sequence out of a paged cache
    ``[num_blocks, H_kv, P, D]`` -> [H_kv, ctx, D]  (PD:177-186)."""
    n_pages = -(-ctx // block_size)
    parts = [cache[int(table_row[j]), :, :block_size, :] for j in range(n_pages)]
    if not parts:
        return cache[:0, :, :0, :].reshape(cache.shape[1], 0, cache.shape[3])
    return np.concatenate(parts, axis=1)[:, :ctx, :]


def paged_decode(q, k_cache, v_cache, block_tables, context_lens, block_size=16, acc=np.float64):
    """One query token per sequence against a paged KV cache.

    A sequence with context length 0 yields out = 0, lse = -inf (the reference
    leaves this case undefined: its torch path raises on an empty concat).
    """
    q = _np(q, acc)
    k_cache, v_cache = _np(k_cache, acc), _np(v_cache, acc)
    bt, cl = _np(block_tables).astype(np.int64), _np(context_lens).astype(np.int64)
    B, H, D = q.shape
    Hkv = k_cache.shape[1]
    G = H // Hkv
    scale = 1.0 / math.sqrt(D)
    out = np.zeros((B, H, v_cache.shape[3]), acc)
    lse = np.full((B, H), NEG_INF, acc)
    for i in range(B):
        ctx = int(cl[i])
        if ctx <= 0:
            continue
        ks = gather_pages(k_cache, bt[i], ctx, block_size)
        vs = gather_pages(v_cache, bt[i], ctx, block_size)
        for g in range(Hkv):
            qg = q[i, g * G:(g + 1) * G, :]                 # [G,D]
            s = (qg @ ks[g].T) * scale                      # [G,ctx]
            p, l, m = _softmax_rows(s)
            o, ls = _finish(p, l, m, vs[g])
            out[i, g * G:(g + 1) * G] = o
            lse[i, g * G:(g + 1) * G] = ls
    return out, lse


# ---------------------------------------------------------------------------
# Top-k sparse attention with sinks  (kernels SA:10-98, SA:105-246;
# torch references SA:389-426, SA:429-470)
# ---------------------------------------------------------------------------

def sparse_prefill(q, k, v, topk_idxs, cu_seqlens=None, attn_sink=None, acc=np.float64):
    """Every token t attends to rows ``topk_idxs[t, :]`` of k/v; entries < 0 are
    masked (SA:55-57).  Entries >= k.shape[0] are treated as masked as well (the
    reference reads out of bounds there).  ``attn_sink [H]`` adds exp(sink_h) to
    the denominator only (SA:86-92).  As in the kernel (grid over all tokens,
    SA:296) ``cu_seqlens`` does not enter the math.  v may have a different head
    dim than q/k (MLA-style latent: Dqk = 576, Dv = 512).
    """
    q, k, v = _np(q, acc), _np(k, acc), _np(v, acc)
    idx = _np(topk_idxs).astype(np.int64)
    sink = None if attn_sink is None else _np(attn_sink, acc)
    T, H, D = q.shape
    Hkv, Dv, rows = k.shape[1], v.shape[2], k.shape[0]
    G = H // Hkv
    scale = 1.0 / math.sqrt(D)
    out = np.zeros((T, H, Dv), acc)
    lse = np.full((T, H), NEG_INF, acc)
    for t in range(T):
        sel = idx[t][(idx[t] >= 0) & (idx[t] < rows)]
        for g in range(Hkv):
            kg, vg = k[sel, g, :], v[sel, g, :]
            qg = q[t, g * G:(g + 1) * G, :]
            s = (qg @ kg.T) * scale
            p, l, m = _softmax_rows(s, None if sink is None else sink[g * G:(g + 1) * G])
            o, ls = _finish(p, l, m, vg)
            out[t, g * G:(g + 1) * G] = o
            lse[t, g * G:(g + 1) * G] = ls
    return out, lse


def sparse_decode(q, k_cache, v_cache, compressed_k, compressed_v, block_tables, topk_idxs,
                  context_lens, num_win, block_size=16, attn_sink=None, acc=np.float64):
    """Decode form, with the kernel's slot-position semantics (SA:151-210):
    slots [0, num_win) are valid iff 0 <= idx < ctx and address the paged cache
    (page ``block_tables[s, idx // P]``, row ``idx % P``); slots [num_win, K)
    are valid iff idx >= ctx and address ``compressed[idx - ctx]`` (bounded by
    the compressed row count here).  On index rows built by the reference's own
    builders this equals the torch reference's value-based rule (SA:451-459).
    """
    q = _np(q, acc)
    kc, vc = _np(k_cache, acc), _np(v_cache, acc)
    ck, cv = _np(compressed_k, acc), _np(compressed_v, acc)
    bt, cl = _np(block_tables).astype(np.int64), _np(context_lens).astype(np.int64)
    idx = _np(topk_idxs).astype(np.int64)
    sink = None if attn_sink is None else _np(attn_sink, acc)
    B, H, D = q.shape
    Hkv = kc.shape[1]
    G = H // Hkv
    K = idx.shape[1]
    nc = ck.shape[0]
    scale = 1.0 / math.sqrt(D)
    out = np.zeros((B, H, vc.shape[3]), acc)
    lse = np.full((B, H), NEG_INF, acc)
    for s in range(B):
        ctx = int(cl[s])
        krows, vrows = [], []
        for j in range(K):
            r = int(idx[s, j])
            if j < num_win:
                if 0 <= r < ctx:
                    pg, off = int(bt[s, r // block_size]), r % block_size
                    krows.append(kc[pg, :, off, :])
                    vrows.append(vc[pg, :, off, :])
            elif r >= ctx and r - ctx < nc:
                krows.append(ck[r - ctx])
                vrows.append(cv[r - ctx])
        if krows:
            ks, vs = np.stack(krows, 1), np.stack(vrows, 1)           # [Hkv,N,D]
        else:
            ks = np.zeros((Hkv, 0, D), acc)
            vs = np.zeros((Hkv, 0, vc.shape[3]), acc)
        for g in range(Hkv):
            qg = q[s, g * G:(g + 1) * G, :]
            sc = (qg @ ks[g].T) * scale
            p, l, m = _softmax_rows(sc, None if sink is None else sink[g * G:(g + 1) * G])
            o, ls = _finish(p, l, m, vs[g])
            out[s, g * G:(g + 1) * G] = o
            lse[s, g * G:(g + 1) * G] = ls
    return out, lse


def build_token_to_seq(cu_seqlens, total_tokens):
    """token -> sequence id, 0 for tokens outside every sequence (SA:253-260)."""
    t2s = np.zeros(total_tokens, np.int32)
    for i, (s, e) in enumerate(_bounds(cu_seqlens)):
        if e > s:
            t2s[s:e] = i
    return t2s


# ---------------------------------------------------------------------------
# KV compression  (CSA:9-69 overlap pooling; HCA:9-69 simple pooling)
# ---------------------------------------------------------------------------

def comp_offsets_for(lengths, stride):
    """n_c = max(1, ceil(L/stride)) slots for L > 0, none for L = 0; cumulative
    offsets [S+1] (CSA:38-45, CSA:59, CSA:68)."""
    offs = [0]
    for L in lengths:
        offs.append(offs[-1] + (max(1, -(-int(L) // stride)) if L > 0 else 0))
    return np.asarray(offs, np.int32)


def compress_kv(k, v, cu_seqlens, stride, window, gate=None, acc=np.float64):
    """Window pooling of K and V per sequence.

    Slot i of a sequence pools rows [i*stride, min(i*stride + window, L)).
    CSA: window = 2m, stride = m (CSA:49-55); HCA: window = stride = m'
    (HCA:49-55).  ``gate=None`` gives the reference's plain mean; ``gate [T]``
    (fp32 logits) gives the softmax(gate)-weighted sum over the window's rows --
    an extension with no counterpart in the reference (parity unpinned there).
    A -inf logit masks its row (weight 0); a window whose logits are all -inf
    pools to zeros.
    Returns (ck [Nc,H_kv,D], cv [Nc,H_kv,Dv], comp_offsets [S+1] int32).
    """
    k, v = _np(k, acc), _np(v, acc)
    g = None if gate is None else _np(gate, acc)
    bounds = _bounds(cu_seqlens)
    offs = comp_offsets_for([e - s for s, e in bounds], stride)
    nc = int(offs[-1])
    ck = np.zeros((nc,) + k.shape[1:], acc)
    cv = np.zeros((nc,) + v.shape[1:], acc)
    for si, (s, e) in enumerate(bounds):
        L = e - s
        for i in range(int(offs[si + 1] - offs[si])):
            a, b = s + i * stride, s + min(i * stride + window, L)
            if g is None:
                ck[offs[si] + i] = k[a:b].mean(0)
                cv[offs[si] + i] = v[a:b].mean(0)
            else:
                gmax = g[a:b].max()
                if gmax == -np.inf:  # every row masked
                    continue
                w = np.exp(g[a:b] - gmax)
                w = w / w.sum()
                ck[offs[si] + i] = np.tensordot(w, k[a:b], 1)
                cv[offs[si] + i] = np.tensordot(w, v[a:b], 1)
    return ck, cv, offs


# ---------------------------------------------------------------------------
# Index builders  (CSA:76-164, HCA:76-146, decode forms CSA:259-302, HCA:234-259)
# ---------------------------------------------------------------------------

def build_window_idxs(cu_seqlens, total_tokens, n_win):
    """Sliding-window part: slot wi of token (seq start s0, local pos p) holds
    s0 + p - n_win + 1 + wi when that is >= s0, else -1 (CSA:108-117)."""
    out = np.full((total_tokens, n_win), -1, np.int32)
    for s0, e in _bounds(cu_seqlens):
        for p in range(e - s0):
            for wi in range(n_win):
                src = p - n_win + 1 + wi
                if src >= 0:
                    out[s0 + p, wi] = s0 + src
    return out


def hca_max_n_comp(lengths, offs, m_prime):
    """max over sequences of min(n_comp_s, ceil(L/m')) (HCA:103-115)."""
    best = 0
    for i, L in enumerate(lengths):
        best = max(best, min(int(offs[i + 1] - offs[i]), -(-int(L) // m_prime)))
    return best


def build_hca_topk_idxs(cu_seqlens, comp_offsets, total_tokens, n_win, m_prime):
    """[T, n_win + max_n_comp]: window part, then compressed slots
    ci < min(ceil(p/m'), max_n_comp) as total_tokens + comp_offsets[s] + ci
    (HCA:117-144)."""
    bounds = _bounds(cu_seqlens)
    offs = _np(comp_offsets).astype(np.int64)
    mx = hca_max_n_comp([e - s for s, e in bounds], offs, m_prime)
    out = np.full((total_tokens, n_win + mx), -1, np.int32)
    out[:, :n_win] = build_window_idxs(cu_seqlens, total_tokens, n_win)
    for si, (s0, e) in enumerate(bounds):
        for p in range(e - s0):
            n_causal = min(-(-p // m_prime), mx)
            out[s0 + p, n_win:n_win + n_causal] = total_tokens + offs[si] + np.arange(n_causal)
    return out


def round_to(x, dtype_name):
    """Round float scores to the storage precision the reference's indexer
    matmul returns them in (its output dtype is the input dtype, CSA:144)."""
    if dtype_name == "float16":
        return x.astype(np.float16).astype(np.float64)
    if dtype_name == "bfloat16":
        u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
        u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16          # round to nearest even
        return u.astype(np.uint32).view(np.float32).astype(np.float64)
    return np.asarray(x, np.float32).astype(np.float64)


def topk_order(scores, valid, k_sel):
    """Indices of the k_sel best slots: finite (valid) scores in descending
    order, ties broken by the lower slot index; then, if fewer than k_sel slots
    are valid, the masked slots in ascending index order.  This is the
    deterministic rule of this repository for the ``torch.topk`` call of
    CSA:153 / CSA:296, whose order among equal values (in particular among the
    masked -inf slots) is backend-defined."""
    n = scores.shape[0]
    cand = np.nonzero(valid)[0]
    order = cand[np.lexsort((cand, -scores[cand]))]
    if order.shape[0] < k_sel:
        rest = np.nonzero(~valid)[0]
        order = np.concatenate([order, rest])
    return order[:k_sel]


def csa_indexer_scores(qrow, ck_rows, dtype_name):
    """Unscaled q . k~ of the Lightning indexer (CSA:144), rounded to dtype."""
    return round_to(ck_rows @ qrow, dtype_name)


def build_csa_topk_idxs(q, compressed_k, cu_seqlens, comp_offsets, n_win, top_k, m, dtype_name="float32"):
    """[T, n_win + top_k] int32.  Window part as CSA:108-117.  Compressed part:
    the reference writes every head's top-k into the same row, so the last query
    head (H-1, against KV head H_kv-1) decides it (CSA:136-162).  Slot i of the
    sequence is causal iff i*m < p (CSA:149); k_sel = min(top_k, n_c)
    (CSA:152); entry = total_tokens + comp_offsets[s] + i (CSA:162)."""
    qn = _np(q, np.float64)
    ckn = _np(compressed_k, np.float64)
    T = qn.shape[0]
    offs = _np(comp_offsets).astype(np.int64)
    out = np.full((T, n_win + top_k), -1, np.int32)
    out[:, :n_win] = build_window_idxs(cu_seqlens, T, n_win)
    for si, (s0, e) in enumerate(_bounds(cu_seqlens)):
        c0, c1 = int(offs[si]), int(offs[si + 1])
        nc = c1 - c0
        if e - s0 == 0 or nc == 0:
            continue
        k_sel = min(top_k, nc)
        kr = ckn[c0:c1, -1, :]
        slots = np.arange(nc)
        for p in range(e - s0):
            sc = csa_indexer_scores(qn[s0 + p, -1, :], kr, dtype_name)
            order = topk_order(sc, slots * m < p, k_sel)
            out[s0 + p, n_win:n_win + k_sel] = T + c0 + order
    return out


def decode_window_idxs(context_lens, n_win):
    """Decode window part: slot wi = ctx - n_win + wi when >= 0 (CSA:270-273)."""
    cl = _np(context_lens).astype(np.int64)
    out = np.full((cl.shape[0], n_win), -1, np.int32)
    for s, ctx in enumerate(cl):
        for wi in range(n_win):
            pos = int(ctx) - n_win + wi
            if pos >= 0:
                out[s, wi] = pos
    return out


def csa_decode_idxs(q, compressed_k, context_lens, comp_offsets, n_win, top_k, m, dtype_name="float32"):
    """Decode index rows of csa_decode_forward (CSA:259-302): causal iff
    i*m < ctx; entry = ctx + comp_offsets[s] + i."""
    qn = _np(q, np.float64)
    ckn = _np(compressed_k, np.float64)
    cl = _np(context_lens).astype(np.int64)
    offs = _np(comp_offsets).astype(np.int64)
    B = qn.shape[0]
    out = np.full((B, n_win + top_k), -1, np.int32)
    out[:, :n_win] = decode_window_idxs(cl, n_win)
    for s in range(B):
        ctx = int(cl[s])
        c0, c1 = int(offs[s]), int(offs[s + 1])
        nc = c1 - c0
        if nc == 0:
            continue
        k_sel = min(top_k, nc)
        sc = csa_indexer_scores(qn[s, -1, :], ckn[c0:c1, -1, :], dtype_name)
        order = topk_order(sc, np.arange(nc) * m < ctx, k_sel)
        out[s, n_win:n_win + k_sel] = ctx + c0 + order
    return out


def hca_decode_idxs(context_lens, comp_offsets, n_win, m_prime):
    """Decode index rows of hca_decode_forward (HCA:234-259)."""
    cl = _np(context_lens).astype(np.int64)
    offs = _np(comp_offsets).astype(np.int64)
    B = cl.shape[0]
    mx = hca_max_n_comp(cl, offs, m_prime)
    out = np.full((B, n_win + mx), -1, np.int32)
    out[:, :n_win] = decode_window_idxs(cl, n_win)
    for s in range(B):
        ctx = int(cl[s])
        n_causal = min(-(-ctx // m_prime), int(offs[s + 1] - offs[s]), mx)
        out[s, n_win:n_win + n_causal] = ctx + offs[s] + np.arange(n_causal)
    return out


def gather_paged_to_tnd(cache, block_tables, context_lens, block_size):
    """Concatenate each sequence's first ctx rows of a paged cache into TND
    layout [sum ctx, H_kv, D] with cu_seqlens (CSA:226-253)."""
    c = _np(cache)
    bt, cl = _np(block_tables).astype(np.int64), _np(context_lens).astype(np.int64)
    parts, cu = [], [0]
    for s in range(cl.shape[0]):
        ctx = int(cl[s])
        parts.append(gather_pages(c, bt[s], ctx, block_size).transpose(1, 0, 2))
        cu.append(cu[-1] + ctx)
    tnd = np.concatenate(parts, 0) if parts else c[:0, :, 0, :]
    return tnd, np.asarray(cu, np.int32)


# ---------------------------------------------------------------------------
# Composite forwards  (CSA:171-306, HCA:153-263)
# ---------------------------------------------------------------------------

def csa_prefill_forward(q, k, v, cu_seqlens, n_win, top_k, m, attn_sink=None, dtype_name="float32"):
    ck, cv, offs = compress_kv(k, v, cu_seqlens, m, 2 * m)
    idx = build_csa_topk_idxs(q, round_to(ck, dtype_name), cu_seqlens, offs, n_win, top_k, m, dtype_name)
    kf = np.concatenate([_np(k, np.float64), round_to(ck, dtype_name)], 0)
    vf = np.concatenate([_np(v, np.float64), round_to(cv, dtype_name)], 0)
    out, lse = sparse_prefill(q, kf, vf, idx, cu_seqlens, attn_sink)
    return out, lse, idx


def hca_prefill_forward(q, k, v, cu_seqlens, n_win, m_prime, attn_sink=None, dtype_name="float32"):
    ck, cv, offs = compress_kv(k, v, cu_seqlens, m_prime, m_prime)
    T = _np(q).shape[0]
    idx = build_hca_topk_idxs(cu_seqlens, offs, T, n_win, m_prime)
    kf = np.concatenate([_np(k, np.float64), round_to(ck, dtype_name)], 0)
    vf = np.concatenate([_np(v, np.float64), round_to(cv, dtype_name)], 0)
    out, lse = sparse_prefill(q, kf, vf, idx, cu_seqlens, attn_sink)
    return out, lse, idx


def _decode_compress(k_cache, v_cache, block_tables, context_lens, block_size, stride, window, dtype_name):
    kt, cu = gather_paged_to_tnd(k_cache, block_tables, context_lens, block_size)
    vt, _ = gather_paged_to_tnd(v_cache, block_tables, context_lens, block_size)
    ck, cv, offs = compress_kv(kt, vt, cu, stride, window)
    return round_to(ck, dtype_name), round_to(cv, dtype_name), offs


def csa_decode_forward(q, k_cache, v_cache, block_tables, context_lens, n_win, top_k, m,
                       block_size=16, attn_sink=None, dtype_name="float32"):
    ck, cv, offs = _decode_compress(k_cache, v_cache, block_tables, context_lens, block_size, m, 2 * m, dtype_name)
    idx = csa_decode_idxs(q, ck, context_lens, offs, n_win, top_k, m, dtype_name)
    out, lse = sparse_decode(q, k_cache, v_cache, ck, cv, block_tables, idx, context_lens, n_win,
                             block_size, attn_sink)
    return out, lse, idx


def hca_decode_forward(q, k_cache, v_cache, block_tables, context_lens, n_win, m_prime,
                       block_size=16, attn_sink=None, dtype_name="float32"):
    ck, cv, offs = _decode_compress(k_cache, v_cache, block_tables, context_lens, block_size,
                                    m_prime, m_prime, dtype_name)
    idx = hca_decode_idxs(context_lens, offs, n_win, m_prime)
    out, lse = sparse_decode(q, k_cache, v_cache, ck, cv, block_tables, idx, context_lens, n_win,
                             block_size, attn_sink)
    return out, lse, idx

"""CSA: overlapping KV compression + Lightning-indexer top-k sparse attention on B200.

Drop-in for attention/csa.py of suluner/triton-ascend-kernels: the public
functions keep the reference's names, arguments, defaults and return values
(CSA:9-306).  Compression, index building and attention run as sm_100a kernels
of libtak_b200.so; the host only sizes outputs (one small device->host copy of
the sequence lengths, as the reference).

Index rows follow the reference exactly except where it is itself undefined:
among exactly equal indexer scores (and among the masked slots it picks when a
query has fewer than top_k causal slots) torch.topk's order is backend-defined;
here ties go to the lower slot and masked picks come in ascending slot order.
"""

import _tak_b200 as _t
from sparse_attn_fwd import sparse_attn_prefill, sparse_attn_prefill_two_sources, sparse_attn_decode

torch = _t.torch


def compress_kv_overlap(k, v, cu_seqlens, m, *, gate=None):
    """CSA-style overlapping pooling: kernel_size = 2*m, stride = m.

    Args:
        k, v: [total_tokens, num_kv_heads, head_dim]
        cu_seqlens: [num_seqs + 1]
        m: compression stride
        gate: (keyword-only addition) optional [total_tokens] float32 logits;
            each slot is then the softmax(gate)-weighted sum of its window
            instead of the mean

    Returns:
        compressed_k, compressed_v: [total_compressed, num_kv_heads, head_dim]
        comp_offsets: [num_seqs + 1] int32 cumulative offsets
    """
    return _t.compress_tnd(k, v, cu_seqlens, m, 2 * m, gate)


def compress_kv_csa_hca(k, v, cu_seqlens, m, m_prime, *, gate=None):
    """compress_kv_overlap(k, v, cu_seqlens, m) and hca.compress_kv_simple(k,
    v, cu_seqlens, m_prime) of the same K/V (and gate) in one pass over K/V.

    Returns ((csa_k, csa_v, csa_offsets), (hca_k, hca_v, hca_offsets)), each
    triple as the single-stride function returns it.
    """
    return _t.compress_csa_hca(k, v, cu_seqlens, m, m_prime, gate)


def build_csa_topk_idxs(q, compressed_k, cu_seqlens, comp_offsets, n_win, top_k, m):
    """topk_idxs [total_tokens, n_win + top_k] int32, -1 for padding:
    [n_win sliding-window positions] + [top_k compressed indices + total_tokens]."""
    _t.require_cuda(q, compressed_k)
    dev = q.device
    total_tokens, num_q_heads, head_dim = q.shape
    num_kv_heads = compressed_k.shape[1]
    cu = _t.as_i32(cu_seqlens, dev)
    offs = _t.as_i32(comp_offsets, dev)
    num_seqs = cu.numel() - 1
    K = n_win + top_k
    out = torch.full((total_tokens, K), -1, dtype=torch.int32, device=dev)
    L = _t.lib()
    st = _t.stream_of(q)
    if total_tokens and n_win:
        _t.check(L.tak_build_window_idxs(_t.ptr(cu), num_seqs, total_tokens, n_win, _t.ptr(out), K, st))
    mc = _t.max_comp_per_seq(offs, compressed_k.shape[0])
    if total_tokens and top_k and mc:
        # score scratch: the dot products run as tensor-core GEMM tiles (CSA:144's matmul)
        ws_bytes = L.tak_csa_indexer_workspace_size(total_tokens, mc, _t.dtype_code(q))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
        _t.check(L.tak_csa_indexer_topk(
            _t.ptr(q), _t.strides(q), _t.ptr(compressed_k), _t.strides(compressed_k), _t.ptr(cu), None, _t.ptr(offs),
            num_seqs, total_tokens, num_q_heads, num_kv_heads, head_dim, n_win, top_k, m, mc, _t.ptr(out), K,
            _t.dtype_code(q), _t.ptr(ws), ws_bytes, compressed_k.shape[0], st))
    return out


def csa_prefill_forward(q, k, v, cu_seqlens, n_win, top_k, m, attn_sink=None, *, gate=None, return_lse=False):
    """CSA prefill forward (TND layout): compress (kernel 2m, stride m), build
    topk_idxs with the Lightning indexer, sparse attention over [K | compressed K]."""
    compressed_k, compressed_v, comp_offsets = compress_kv_overlap(k, v, cu_seqlens, m, gate=gate)
    topk_idxs = build_csa_topk_idxs(q, compressed_k, cu_seqlens, comp_offsets, n_win, top_k, m)
    # the index rows address [K | compressed K] (CSA:191-192); the attention reads
    # both sources in place instead of concatenating them.  One latent tensor
    # as K and V (MLA): its compressed K and V are equal, so each gathered row
    # serves both.
    v2 = compressed_k if v is k else compressed_v
    return sparse_attn_prefill_two_sources(q, k, v, compressed_k, v2, topk_idxs, attn_sink=attn_sink,
                                           return_lse=return_lse)


def csa_decode_forward(q, k_cache, v_cache, block_tables, context_lens,
                       n_win, top_k, m, block_size=16, attn_sink=None, *, return_lse=False, max_compressed=None):
    """CSA decode forward (paged layout): compress each sequence's context
    straight from the pages, index with the Lightning indexer, sparse decode.

    max_compressed (keyword-only addition): None sizes the compressed rows
    exactly from context_lens read on the host (as the reference does); an
    int bound on sum_s max(1, ceil(ctx_s / m)) keeps everything on the device
    (no host read, so the call can be captured in a CUDA graph); a total above
    it records device error 3."""
    _t.require_cuda(q, k_cache, v_cache)
    dev = q.device
    num_seqs, num_q_heads, head_dim = q.shape
    num_kv_heads = k_cache.shape[1]
    ck, cv, offs, lens, offs_h = _t.compress_paged(k_cache, v_cache, block_tables, context_lens, block_size, m, 2 * m,
                                                   capacity=max_compressed)
    if lens is not None and sum(lens) == 0:
        out = torch.zeros_like(q)
        if return_lse:
            return out, torch.full((num_seqs, num_q_heads), float("-inf"), device=dev)
        return out
    cl = _t.as_i32(context_lens, dev)
    K = n_win + top_k
    idx = torch.empty((num_seqs, K), dtype=torch.int32, device=dev)
    L = _t.lib()
    st = _t.stream_of(q)
    _t.check(L.tak_build_decode_topk_idxs(_t.ptr(cl), _t.ptr(offs), num_seqs, n_win, top_k, 0, _t.ptr(idx), K, st))
    if offs_h is not None:
        mc = max((offs_h[i + 1] - offs_h[i] for i in range(num_seqs)), default=0)
    else:
        mc = min(_t.max_slots_per_seq(block_tables, block_size, m), ck.shape[0])
    if top_k and mc:
        ws_bytes = L.tak_csa_indexer_workspace_size(num_seqs, mc, _t.dtype_code(q))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
        _t.check(L.tak_csa_indexer_topk(
            _t.ptr(q), _t.strides(q), _t.ptr(ck), _t.strides(ck), None, _t.ptr(cl), _t.ptr(offs), num_seqs,
            num_seqs, num_q_heads, num_kv_heads, head_dim, n_win, top_k, m, mc, _t.ptr(idx), K, _t.dtype_code(q),
            _t.ptr(ws), ws_bytes, ck.shape[0], st))
    return sparse_attn_decode(q, k_cache, v_cache, ck, cv, block_tables, idx, cl, num_win=n_win,
                              block_size=block_size, attn_sink=attn_sink, return_lse=return_lse)

"""HCA: non-overlapping KV compression + all-causal-slots sparse attention on B200.

Drop-in for attention/hca.py of suluner/triton-ascend-kernels: the public
functions keep the reference's names, arguments, defaults and return values
(HCA:9-263).  Compression, index building and attention run as sm_100a kernels
of libtak_b200.so; the host only sizes outputs (one small device->host copy of
the sequence lengths and offsets, as the reference).
"""

import _tak_b200 as _t
from sparse_attn_fwd import sparse_attn_prefill, sparse_attn_prefill_two_sources, sparse_attn_decode

torch = _t.torch


def compress_kv_simple(k, v, cu_seqlens, m_prime, *, gate=None):
    """HCA-style non-overlapping pooling: kernel_size = stride = m_prime.

    Args:
        k, v: [total_tokens, num_kv_heads, head_dim]
        cu_seqlens: [num_seqs + 1]
        m_prime: compression ratio
        gate: (keyword-only addition) optional [total_tokens] float32 logits;
            each slot is then the softmax(gate)-weighted sum of its window

    Returns:
        compressed_k, compressed_v: [total_compressed, num_kv_heads, head_dim]
        comp_offsets: [num_seqs + 1] int32 cumulative offsets
    """
    return _t.compress_tnd(k, v, cu_seqlens, m_prime, m_prime, gate)


def _max_n_comp(lengths, offs, m_prime):
    """max over sequences of min(n_comp_s, ceil(L_s / m')) (HCA:103-115)."""
    best = 0
    for i, L in enumerate(lengths):
        best = max(best, min(offs[i + 1] - offs[i], -(-int(L) // m_prime)))
    return best


def build_hca_topk_idxs(cu_seqlens, comp_offsets, total_tokens, n_win, m_prime):
    """topk_idxs [total_tokens, n_win + max_n_compressed] int32, -1 for padding:
    sliding window + every compressed slot ci < ceil(pos / m_prime)."""
    dev = cu_seqlens.device if isinstance(cu_seqlens, torch.Tensor) else torch.device("cuda")
    assert dev.type == "cuda", "Tensors must be on a CUDA device"
    cu = _t.as_i32(cu_seqlens, dev)
    offs = _t.as_i32(comp_offsets, dev)
    cu_h, offs_h = cu.cpu().tolist(), offs.cpu().tolist()
    mx = _max_n_comp([cu_h[i + 1] - cu_h[i] for i in range(len(cu_h) - 1)], offs_h, m_prime)
    K = n_win + mx
    out = torch.empty((total_tokens, K), dtype=torch.int32, device=dev)
    if total_tokens and K:
        _t.check(_t.lib().tak_build_hca_topk_idxs(_t.ptr(cu), _t.ptr(offs), len(cu_h) - 1, total_tokens, n_win, mx,
                                                  m_prime, _t.ptr(out), K, _t.stream_of(out)))
    return out


def hca_prefill_forward(q, k, v, cu_seqlens, n_win, m_prime, attn_sink=None, *, gate=None, return_lse=False):
    """HCA prefill forward (TND layout): compress (kernel = stride = m'),
    index (window + all causal compressed slots), sparse attention."""
    compressed_k, compressed_v, comp_offsets = compress_kv_simple(k, v, cu_seqlens, m_prime, gate=gate)
    total_tokens = q.shape[0]
    topk_idxs = build_hca_topk_idxs(cu_seqlens, comp_offsets, total_tokens, n_win, m_prime)
    # the index rows address [K | compressed K] (HCA:173-174); the attention reads
    # both sources in place instead of concatenating them.  One latent tensor
    # as K and V (MLA): its compressed K and V are equal, so each gathered row
    # serves both.
    v2 = compressed_k if v is k else compressed_v
    return sparse_attn_prefill_two_sources(q, k, v, compressed_k, v2, topk_idxs, attn_sink=attn_sink,
                                           return_lse=return_lse)


def hca_decode_forward(q, k_cache, v_cache, block_tables, context_lens,
                       n_win, m_prime, block_size=16, attn_sink=None, *, return_lse=False, max_compressed=None):
    """HCA decode forward (paged layout): compress each sequence's context
    straight from the pages, index (window + all causal slots), sparse decode.

    max_compressed (keyword-only addition): as for csa_decode_forward; with an
    int the compressed columns of the index rows are sized from the block
    table's reach, max(1, ceil(max_blocks * P / m')), the extra columns -1."""
    _t.require_cuda(q, k_cache, v_cache)
    dev = q.device
    num_seqs, num_q_heads, _ = q.shape
    ck, cv, offs, lens, offs_h = _t.compress_paged(k_cache, v_cache, block_tables, context_lens, block_size,
                                                   m_prime, m_prime, capacity=max_compressed)
    if lens is not None and sum(lens) == 0:
        out = torch.zeros_like(q)
        if return_lse:
            return out, torch.full((num_seqs, num_q_heads), float("-inf"), device=dev)
        return out
    cl = _t.as_i32(context_lens, dev)
    if lens is not None:
        mx = _max_n_comp(lens, offs_h, m_prime)
    else:
        mx = min(_t.max_slots_per_seq(block_tables, block_size, m_prime), ck.shape[0])
    K = n_win + mx
    idx = torch.empty((num_seqs, K), dtype=torch.int32, device=dev)
    _t.check(_t.lib().tak_build_decode_topk_idxs(_t.ptr(cl), _t.ptr(offs), num_seqs, n_win, mx, m_prime,
                                                 _t.ptr(idx), K, _t.stream_of(q)))
    return sparse_attn_decode(q, k_cache, v_cache, ck, cv, block_tables, idx, cl, num_win=n_win,
                              block_size=block_size, attn_sink=attn_sink, return_lse=return_lse)

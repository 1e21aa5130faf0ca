"""Top-k sparse attention with per-head sink logits (prefill and decode) on B200.

Drop-in for attention/sparse_attn_fwd.py of suluner/triton-ascend-kernels:
``build_token_to_seq``, ``sparse_attn_prefill`` and ``sparse_attn_decode`` keep
the reference's names, arguments, defaults and assertion behaviour
(SA:253-382), running sm_100a kernels of libtak_b200.so.

Differences that only widen what is accepted:
  * v may have a different head dim than q/k (MLA-style latent KV: Dqk = 576,
    Dv = 512); the output then has v's head dim.  The reference asserts
    k.shape == v.shape (SA:279).
  * index entries >= the number of K/V rows are masked like -1 (the reference
    kernel would read out of bounds there).
"""

import math

import _tak_b200 as _t

torch = _t.torch


def build_token_to_seq(cu_seqlens, total_tokens, device):
    """token -> sequence id ([total_tokens] int32, 0 outside every sequence)."""
    dev = torch.device(device)
    assert dev.type == "cuda", "Tensors must be on a CUDA device"
    cu = _t.as_i32(cu_seqlens, dev)
    out = torch.empty(total_tokens, dtype=torch.int32, device=dev)
    if total_tokens:
        _t.check(_t.lib().tak_build_token_to_seq(_t.ptr(cu), cu.numel() - 1, total_tokens, _t.ptr(out),
                                                 _t.stream_of(out)))
    return out


def _sink_arg(attn_sink, num_q_heads, device):
    if attn_sink is None:
        return None
    assert attn_sink.shape == (num_q_heads,)
    return attn_sink.to(device=device, dtype=torch.float32).contiguous()


def sparse_attn_prefill(q, k, v, topk_idxs, cu_seqlens, attn_sink=None, *, return_lse=False):
    """Sparse attention prefill with GQA support (TND layout).

    Args:
        q:  [total_tokens, num_q_heads, head_dim]
        k:  [total_kv_tokens, num_kv_heads, head_dim]
        v:  [total_kv_tokens, num_kv_heads, head_dim_v]
        topk_idxs:  [total_tokens, K_TOPK] int32 -- indices into k/v rows, -1 = masked
        cu_seqlens: [num_seqs + 1] (does not enter the math, as in the reference kernel)
        attn_sink: optional [num_q_heads] per-head sink logit
        return_lse: (keyword-only addition) also return lse [total_tokens, num_q_heads]
    """
    _t.require_cuda(q, k, v)
    total_tokens, num_q_heads, head_dim = q.shape
    num_kv_heads = k.shape[1]

    assert num_q_heads % num_kv_heads == 0
    assert k.shape[:2] == v.shape[:2] and k.shape[2] == head_dim
    assert topk_idxs.shape[0] == total_tokens

    idx = _t.as_i32(topk_idxs, q.device)
    sink = _sink_arg(attn_sink, num_q_heads, q.device)
    head_dim_v = v.shape[2]
    out = q.new_empty((total_tokens, num_q_heads, head_dim_v))
    lse = q.new_empty((total_tokens, num_q_heads), dtype=torch.float32) if return_lse else None
    scale = 1.0 / math.sqrt(head_dim)
    _t.check(_t.lib().tak_sparse_attn_prefill(
        _t.ptr(q), _t.strides(q), _t.ptr(k), _t.strides(k), _t.ptr(v), _t.strides(v), _t.ptr(idx), _t.strides(idx),
        _t.ptr(sink), _t.ptr(out), _t.strides(out), _t.ptr(lse), total_tokens, num_q_heads, num_kv_heads,
        head_dim, head_dim_v, k.shape[0], idx.shape[1], scale, _t.dtype_code(q), _t.stream_of(q)))
    return (out, lse) if return_lse else out


def sparse_attn_prefill_two_sources(q, k, v, k2, v2, topk_idxs, attn_sink=None, *, return_lse=False):
    """sparse_attn_prefill over the rows of k/v followed by the rows of k2/v2,
    without building their concatenation (an addition used by the CSA / HCA
    forwards, whose index rows address [K | compressed K], CSA:191-194).
    Index j < k.shape[0] is row j of k/v, index j >= k.shape[0] row
    j - k.shape[0] of k2/v2; -1 and indices past both are masked."""
    _t.require_cuda(q, k, v, k2, v2)
    total_tokens, num_q_heads, head_dim = q.shape
    num_kv_heads = k.shape[1]
    assert num_q_heads % num_kv_heads == 0
    assert k.shape[1:] == k2.shape[1:] and v.shape[1:] == v2.shape[1:] and k.shape[:2] == v.shape[:2]
    assert k2.shape[0] == v2.shape[0] and topk_idxs.shape[0] == total_tokens
    idx = _t.as_i32(topk_idxs, q.device)
    sink = _sink_arg(attn_sink, num_q_heads, q.device)
    head_dim_v = v.shape[2]
    out = q.new_empty((total_tokens, num_q_heads, head_dim_v))
    lse = q.new_empty((total_tokens, num_q_heads), dtype=torch.float32) if return_lse else None
    if total_tokens:
        _t.check(_t.lib().tak_sparse_attn_prefill_2src(
            _t.ptr(q), _t.strides(q), _t.ptr(k), _t.strides(k), _t.ptr(v), _t.strides(v), k.shape[0], _t.ptr(k2),
            _t.strides(k2), _t.ptr(v2), _t.strides(v2), k2.shape[0], _t.ptr(idx), _t.strides(idx), _t.ptr(sink),
            _t.ptr(out), _t.strides(out), _t.ptr(lse), total_tokens, num_q_heads, num_kv_heads, head_dim, head_dim_v,
            idx.shape[1], 1.0 / math.sqrt(head_dim), _t.dtype_code(q), _t.stream_of(q)))
    return (out, lse) if return_lse else out


def sparse_attn_decode(q, k_cache, v_cache, compressed_k, compressed_v,
                       block_tables, topk_idxs, context_lens,
                       num_win, block_size=16, attn_sink=None, *, return_lse=False):
    """Sparse attention decode with GQA support (paged attention layout).

    Args:
        q:  [num_seqs, num_q_heads, head_dim]
        k_cache: [num_blocks, num_kv_heads, block_size, head_dim]
        v_cache: [num_blocks, num_kv_heads, block_size, head_dim_v]
        compressed_k: [num_compressed, num_kv_heads, head_dim]
        compressed_v: [num_compressed, num_kv_heads, head_dim_v]
        block_tables: [num_seqs, max_num_blocks_per_seq]
        topk_idxs: [num_seqs, K_TOPK] -- the first num_win entries are window
                   positions (valid when 0 <= idx < context_len), the rest
                   compressed indices offset by context_len (valid when
                   idx >= context_len)
        context_lens: [num_seqs]
        num_win: number of sliding-window entries in topk_idxs
        block_size: page block size
        attn_sink: optional [num_q_heads] per-head sink logit
        return_lse: (keyword-only addition) also return lse [num_seqs, num_q_heads]
    """
    _t.require_cuda(q, k_cache, v_cache)
    num_seqs, num_q_heads, head_dim = q.shape
    num_kv_heads = k_cache.shape[1]

    assert num_q_heads % num_kv_heads == 0
    assert k_cache.shape[:3] == v_cache.shape[:3]
    assert compressed_k.shape[:2] == compressed_v.shape[:2]

    bt = _t.as_i32(block_tables, q.device)
    idx = _t.as_i32(topk_idxs, q.device)
    cl = _t.as_i32(context_lens, q.device)
    sink = _sink_arg(attn_sink, num_q_heads, q.device)
    head_dim_v = v_cache.shape[3]
    out = q.new_empty((num_seqs, num_q_heads, head_dim_v))
    lse = q.new_empty((num_seqs, num_q_heads), dtype=torch.float32) if return_lse else None
    scale = 1.0 / math.sqrt(head_dim)
    ck, cv = compressed_k, compressed_v
    _t.check(_t.lib().tak_sparse_attn_decode(
        _t.ptr(q), _t.strides(q), _t.ptr(k_cache), _t.strides(k_cache), _t.ptr(v_cache), _t.strides(v_cache),
        _t.ptr(ck), _t.strides(ck), _t.ptr(cv), _t.strides(cv), _t.ptr(bt), _t.strides(bt), _t.ptr(idx),
        _t.strides(idx), _t.ptr(cl), _t.ptr(sink), _t.ptr(out), _t.strides(out), _t.ptr(lse), num_seqs,
        num_q_heads, num_kv_heads, head_dim, head_dim_v, ck.shape[0], idx.shape[1], num_win, block_size,
        bt.shape[1], k_cache.shape[0], scale, _t.dtype_code(q), _t.stream_of(q)))
    return (out, lse) if return_lse else out

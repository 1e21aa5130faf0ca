"""Paged attention decode (MHA / GQA / MQA) on B200.

Drop-in for attention/paged_attention_decode.py of suluner/triton-ascend-kernels:
same function name, arguments, defaults and assertion behaviour (PD:104-151),
running the split-KV sm_100a kernel of libtak_b200.so.
"""

import math

import _tak_b200 as _t


def paged_attention_decode(q, k_cache, v_cache, block_tables, context_lens, block_size=16, block_n=16, *,
                           return_lse=False, split_pages=0):
    """Paged attention decode with GQA/MQA/MHA support.

    Args:
        q:        [num_seqs, num_q_heads, head_dim]
        k_cache:  [num_blocks, num_kv_heads, block_size, head_dim]
        v_cache:  [num_blocks, num_kv_heads, block_size, head_dim]
        block_tables: [num_seqs, max_num_blocks_per_seq] int32 page ids
        context_lens: [num_seqs] int32
        block_size: rows per page used for the page arithmetic
        block_n: tile hint of the reference kernel; validated as there
            (PD:121-123), the B200 kernel picks its own tiles
        return_lse: (keyword-only addition) also return lse [num_seqs,
            num_q_heads] float32 (natural log of the softmax denominator)
        split_pages: (keyword-only addition) pages per split-KV work unit,
            0 = automatic

    A sequence with context length 0 yields zeros (lse -inf); the reference
    leaves that case undefined.
    """
    _t.require_cuda(q, k_cache, v_cache)
    assert block_n <= block_size and block_size % block_n == 0, \
        f"block_n ({block_n}) must be <= block_size ({block_size}) and divide it evenly: " \
        f"a single BLOCK_N iteration cannot span multiple paged physical blocks"

    num_seqs, num_q_heads, head_dim = q.shape
    num_kv_heads = k_cache.shape[1]

    assert num_q_heads % num_kv_heads == 0, \
        f"num_q_heads ({num_q_heads}) must be divisible by num_kv_heads ({num_kv_heads})"

    out = q.new_empty(q.shape)
    lse = q.new_empty((num_seqs, num_q_heads), dtype=_t.torch.float32) if return_lse else None
    scale = 1.0 / math.sqrt(head_dim)
    bt = _t.as_i32(block_tables, q.device)
    cl = _t.as_i32(context_lens, q.device)
    max_blocks = bt.shape[1]
    L = _t.lib()
    st = _t.stream_of(q)
    ws_bytes = L.tak_paged_attention_decode_workspace_size(num_seqs, num_q_heads, num_kv_heads, head_dim,
                                                           block_size, max_blocks, int(split_pages))
    ws = _t.workspace(q.device, st, ws_bytes)
    _t.check(L.tak_paged_attention_decode(
        _t.ptr(q), _t.strides(q), _t.ptr(k_cache), _t.strides(k_cache), _t.ptr(v_cache), _t.strides(v_cache),
        _t.ptr(bt), _t.strides(bt), _t.ptr(cl), _t.ptr(out), _t.strides(out), _t.ptr(lse),
        num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, max_blocks, k_cache.shape[0],
        k_cache.shape[2], scale, _t.dtype_code(q), _t.ptr(ws), ws.numel(), int(split_pages), st))
    return (out, lse) if return_lse else out

"""A serving step's varlen prefill and paged decode in one launch on B200.

An addition beside the drop-in modules: the reference runs
``flash_attention_prefill`` (FP:108-171) and ``paged_attention_decode``
(PD:104-151) as two launches; ``prefill_and_decode`` returns exactly what the
two return, computed by one persistent sm_100a kernel whose CTAs pull prefill
row blocks and decode splits from one work queue (decode spread through it,
so the HBM-bound decode overlaps the tensor-bound prefill).  Shapes that
kernel does not take (head dims other than 128, pages not a multiple of 64
rows, fp32, mixed dtypes) run the two kernels back to back.
"""

import math

import _tak_b200 as _t


def prefill_and_decode(q, k, v, cu_seqlens, q_dec, k_cache, v_cache, block_tables, context_lens, block_size,
                       causal=True, *, return_lse=False):
    """(prefill out, decode out) -- or ((out, lse), (out_dec, lse_dec)) with
    return_lse -- of flash_attention_prefill(q, k, v, cu_seqlens, causal) and
    paged_attention_decode(q_dec, k_cache, v_cache, block_tables,
    context_lens, block_size) in one launch.  Same asserts as those two."""
    _t.require_cuda(q, k, v, q_dec, k_cache, v_cache)
    total_tokens, num_q_heads, head_dim = q.shape
    num_kv_heads = k.shape[1]
    assert num_q_heads % num_kv_heads == 0, \
        f"num_q_heads ({num_q_heads}) must be divisible by num_kv_heads ({num_kv_heads})"
    assert k.shape == v.shape, "K and V must have the same shape"
    assert k.shape[0] == total_tokens and k.shape[2] == head_dim, \
        "K/V shape must be [total_tokens, num_kv_heads, head_dim]"
    num_reqs, dec_q_heads, dec_head_dim = q_dec.shape
    dec_kv_heads = k_cache.shape[1]
    assert dec_q_heads % dec_kv_heads == 0, \
        f"num_q_heads ({dec_q_heads}) must be divisible by num_kv_heads ({dec_kv_heads})"
    assert q.dtype == q_dec.dtype, "prefill and decode must share one dtype"

    out = q.new_empty(q.shape)
    out_dec = q_dec.new_empty(q_dec.shape)
    f32 = _t.torch.float32
    lse = q.new_empty((total_tokens, num_q_heads), dtype=f32) if return_lse else None
    lse_dec = q.new_empty((num_reqs, dec_q_heads), dtype=f32) if return_lse else None
    cu = _t.as_i32(cu_seqlens, q.device)
    bt = _t.as_i32(block_tables, q.device)
    cl = _t.as_i32(context_lens, q.device)
    L = _t.lib()
    st = _t.stream_of(q)
    max_blocks = bt.shape[1]
    ws_bytes = L.tak_mixed_prefill_decode_workspace_size(num_reqs, dec_q_heads, dec_kv_heads, dec_head_dim,
                                                         block_size, max_blocks)
    ws = _t.workspace(q.device, st, ws_bytes)
    _t.check(L.tak_mixed_prefill_decode(
        _t.ptr(q), _t.strides(q), _t.ptr(k), _t.strides(k), _t.ptr(v), _t.strides(v), _t.ptr(cu), cu.numel() - 1,
        _t.ptr(out), _t.strides(out), _t.ptr(lse), total_tokens, num_q_heads, num_kv_heads, head_dim,
        1.0 / math.sqrt(head_dim), int(bool(causal)),
        _t.ptr(q_dec), _t.strides(q_dec), _t.ptr(k_cache), _t.strides(k_cache), _t.ptr(v_cache),
        _t.strides(v_cache), _t.ptr(bt), _t.strides(bt), _t.ptr(cl), _t.ptr(out_dec), _t.strides(out_dec),
        _t.ptr(lse_dec), num_reqs, dec_q_heads, dec_kv_heads, dec_head_dim, block_size, max_blocks,
        k_cache.shape[0], k_cache.shape[2], 1.0 / math.sqrt(dec_head_dim), _t.dtype_code(q), _t.ptr(ws), ws.numel(),
        st))
    if return_lse:
        return (out, lse), (out_dec, lse_dec)
    return out, out_dec

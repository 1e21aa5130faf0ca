"""Varlen flash prefill (TND layout, MHA / GQA / MQA) on B200.

Drop-in for attention/flash_attention_prefill.py of suluner/triton-ascend-kernels:
same function name, arguments, defaults, return value and assertion behaviour
(FP:108-171), running hand-written sm_100a kernels through libtak_b200.so.
"""

import math

import _tak_b200 as _t


def flash_attention_prefill(q, k, v, cu_seqlens, causal=True, *, return_lse=False):
    """Prefill attention with GQA/MQA/MHA support (TND layout).

    Args:
        q: [total_tokens, num_q_heads, head_dim]
        k: [total_tokens, num_kv_heads, head_dim]
        v: [total_tokens, num_kv_heads, head_dim]
        cu_seqlens: [num_seqs + 1] int32 cumulative sequence lengths
        causal: whether to apply the causal mask
        return_lse: (keyword-only addition) also return lse [total_tokens,
            num_q_heads] float32, the natural log of each row's softmax
            denominator

    Returns ``out`` (same dtype and shape as q), or ``(out, lse)``.
    Tokens outside every sequence of cu_seqlens get zeros.  As in the
    reference kernel (FP:97) the output is acc / (l + 1e-6).
    """
    _t.require_cuda(q, k, v)

    total_tokens, num_q_heads, head_dim = q.shape
    num_kv_heads = k.shape[1]

    assert num_q_heads % num_kv_heads == 0, \
        f"num_q_heads ({num_q_heads}) must be divisible by num_kv_heads ({num_kv_heads})"
    assert k.shape == v.shape, "K and V must have the same shape"
    assert k.shape[0] == total_tokens and k.shape[2] == head_dim, \
        "K/V shape must be [total_tokens, num_kv_heads, head_dim]"

    out = q.new_empty(q.shape)
    lse = q.new_empty((total_tokens, num_q_heads), dtype=_t.torch.float32) if return_lse else None
    scale = 1.0 / math.sqrt(head_dim)
    cu = _t.as_i32(cu_seqlens, q.device)
    num_seqs = cu.numel() - 1

    _t.check(_t.lib().tak_flash_attention_prefill(
        _t.ptr(q), _t.strides(q), _t.ptr(k), _t.strides(k), _t.ptr(v), _t.strides(v), _t.ptr(cu), num_seqs,
        _t.ptr(out), _t.strides(out), _t.ptr(lse), total_tokens, num_q_heads, num_kv_heads, head_dim,
        scale, int(bool(causal)), _t.dtype_code(q), _t.stream_of(q)))
    return (out, lse) if return_lse else out

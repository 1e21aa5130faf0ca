"""ctypes binding of libtak_b200.so (the sm_100a kernels behind include/tak_attention.h).

Shared by the drop-in modules of this folder.  The library is built in-tree by
``triton-ascend-kernels_b200/csrc/build.py``; importing a module works without
it, but the first call raises (there is no CPU fallback).
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "lib", "libtak_b200.so")

_lib = None
_lock = threading.Lock()

_P, _I64, _I32, _F32, _SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_size_t

# argument lists of the extern "C" entry points (include/tak_attention.h)
_SIGS = {
    "tak_version": ([], ctypes.c_char_p),
    "tak_last_error": ([], ctypes.c_char_p),
    "tak_read_device_error": ([_P], _I32),
    "tak_set_kernel_path": ([_I32], _I32),
    "tak_last_kernel": ([], ctypes.c_char_p),
    "tak_flash_attention_prefill": ([_P, _P, _P, _P, _P, _P, _P, _I64, _P, _P, _P, _I64, _I64, _I64, _I64, _F32,
                                     _I32, _I32, _P], _I32),
    "tak_paged_attention_decode_workspace_size": ([_I64, _I64, _I64, _I64, _I64, _I64, _I32], _SZ),
    "tak_paged_attention_decode": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64,
                                    _I64, _I64, _I64, _F32, _I32, _P, _SZ, _I32, _P], _I32),
    "tak_paged_attention_decode_static_scratch": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64,
                                                   _I64, _I64, _I64, _I64, _I64, _F32, _I32, _I32, _P], _I32),
    "tak_sparse_attn_prefill": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64,
                                 _I64, _I64, _F32, _I32, _P], _I32),
    "tak_sparse_attn_prefill_2src": ([_P, _P, _P, _P, _P, _P, _I64, _P, _P, _P, _P, _I64, _P, _P, _P, _P, _P, _P,
                                      _I64, _I64, _I64, _I64, _I64, _I64, _F32, _I32, _P], _I32),
    "tak_sparse_attn_decode": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64,
                                _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _F32, _I32, _P], _I32),
    "tak_build_token_to_seq": ([_P, _I64, _I64, _P, _P], _I32),
    "tak_compress_kv": ([_P, _P, _P, _P, _P, _I64, _P, _P, _I64, _I64, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                         _I64, _I32, _P], _I32),
    "tak_compress_kv_paged": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P, _I64, _I64, _P, _P, _P,
                               _P, _I64, _I64, _I64, _I64, _I64, _I32, _P], _I32),
    "tak_compress_kv_csa_hca": ([_P, _P, _P, _P, _P, _I64, _P, _I64, _I64, _P, _I64, _P, _P, _P, _P, _P, _I64, _P,
                                 _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I32, _P], _I32),
    "tak_build_window_idxs": ([_P, _I64, _I64, _I64, _P, _I64, _P], _I32),
    "tak_build_hca_topk_idxs": ([_P, _P, _I64, _I64, _I64, _I64, _I64, _P, _I64, _P], _I32),
    "tak_build_decode_topk_idxs": ([_P, _P, _I64, _I64, _I64, _I64, _P, _I64, _P], _I32),
    "tak_comp_offsets": ([_P, _I64, _I32, _I64, _I64, _P, _P], _I32),
    "tak_csa_indexer_topk": ([_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                              _P, _I64, _I32, _P, _I64, _I64, _P], _I32),
    "tak_csa_indexer_workspace_size": ([_I64, _I64, _I32], _I64),
}


def lib():
    """Load (once) and return the ctypes handle of libtak_b200.so."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with "
                        "`python triton-ascend-kernels_b200/csrc/build.py` (no CPU fallback exists)")
                h = ctypes.CDLL(LIB_PATH)
                for name, (args, res) in _SIGS.items():
                    fn = getattr(h, name)
                    fn.argtypes = args
                    fn.restype = res
                _lib = h
    return _lib


def check(rc):
    if rc != 0:
        raise RuntimeError(f"tak_b200 error {rc}: {lib().tak_last_error().decode()}")


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def strides(t):
    s = t.stride()
    return (ctypes.c_int64 * len(s))(*s)


_DTYPES = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}


def dtype_code(t):
    if t.dtype not in _DTYPES:
        raise TypeError(f"unsupported dtype {t.dtype}: expected float16, bfloat16 or float32")
    return _DTYPES[t.dtype]


def stream_of(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda(*ts):
    for t in ts:
        if t is not None:
            assert t.is_cuda, "Tensors must be on a CUDA device"


def as_i32(t, device):
    """int32 index tensor on `device` (no copy when it already is one)."""
    if not isinstance(t, torch.Tensor):
        t = torch.tensor(t, dtype=torch.int32)
    return t.to(device=device, dtype=torch.int32)


_ws = {}


def workspace(device, stream_handle, nbytes):
    """Per-(device, stream) scratch buffer, grown on demand.  Its contents do
    not matter between calls: the decode combine only reads split partials
    written earlier in the same call (the zero fill is not relied on)."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), int(stream_handle.value or 0))
    buf = _ws.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _ws[key] = buf
    return buf


def set_kernel_path(path):
    """0 = tensor-core kernels where the shape allows (default), 1 = generic CUDA-core kernels."""
    return lib().tak_set_kernel_path(int(path))


def last_kernel():
    """Name of the main kernel the calling thread's last attention or pooling
    call launched ("" when it launched none), e.g. "prefill_tc" or
    "sparse_generic"."""
    return lib().tak_last_kernel().decode()


def read_device_error(device=None):
    s = torch.cuda.current_stream(device)
    return lib().tak_read_device_error(ctypes.c_void_p(s.cuda_stream))


# ---------------------------------------------------------------------------
# compression helpers shared by csa.py / hca.py
# ---------------------------------------------------------------------------

def comp_offsets_host(lengths, stride):
    """max(1, ceil(L/stride)) slots per non-empty sequence, cumulative (CSA:38-59)."""
    offs = [0]
    for L in lengths:
        offs.append(offs[-1] + (max(1, -(-int(L) // stride)) if L > 0 else 0))
    return offs


def compress_tnd(k, v, cu_seqlens, stride, window, gate=None):
    """Pool K/V rows of TND sequences into compressed slots on the device.

    Needs the sequence lengths on the host to size the output (one
    device->host copy of cu_seqlens, as the reference's .item() loop).
    Returns (compressed_k, compressed_v, comp_offsets[int32, device]).
    """
    require_cuda(k, v)
    dev = k.device
    if isinstance(cu_seqlens, torch.Tensor) and cu_seqlens.is_cuda:
        cu = as_i32(cu_seqlens, dev)
        cu_h = cu.cpu().tolist()          # device -> host copy (sizes the outputs)
    else:                                 # lengths already on the host: no device sync
        cu_h = [int(x) for x in (cu_seqlens.tolist() if isinstance(cu_seqlens, torch.Tensor) else cu_seqlens)]
        cu = torch.tensor(cu_h, dtype=torch.int32).to(dev, non_blocking=True)
    offs = comp_offsets_host([cu_h[i + 1] - cu_h[i] for i in range(len(cu_h) - 1)], stride)
    nc = offs[-1]
    hkv = k.shape[1]
    ck = k.new_empty((nc, hkv, k.shape[2]))
    cv = v.new_empty((nc, hkv, v.shape[2]))
    offs_t = torch.tensor(offs, dtype=torch.int32).to(dev)
    if nc:
        g = None
        if gate is not None:
            g = gate.to(device=dev, dtype=torch.float32)
            assert g.dim() == 1 and g.shape[0] == k.shape[0], "gate must be [total_tokens] logits"
        check(lib().tak_compress_kv(
            ptr(k), strides(k), ptr(v), strides(v), ptr(g), g.stride(0) if g is not None else 0, ptr(cu),
            ptr(offs_t), len(cu_h) - 1, nc, ptr(ck), strides(ck), ptr(cv), strides(cv), hkv, k.shape[2],
            v.shape[2], stride, window, dtype_code(k), stream_of(k)))
    return ck, cv, offs_t


def compress_csa_hca(k, v, cu_seqlens, m, m_prime, gate=None):
    """CSA (window 2m, stride m) and HCA (window = stride = m_prime) pooling of
    the same TND K/V in one pass.  Returns ((csa_k, csa_v, csa_offsets),
    (hca_k, hca_v, hca_offsets)), offsets int32 on the device."""
    require_cuda(k, v)
    dev = k.device
    if isinstance(cu_seqlens, torch.Tensor) and cu_seqlens.is_cuda:
        cu = as_i32(cu_seqlens, dev)
        cu_h = cu.cpu().tolist()          # device -> host copy (sizes the outputs)
    else:
        cu_h = [int(x) for x in (cu_seqlens.tolist() if isinstance(cu_seqlens, torch.Tensor) else cu_seqlens)]
        cu = torch.tensor(cu_h, dtype=torch.int32).to(dev, non_blocking=True)
    lens = [cu_h[i + 1] - cu_h[i] for i in range(len(cu_h) - 1)]
    hkv = k.shape[1]
    res = []
    for stride in (m, m_prime):
        offs = comp_offsets_host(lens, stride)
        nc = offs[-1]
        res.append((k.new_empty((nc, hkv, k.shape[2])), v.new_empty((nc, hkv, v.shape[2])),
                    torch.tensor(offs, dtype=torch.int32).to(dev), nc))
    (ck, cv, co, nc), (hk, hv, ho, nh) = res
    if nc or nh:
        g = None
        if gate is not None:
            g = gate.to(device=dev, dtype=torch.float32)
            assert g.dim() == 1 and g.shape[0] == k.shape[0], "gate must be [total_tokens] logits"
        check(lib().tak_compress_kv_csa_hca(
            ptr(k), strides(k), ptr(v), strides(v), ptr(g), g.stride(0) if g is not None else 0, ptr(cu),
            len(cu_h) - 1, k.shape[0], ptr(co), nc, ptr(ck), strides(ck), ptr(cv), strides(cv), ptr(ho), nh, ptr(hk),
            strides(hk), ptr(hv), strides(hv), hkv, k.shape[2], v.shape[2], m, m_prime, dtype_code(k), stream_of(k)))
    return (ck, cv, co), (hk, hv, ho)


def is_prefix_view(v, k):
    """v is k or k[..., :Dv] (same storage offset and strides): pooling k
    then covers v."""
    return (v.data_ptr() == k.data_ptr() and v.stride() == k.stride() and v.dim() == k.dim()
            and v.shape[:-1] == k.shape[:-1] and v.shape[-1] <= k.shape[-1] and v.dtype == k.dtype)


def comp_offsets_device(lens, stride, capacity=-1, is_cu=False):
    """comp_offsets [n + 1] int32 computed on the device from int32 lengths
    (or cu_seqlens, is_cu=True); no host read.  capacity >= 0 clamps the
    offsets and records device error 3 when the total exceeds it."""
    n = lens.shape[0] - (1 if is_cu else 0)
    offs = torch.empty(n + 1, dtype=torch.int32, device=lens.device)
    check(lib().tak_comp_offsets(ptr(lens), n, 1 if is_cu else 0, stride, capacity, ptr(offs), stream_of(lens)))
    return offs


def max_slots_per_seq(block_tables, block_size, stride):
    """Slots of the longest context a block table can address (a host bound
    from shapes: max(1, ceil(max_blocks * P / stride)))."""
    return max(1, -(-int(block_tables.shape[1]) * int(block_size) // stride))


def compress_paged(k_cache, v_cache, block_tables, context_lens, block_size, stride, window, capacity=None):
    """Pool each sequence's first context_lens[s] rows straight out of a paged
    cache (fuses the reference's page gather, CSA:225-256 / HCA:204-232).
    When v_cache is a prefix view of k_cache (MLA latent caches) K is pooled
    once and compressed_v is the same view of compressed_k.
    capacity=None sizes the outputs exactly (one device->host read of
    context_lens); an int sizes them [capacity, ...] and computes the offsets
    on the device, with no host read (CUDA-graph capturable; a total above
    the capacity records device error 3).
    Returns (compressed_k, compressed_v, comp_offsets[int32, device],
    lengths[host] or None, comp_offsets[host] or None)."""
    dev = k_cache.device
    bt = as_i32(block_tables, dev)
    cl = as_i32(context_lens, dev)
    if capacity is None:
        lens = cl.cpu().tolist()
        offs = comp_offsets_host(lens, stride)
        nc = offs[-1]
        offs_t = torch.tensor(offs, dtype=torch.int32).to(dev)
    else:
        lens = offs = None
        nc = int(capacity)
        offs_t = comp_offsets_device(cl, stride, nc)
    hkv = k_cache.shape[1]
    k_only = is_prefix_view(v_cache, k_cache)
    ck = k_cache.new_empty((nc, hkv, k_cache.shape[3]))
    cv = ck[..., :v_cache.shape[3]] if k_only else v_cache.new_empty((nc, hkv, v_cache.shape[3]))
    if nc:
        vv, cvv = (None, None) if k_only else (v_cache, cv)
        check(lib().tak_compress_kv_paged(
            ptr(k_cache), strides(k_cache), ptr(vv), None if vv is None else strides(vv), None, None, ptr(bt),
            strides(bt), ptr(cl), block_size, bt.shape[1], k_cache.shape[0], ptr(offs_t), cl.shape[0], nc, ptr(ck),
            strides(ck), ptr(cvv),
            None if cvv is None else strides(cvv), hkv, k_cache.shape[3], 0 if k_only else v_cache.shape[3],
            stride, window, dtype_code(k_cache), stream_of(k_cache)))
    return ck, cv, offs_t, lens, offs


def max_comp_per_seq(comp_offsets, bound):
    """Largest per-sequence slot count, from a cheap bound when it is small."""
    if bound <= 12288:
        return bound
    d = comp_offsets[1:] - comp_offsets[:-1]
    return int(d.max().item()) if d.numel() else 0

"""The allocation-free paged decode entry point.

tak_paged_attention_decode_static_scratch serves callers that cannot allocate
device memory (no cudaMalloc allowed or affordable where they run, or device
memory owned by a framework allocator): its split-KV scratch is a fixed array
inside the library.  This file calls it through the C ABI and checks it
against the workspace-taking entry point on the same inputs, twice in a row
(the scratch is shared and keeps the previous call's contents).  Named so
pytest collects it last.
"""

import ctypes

import numpy as np
import pytest
import torch

import _tak_b200 as T
import paged_attention_decode as PD

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL16, TOL_LSE = 2e-2, 1e-3


def _inputs(seed, B=64, H=32, Hkv=8, D=128, P=128, max_ctx=8192):
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(1, max_ctx + 1, (B,), generator=g).to(torch.int32)
    ctx[0], ctx[1] = 1, max_ctx
    maxb = max_ctx // P
    pool = int(((ctx + P - 1) // P).sum()) + 8
    perm = torch.randperm(pool, generator=g).to(torch.int32)
    bt = torch.zeros(B, maxb, dtype=torch.int32)
    i = 0
    for b in range(B):
        n = (int(ctx[b]) + P - 1) // P
        bt[b, :n] = perm[i:i + n]
        i += n
    q = torch.randn(B, H, D, generator=g).to(DEV, torch.bfloat16)
    kc = torch.randn(pool, Hkv, P, D, generator=g).to(DEV, torch.bfloat16)
    vc = torch.randn(pool, Hkv, P, D, generator=g).to(DEV, torch.bfloat16)
    return q, kc, vc, bt.to(DEV), ctx.to(DEV), P


def _static_call(q, kc, vc, bt, cl, P, out, lse, split_pages=0):
    B, H, D = q.shape
    return T.lib().tak_paged_attention_decode_static_scratch(
        T.ptr(q), T.strides(q), T.ptr(kc), T.strides(kc), T.ptr(vc), T.strides(vc), T.ptr(bt), T.strides(bt),
        T.ptr(cl), T.ptr(out), T.strides(out), T.ptr(lse), B, H, kc.shape[1], D, P, bt.shape[1], kc.shape[0],
        kc.shape[2], 1.0 / D ** 0.5, T.dtype_code(q), split_pages, T.stream_of(q))


def test_static_scratch_matches_workspace_entry_point():
    q, kc, vc, bt, cl, P = _inputs(5)
    ref, ref_lse = PD.paged_attention_decode(q, kc, vc, bt, cl, P, P, return_lse=True)
    assert T.lib().tak_paged_attention_decode_workspace_size(64, 32, 8, 128, P, bt.shape[1], 0) > 0  # split path
    for call in range(2):
        out = torch.empty_like(q)
        lse = torch.empty(q.shape[:2], dtype=torch.float32, device=DEV)
        rc = _static_call(q, kc, vc, bt, cl, P, out, lse)
        assert rc == 0, T.lib().tak_last_error().decode()
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs().max().item()
        assert err <= TOL16, f"call {call}: max abs err {err}"
        assert (lse - ref_lse).abs().max().item() <= TOL_LSE
    # a different problem in between: the shared scratch must not leak state
    q2, kc2, vc2, bt2, cl2, P2 = _inputs(6, B=8, H=16, Hkv=2, max_ctx=2048)
    out2 = torch.empty_like(q2)
    lse2 = torch.empty(q2.shape[:2], dtype=torch.float32, device=DEV)
    assert _static_call(q2, kc2, vc2, bt2, cl2, P2, out2, lse2) == 0
    ref2, ref_lse2 = PD.paged_attention_decode(q2, kc2, vc2, bt2, cl2, P2, P2, return_lse=True)
    assert (out2.float() - ref2.float()).abs().max().item() <= TOL16
    assert (lse2 - ref_lse2).abs().max().item() <= TOL_LSE
    assert T.read_device_error() == 0


def test_static_scratch_rejects_oversized_problem():
    """4096 sequences with 64-page block tables and one page per split would
    need ~4.4 GB of partials: rejected on the host before any launch.  The
    tensors really have those shapes (every context is 1 row of page 0), so
    even a wrong acceptance could not read or write out of bounds."""
    B, H, Hkv, D, P, maxb = 4096, 32, 8, 128, 128, 64
    q = torch.zeros(B, H, D, dtype=torch.bfloat16, device=DEV)
    kc = torch.zeros(1, Hkv, P, D, dtype=torch.bfloat16, device=DEV)
    bt = torch.zeros(B, maxb, dtype=torch.int32, device=DEV)
    cl = torch.ones(B, dtype=torch.int32, device=DEV)
    out = torch.empty_like(q)
    lse = torch.empty(B, H, dtype=torch.float32, device=DEV)
    rc = _static_call(q, kc, kc, bt, cl, P, out, lse, split_pages=1)
    assert rc == 2
    msg = T.lib().tak_last_error().decode()
    assert "static scratch" in msg and "33554432" in msg


def test_static_scratch_larger_split_pages_fits():
    """The remedy the rejection names: 256 requests with 64-page tables need
    272 MB of partials at one page per split (rejected) but 17 MB at 16 pages
    per split (4 splits), which runs and matches the workspace entry point."""
    q, kc, vc, bt, cl, P = _inputs(7, B=256, H=32, Hkv=8, P=16, max_ctx=1024)
    out = torch.empty_like(q)
    lse = torch.empty(q.shape[:2], dtype=torch.float32, device=DEV)
    assert _static_call(q, kc, vc, bt, cl, P, out, lse, split_pages=1) == 2
    need = T.lib().tak_paged_attention_decode_workspace_size(256, 32, 8, 128, P, bt.shape[1], 16)
    assert 0 < need <= 32 << 20
    assert _static_call(q, kc, vc, bt, cl, P, out, lse, split_pages=16) == 0, T.lib().tak_last_error().decode()
    ref, ref_lse = PD.paged_attention_decode(q, kc, vc, bt, cl, P, P, return_lse=True, split_pages=16)
    torch.cuda.synchronize()
    assert (out.float() - ref.float()).abs().max().item() <= TOL16
    assert (lse - ref_lse).abs().max().item() <= TOL_LSE
    assert T.read_device_error() == 0

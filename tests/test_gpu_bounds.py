"""Caller indices that point outside the tensors they index never reach memory.

The reference's kernels read block-table entries and cache pages unchecked
(attention/sparse_attn_fwd.py:151-171, attention/paged_attention_decode.py:49-58)
and its paged gather raises past a block-table row (attention/csa.py:229-245).
The B200 entry points bound every such index against the sizes they are given:

* sparse decode masks a window slot whose position lies past its block-table
  row (>= table width x page size) or whose page id lies outside [0, num_blocks);
* paged decode reads a page id outside [0, num_blocks) as zero keys and values
  (its TMA path zero-fills such pages; the CUDA-core path does the same);
* paged pooling reads a context row past the block-table row, or on such a page,
  as a zero row with gate logit 0.

No out-of-range access can happen even if a bound were missing: each block
table is a narrow column view of a wider table whose hidden columns hold valid
page ids, and each cache is a view over a larger allocation, so that page ids
just outside [0, num_blocks) still name real pages of memory.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu

import _tak_b200 as T  # noqa: E402
import paged_attention_decode as PD  # noqa: E402
import sparse_attn_fwd as SA  # noqa: E402

DEV = "cuda"
TOL16, TOL_LSE, TOL32 = 2e-2, 1e-3, 1e-4
LO = 8  # hidden pages on each side of every cache view


def npy(t):
    return t.detach().float().cpu().numpy()


def close(out, ref, tol):
    err = np.abs(npy(out).astype(np.float64) - ref).max() if out.numel() else 0.0
    assert err <= tol, f"max abs err {err:.3e} > {tol:.1e}"


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert T.read_device_error() == 0, "a kernel reported a timed-out wait"


@pytest.fixture(params=[0, 1], ids=["auto", "generic"])
def kernel_path(request):
    old = T.set_kernel_path(request.param)
    yield request.param
    T.set_kernel_path(old)


def _cache_view(n_view, hkv, P, D, dtype, g):
    """(full, view): view = full[LO:LO + n_view], so page ids -LO..-1 and
    n_view..n_view + LO - 1 of the view are real memory of `full`."""
    full = torch.randn(n_view + 2 * LO, hkv, P, D, generator=g).to(DEV, dtype)
    return full, full[LO:LO + n_view]


def _tables(ctx, P, width, n_view, g, wide=8):
    """A [B, wide] table of distinct valid page ids and its [:, :width] view."""
    B = len(ctx)
    perm = torch.randperm(n_view, generator=g)[:B * wide].view(B, wide).to(torch.int32)
    wide_t = perm.to(DEV)
    return wide_t, wide_t[:, :width]


def _page_ok(bt_h, s, pos, P, width, n_view):
    pg = pos // P
    return pg < width and 0 <= int(bt_h[s, pg]) < n_view


@pytest.mark.parametrize("shape", ["gqa128", "latent576"])
def test_sparse_decode_masks_slots_outside_table_and_cache(shape, kernel_path):
    g = torch.Generator().manual_seed(201)
    P, width, n_view, n_win = 64, 4, 64, 128
    ctx = [300, 200, 130, 64, 0, 5]
    B = len(ctx)
    if shape == "gqa128":
        H, Hkv, D, Dv = 16, 4, 128, 128
        kfull, kc = _cache_view(n_view, Hkv, P, D, torch.bfloat16, g)
        vfull, vc = _cache_view(n_view, Hkv, P, Dv, torch.bfloat16, g)
        ck = torch.randn(90, Hkv, D, generator=g).to(DEV, torch.bfloat16)
        cv = torch.randn(90, Hkv, Dv, generator=g).to(DEV, torch.bfloat16)
    else:
        H, Hkv, D, Dv = 64, 1, 576, 512
        kfull, kc = _cache_view(n_view, Hkv, P, D, torch.bfloat16, g)
        vc = kc[..., :Dv]
        ck = torch.randn(90, Hkv, D, generator=g).to(DEV, torch.bfloat16)
        cv = ck[..., :Dv]
    wide, bt = _tables(ctx, P, width, n_view, g)
    wide[1, 2] = n_view + 1      # a real page, but past num_blocks
    wide[2, 1] = -2              # a real page, but negative
    wide[3, 0] = n_view          # the first page past num_blocks
    q = torch.randn(B, H, D, generator=g).to(DEV, torch.bfloat16)
    n_comp = 40
    idx = torch.full((B, n_win + n_comp), -1, dtype=torch.int32)
    for b, c in enumerate(ctx):
        idx[b, :n_win] = torch.arange(c - n_win, c, dtype=torch.int32)
        rows = torch.randperm(90, generator=g)[:(b * 11) % n_comp].sort().values.to(torch.int32)
        idx[b, n_win:n_win + rows.numel()] = c + rows
    sink = torch.randn(H, generator=g).to(DEV)
    cl = torch.tensor(ctx, dtype=torch.int32, device=DEV)
    out, lse = SA.sparse_attn_decode(q, kc, vc, ck, cv, bt, idx.to(DEV), cl, n_win, P, sink, return_lse=True)
    if kernel_path == 0:
        assert T.last_kernel() == "sparse_tc"
    # the oracle with every window slot past the table or on a bad page dropped
    bt_h = bt.cpu()
    ref_idx = idx.clone()
    n_masked = 0
    for b, c in enumerate(ctx):
        for w in range(n_win):
            pos = int(idx[b, w])
            if 0 <= pos < c and not _page_ok(bt_h, b, pos, P, width, n_view):
                ref_idx[b, w] = -1
                n_masked += 1
    assert n_masked > 0
    bt_ref = torch.where((bt_h >= 0) & (bt_h < n_view), bt_h, torch.zeros_like(bt_h))  # never read at masked slots
    ref, ref_lse = O.sparse_decode(npy(q), npy(kc), npy(vc), npy(ck), npy(cv), bt_ref, ref_idx, cl.cpu(), n_win, P,
                                   sink.cpu())
    close(out, ref, TOL16)
    fin = np.isfinite(ref_lse)
    assert (np.isfinite(lse.cpu().numpy()) == fin).all()
    assert np.abs(lse.cpu().numpy()[fin] - ref_lse[fin]).max() <= TOL_LSE


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_paged_decode_reads_bad_pages_as_zero_rows(dtype, kernel_path):
    """Both decode paths agree: a block-table entry outside [0, num_blocks) is
    never read and its rows count as zero keys and values."""
    g = torch.Generator().manual_seed(202)
    P, width, n_view = 64, 8, 64
    ctx = [300, 64, 129, 1, 500, 0]
    B, H, Hkv, D = len(ctx), 32, 8, 128
    _, kc = _cache_view(n_view, Hkv, P, D, dtype, g)
    _, vc = _cache_view(n_view, Hkv, P, D, dtype, g)
    wide, bt = _tables(ctx, P, width, n_view, g, wide=10)
    wide[0, 1] = n_view + 2
    wide[2, 0] = -1
    wide[4, 3] = n_view
    q = torch.randn(B, H, D, generator=g).to(DEV, dtype)
    cl = torch.tensor(ctx, dtype=torch.int32, device=DEV)
    out, lse = PD.paged_attention_decode(q, kc, vc, bt, cl, P, 16, return_lse=True)
    if kernel_path == 0 and dtype == torch.bfloat16:
        assert T.last_kernel() == "paged_decode_tc"
    elif kernel_path == 1:
        assert T.last_kernel() == "paged_decode_generic"
    # oracle: one extra all-zero page at index n_view stands in for every bad entry
    kz = np.concatenate([npy(kc), np.zeros((1, Hkv, P, D), np.float32)], 0)
    vz = np.concatenate([npy(vc), np.zeros((1, Hkv, P, D), np.float32)], 0)
    bt_h = bt.cpu()
    bt_ref = torch.where((bt_h >= 0) & (bt_h < n_view), bt_h, torch.full_like(bt_h, n_view))
    ref, ref_lse = O.paged_decode(npy(q), kz, vz, bt_ref, cl.cpu(), P)
    close(out, ref, TOL32 if dtype == torch.float32 else TOL16)
    fin = np.isfinite(ref_lse)
    assert np.abs(lse.cpu().numpy()[fin] - ref_lse[fin]).max() <= TOL_LSE


def _compress_paged(kc, vc, gate, bt, cl, P, offs, nc, stride, window):
    ck = kc.new_empty((nc, kc.shape[1], kc.shape[3]))
    cv = vc.new_empty((nc, vc.shape[1], vc.shape[3]))
    gs = (ctypes.c_int64 * 2)(*gate.stride()) if gate is not None else None
    T.check(T.lib().tak_compress_kv_paged(
        T.ptr(kc), T.strides(kc), T.ptr(vc), T.strides(vc), T.ptr(gate), gs, T.ptr(bt), T.strides(bt), T.ptr(cl), P,
        bt.shape[1], kc.shape[0], T.ptr(offs), cl.shape[0], nc, T.ptr(ck), T.strides(ck), T.ptr(cv), T.strides(cv),
        kc.shape[1], kc.shape[3], vc.shape[3], stride, window, T.dtype_code(kc), T.stream_of(kc)))
    return ck, cv


@pytest.mark.parametrize("case", ["bulk_pages_csa", "bulk_pages_hca", "bulk_rows_csa", "gated_csa",
                                  "gated_hca", "fp32_csa"])
def test_compress_paged_rows_outside_table_and_cache_pool_as_zeros(case):
    g = torch.Generator().manual_seed(203)
    P, width, n_view, hkv, D = 64, 4, 64, 2, 128
    ctx = [300, 200, 130, 64, 17, 0]
    B = len(ctx)
    dtype = torch.float32 if case.startswith("fp32") else torch.bfloat16
    stride, window = (128, 128) if case.endswith("hca") else (4, 8)
    if case.startswith("bulk_rows"):
        # rows not contiguous within a page: one copy per row instead of per page piece
        _, kbig = _cache_view(n_view, hkv, P, 2 * D, dtype, g)
        _, vbig = _cache_view(n_view, hkv, P, 2 * D, dtype, g)
        kc, vc = kbig[..., :D], vbig[..., D:]
    else:
        _, kc = _cache_view(n_view, hkv, P, D, dtype, g)
        _, vc = _cache_view(n_view, hkv, P, D, dtype, g)
    gate = None
    if case.startswith("gated"):
        gfull = torch.randn(n_view + 2 * LO, P, generator=g).to(DEV)
        gate = gfull[LO:LO + n_view]
    wide, bt = _tables(ctx, P, width, n_view, g)
    wide[1, 2] = n_view + 1
    wide[2, 0] = -3
    wide[3, 0] = n_view
    cl = torch.tensor(ctx, dtype=torch.int32, device=DEV)
    offs_h = T.comp_offsets_host(ctx, stride)
    offs = torch.tensor(offs_h, dtype=torch.int32, device=DEV)
    ck, cv = _compress_paged(kc, vc, gate, bt, cl, P, offs, offs_h[-1], stride, window)
    expect = {"bulk": "compress_bulk", "gated": "compress_stream" if stride == 4 else "compress_split",
              "fp32": "compress_rows"}[case.split("_")[0]]
    assert T.last_kernel() == expect
    # the oracle on TND rows where every row past the table or on a bad page is zero (gate logit 0)
    bt_h, kn, vn = bt.cpu(), npy(kc), npy(vc)
    gn = None if gate is None else gate.cpu().numpy()
    rows_k, rows_v, rows_g, cu = [], [], [], [0]
    for s, c in enumerate(ctx):
        for r in range(c):
            ok = _page_ok(bt_h, s, r, P, width, n_view)
            pg = int(bt_h[s, r // P]) if ok else 0
            rows_k.append(kn[pg, :, r % P] if ok else np.zeros((hkv, D), np.float32))
            rows_v.append(vn[pg, :, r % P] if ok else np.zeros((hkv, D), np.float32))
            rows_g.append(gn[pg, r % P] if (ok and gn is not None) else 0.0)
        cu.append(cu[-1] + c)
    kt, vt = np.stack(rows_k), np.stack(rows_v)
    rk, rv, roffs = O.compress_kv(kt, vt, cu, stride, window, None if gate is None else np.array(rows_g))
    np.testing.assert_array_equal(np.asarray(offs_h), roffs)
    tol = TOL32 if dtype == torch.float32 else 1e-2
    close(ck, rk, tol)
    close(cv, rv, tol)

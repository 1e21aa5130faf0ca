"""Inputs of the reference's own test runners, rebuilt on the CPU.

Each function replays one ``run_*test`` of suluner/triton-ascend-kernels'
``attention/*.py`` -- same seed, same order of ``torch.randn`` /
``torch.randperm`` calls, fp16 -- but on the CPU generator instead of
``npu:0``.  The SHA-256 of every tensor is stored in
``reference_golden_inputs.json`` so that a change of torch's CPU generator is
caught instead of silently producing other inputs.
"""

from __future__ import annotations

import math

import torch

F16 = torch.float16

# FP:235-286
FP_LENS = [128, 35, 256]
FP_CU = [0, 128, 163, 419]
FP_HEADS = [(8, 8), (8, 4), (8, 2), (8, 1)]
FP_SEED = 123
FP_D = 128

# PD:208-266
PD_CTX = [12, 35, 22, 54]
PD_BLOCK = 16
PD_MAXB = 4
PD_HEADS = [(16, 16), (16, 8), (16, 4), (16, 2)]
PD_SEED = 42

# SA:504-675, CSA:470-594, HCA:416-538 share the head sweep
SA_HEADS = [(4, 2), (2, 4), (1, 8)]
SA_CU = [0, 64, 192, 288]
SA_NWIN_P, SA_NCOMP = 32, 8
SA_CTX = [32, 48, 16, 56]
SA_BLOCK = 16
SA_MAXB = 8
SA_NWIN_D = 16

CSA_M, CSA_NWIN_P, CSA_NWIN_D, CSA_TOPK = 4, 16, 8, 4
HCA_M, HCA_NWIN = 128, 16
HCA_CU = [0, 256, 768, 1152]
HCA_CTX = [256, 512, 128, 384]
HCA_MAXB = 48

D = 128


def _cu(cu):
    return torch.tensor(cu, dtype=torch.int32)


def _block_tables(ctx, maxb, block):
    n = len(ctx)
    allb = torch.randperm(n * maxb, dtype=torch.int32)
    bt = torch.zeros(n, maxb, dtype=torch.int32)
    i = 0
    for s in range(n):
        for j in range(math.ceil(ctx[s] / block)):
            bt[s, j] = allb[i]
            i += 1
    return bt


def fp_inputs(hq, hkv):
    torch.manual_seed(FP_SEED)
    T = FP_CU[-1]
    q = torch.randn(T, hq, FP_D, dtype=F16)
    k = torch.randn(T, hkv, FP_D, dtype=F16)
    v = torch.randn(T, hkv, FP_D, dtype=F16)
    return {"q": q, "k": k, "v": v, "cu_seqlens": _cu(FP_CU)}


def pd_inputs(hq, hkv):
    torch.manual_seed(PD_SEED)
    n = len(PD_CTX)
    q = torch.randn(n, hq, D, dtype=F16)
    cl = torch.tensor(PD_CTX, dtype=torch.int32)
    bt = _block_tables(PD_CTX, PD_MAXB, PD_BLOCK)
    nb = n * PD_MAXB
    kc = torch.randn(nb, hkv, PD_BLOCK, D, dtype=F16)
    vc = torch.randn(nb, hkv, PD_BLOCK, D, dtype=F16)
    return {"q": q, "k_cache": kc, "v_cache": vc, "block_tables": bt, "context_lens": cl}


def _window_idxs(cu, n_win):
    T = cu[-1]
    out = torch.full((T, n_win), -1, dtype=torch.int32)
    for s in range(len(cu) - 1):
        for p in range(cu[s + 1] - cu[s]):
            for wi in range(n_win):
                src = p - n_win + 1 + wi
                if 0 <= src <= p:
                    out[cu[s] + p, wi] = cu[s] + src
    return out


def _sinks(hq, base):
    """The runners draw the sink vector inside the sink loop: no draw for
    sink=False, one torch.randn(H) fp32 draw for sink=True (SA:562-564)."""
    yield False, dict(base)
    d = dict(base)
    d["attn_sink"] = torch.randn(hq, dtype=torch.float32)
    yield True, d


def sa_prefill_inputs(hkv, grp):
    hq = hkv * grp
    torch.manual_seed(42)
    T, S = SA_CU[-1], len(SA_CU) - 1
    q = torch.randn(T, hq, D, dtype=F16)
    k = torch.randn(T + S * SA_NCOMP, hkv, D, dtype=F16)
    v = torch.randn(T + S * SA_NCOMP, hkv, D, dtype=F16)
    win = _window_idxs(SA_CU, SA_NWIN_P)
    comp = torch.full((T, SA_NCOMP), -1, dtype=torch.int32)
    for s in range(S):
        for p in range(SA_CU[s + 1] - SA_CU[s]):
            for ci in range(SA_NCOMP):
                comp[SA_CU[s] + p, ci] = T + s * SA_NCOMP + ci
    base = {"q": q, "k": k, "v": v, "topk_idxs": torch.cat([win, comp], 1), "cu_seqlens": _cu(SA_CU)}
    yield from _sinks(hq, base)


def sa_decode_inputs(hkv, grp):
    hq = hkv * grp
    torch.manual_seed(123)
    n = len(SA_CTX)
    q = torch.randn(n, hq, D, dtype=F16)
    cl = torch.tensor(SA_CTX, dtype=torch.int32)
    bt = _block_tables(SA_CTX, SA_MAXB, SA_BLOCK)
    nb = n * SA_MAXB
    kc = torch.randn(nb, hkv, SA_BLOCK, D, dtype=F16)
    vc = torch.randn(nb, hkv, SA_BLOCK, D, dtype=F16)
    ck = torch.randn(n * SA_NCOMP, hkv, D, dtype=F16)
    cv = torch.randn(n * SA_NCOMP, hkv, D, dtype=F16)
    idx = torch.full((n, SA_NWIN_D + SA_NCOMP), -1, dtype=torch.int32)
    for s in range(n):
        ctx = SA_CTX[s]
        for wi in range(SA_NWIN_D):
            if ctx - SA_NWIN_D + wi >= 0:
                idx[s, wi] = ctx - SA_NWIN_D + wi
        for ci in range(SA_NCOMP):
            idx[s, SA_NWIN_D + ci] = ctx + s * SA_NCOMP + ci
    base = {"q": q, "k_cache": kc, "v_cache": vc, "compressed_k": ck, "compressed_v": cv,
            "block_tables": bt, "topk_idxs": idx, "context_lens": cl}
    yield from _sinks(hq, base)


def _qkv_prefill(hkv, grp, cu, seed):
    hq = hkv * grp
    torch.manual_seed(seed)
    T = cu[-1]
    q = torch.randn(T, hq, D, dtype=F16)
    k = torch.randn(T, hkv, D, dtype=F16)
    v = torch.randn(T, hkv, D, dtype=F16)
    return hq, {"q": q, "k": k, "v": v, "cu_seqlens": _cu(cu)}


def csa_prefill_inputs(hkv, grp):
    hq, base = _qkv_prefill(hkv, grp, SA_CU, 42)
    yield from _sinks(hq, base)


def hca_prefill_inputs(hkv, grp):
    hq, base = _qkv_prefill(hkv, grp, HCA_CU, 42)
    yield from _sinks(hq, base)


def _paged_decode(hkv, grp, ctx, maxb, seed):
    hq = hkv * grp
    torch.manual_seed(seed)
    n = len(ctx)
    q = torch.randn(n, hq, D, dtype=F16)
    cl = torch.tensor(ctx, dtype=torch.int32)
    bt = _block_tables(ctx, maxb, SA_BLOCK)
    nb = n * maxb
    kc = torch.randn(nb, hkv, SA_BLOCK, D, dtype=F16)
    vc = torch.randn(nb, hkv, SA_BLOCK, D, dtype=F16)
    return hq, {"q": q, "k_cache": kc, "v_cache": vc, "block_tables": bt, "context_lens": cl}


def csa_decode_inputs(hkv, grp):
    hq, base = _paged_decode(hkv, grp, SA_CTX, SA_MAXB, 123)
    yield from _sinks(hq, base)


def hca_decode_inputs(hkv, grp):
    hq, base = _paged_decode(hkv, grp, HCA_CTX, HCA_MAXB, 123)
    yield from _sinks(hq, base)


def case_inputs(case):
    """Rebuild the inputs of a golden case by its name."""
    kind, heads = case.split("_")[0], case.split("_")[1:]
    hq, hkv = int(heads[0][1:]), int(heads[1])
    if kind == "fp":
        return fp_inputs(hq, hkv)
    if kind == "pd":
        return pd_inputs(hq, hkv)
    sink_on = heads[2] == "s1"
    gen = {"sap": sa_prefill_inputs, "sad": sa_decode_inputs, "csap": csa_prefill_inputs,
           "csad": csa_decode_inputs, "hcap": hca_prefill_inputs, "hcad": hca_decode_inputs}[kind]
    for on, inp in gen(hkv, hq // hkv):
        if on == sink_on:
            return inp
    raise KeyError(case)

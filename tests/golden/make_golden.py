"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run where a checkout of the reference is available, passing its attention/
folder (the script only reads it):

    python tests/golden/make_golden.py <reference checkout>/attention

For each test runner of the reference (``run_*test`` in attention/*.py) this
script rebuilds that runner's inputs on the CPU -- same seed, same sequence of
``torch.randn`` / ``torch.randperm`` calls, fp16 -- calls the reference's own
``torch_*_reference`` functions and index builders, and stores:

  * in ``reference_golden_inputs.json``: the sha256 of every input tensor (tests
    regenerate the inputs with ``golden_inputs.py`` and check the hash);
  * ``<case>/out`` (+ ``rows``) the reference output, fp16; for large outputs
                           only the token rows listed in ``rows`` are kept;
  * index tensors (top-k rows, compression offsets) in full, and the compressed
    K/V of the CSA/HCA runners;
  * in ``reference_edges.npz``: the index builders and mean compressors on edge
    lengths and strides (``main_edges``), inputs included.

The reference's Triton kernels need an Ascend NPU and are not run; the torch
reference functions are what the reference's tests compare them against.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import golden_inputs as gi  # noqa: E402

MAX_ROWS = 24


def sha(t):
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def subset_rows(n_rows, cu):
    if n_rows <= MAX_ROWS:
        return np.arange(n_rows, dtype=np.int32)
    step = -(-n_rows // (MAX_ROWS - 2 * (len(cu) - 1)))
    rows = set(range(0, n_rows, step))
    for i in range(len(cu) - 1):
        if cu[i + 1] > cu[i]:
            rows.add(int(cu[i]))
            rows.add(int(cu[i + 1]) - 1)
    return np.asarray(sorted(rows), np.int32)


def main(ref_dir):
    sys.path.insert(0, ref_dir)
    import flash_attention_prefill as FP
    import paged_attention_decode as PD
    import sparse_attn_fwd as SA
    import csa as CSA
    import hca as HCA

    store, meta = {}, {}

    def put(name, arr):
        store[name] = arr

    def put_inputs(case, tensors):
        meta[case] = {k: sha(v) for k, v in tensors.items() if isinstance(v, torch.Tensor)}

    def put_out(case, out, cu=None):
        o = out.to(torch.float16).numpy()
        rows = subset_rows(o.shape[0], cu if cu is not None else [0, o.shape[0]])
        put(f"{case}/rows", rows)
        put(f"{case}/out", o[rows])

    # FP:235-286
    for hq, hkv in gi.FP_HEADS:
        for causal in (True, False):
            case = f"fp_h{hq}_{hkv}_c{int(causal)}"
            inp = gi.fp_inputs(hq, hkv)
            put_inputs(case, inp)
            out = FP.torch_prefill_tnd_reference(inp["q"], inp["k"], inp["v"], inp["cu_seqlens"], causal=causal)
            put_out(case, out, gi.FP_CU)

    # PD:208-266
    for hq, hkv in gi.PD_HEADS:
        case = f"pd_h{hq}_{hkv}"
        inp = gi.pd_inputs(hq, hkv)
        put_inputs(case, inp)
        out = PD.torch_paged_attention_reference(inp["q"], inp["k_cache"], inp["v_cache"], inp["block_tables"],
                                                 inp["context_lens"], gi.PD_BLOCK)
        put_out(case, out)

    # SA:504-581
    for hkv, grp in gi.SA_HEADS:
        for sink_on, inp in gi.sa_prefill_inputs(hkv, grp):
            case = f"sap_h{hkv * grp}_{hkv}_s{int(sink_on)}"
            put_inputs(case, inp)
            out = SA.torch_sparse_prefill_reference(inp["q"], inp["k"], inp["v"], inp["topk_idxs"],
                                                    inp["cu_seqlens"], attn_sink=inp.get("attn_sink"))
            put_out(case, out, gi.SA_CU)

    # SA:588-675
    for hkv, grp in gi.SA_HEADS:
        for sink_on, inp in gi.sa_decode_inputs(hkv, grp):
            case = f"sad_h{hkv * grp}_{hkv}_s{int(sink_on)}"
            put_inputs(case, inp)
            out = SA.torch_sparse_decode_reference(inp["q"], inp["k_cache"], inp["v_cache"], inp["compressed_k"],
                                                   inp["compressed_v"], inp["block_tables"], inp["topk_idxs"],
                                                   inp["context_lens"], block_size=gi.SA_BLOCK,
                                                   attn_sink=inp.get("attn_sink"))
            put_out(case, out)

    # CSA:470-525
    for hkv, grp in gi.SA_HEADS:
        for sink_on, inp in gi.csa_prefill_inputs(hkv, grp):
            case = f"csap_h{hkv * grp}_{hkv}_s{int(sink_on)}"
            put_inputs(case, inp)
            q, k, v, cu = inp["q"], inp["k"], inp["v"], inp["cu_seqlens"]
            ck, cv, offs = CSA.compress_kv_overlap(k, v, cu, gi.CSA_M)
            idx = CSA.build_csa_topk_idxs(q, ck, cu, offs, gi.CSA_NWIN_P, gi.CSA_TOPK, gi.CSA_M)
            out = CSA.torch_csa_prefill_reference(q, k, v, cu, gi.CSA_NWIN_P, gi.CSA_TOPK, gi.CSA_M,
                                                  attn_sink=inp.get("attn_sink"))
            put(f"{case}/ck", ck.numpy())
            put(f"{case}/cv", cv.numpy())
            put(f"{case}/comp_offsets", offs.numpy())
            put(f"{case}/topk_idxs", idx.numpy())
            put_out(case, out, gi.SA_CU)

    # CSA:528-594
    for hkv, grp in gi.SA_HEADS:
        for sink_on, inp in gi.csa_decode_inputs(hkv, grp):
            case = f"csad_h{hkv * grp}_{hkv}_s{int(sink_on)}"
            put_inputs(case, inp)
            out = CSA.torch_csa_decode_reference(inp["q"], inp["k_cache"], inp["v_cache"], inp["block_tables"],
                                                 inp["context_lens"], gi.CSA_NWIN_D, gi.CSA_TOPK, gi.CSA_M,
                                                 block_size=gi.SA_BLOCK, attn_sink=inp.get("attn_sink"))
            put_out(case, out)

    # HCA:416-470
    for hkv, grp in gi.SA_HEADS:
        for sink_on, inp in gi.hca_prefill_inputs(hkv, grp):
            case = f"hcap_h{hkv * grp}_{hkv}_s{int(sink_on)}"
            put_inputs(case, inp)
            q, k, v, cu = inp["q"], inp["k"], inp["v"], inp["cu_seqlens"]
            ck, cv, offs = HCA.compress_kv_simple(k, v, cu, gi.HCA_M)
            idx = HCA.build_hca_topk_idxs(cu, offs, q.shape[0], gi.HCA_NWIN, gi.HCA_M)
            out = HCA.torch_hca_prefill_reference(q, k, v, cu, gi.HCA_NWIN, gi.HCA_M, attn_sink=inp.get("attn_sink"))
            put(f"{case}/ck", ck.numpy())
            put(f"{case}/cv", cv.numpy())
            put(f"{case}/comp_offsets", offs.numpy())
            put(f"{case}/topk_idxs", idx.numpy())
            put_out(case, out, gi.HCA_CU)

    # HCA:473-538
    for hkv, grp in gi.SA_HEADS:
        for sink_on, inp in gi.hca_decode_inputs(hkv, grp):
            case = f"hcad_h{hkv * grp}_{hkv}_s{int(sink_on)}"
            put_inputs(case, inp)
            out = HCA.torch_hca_decode_reference(inp["q"], inp["k_cache"], inp["v_cache"], inp["block_tables"],
                                                 inp["context_lens"], gi.HCA_NWIN, gi.HCA_M,
                                                 block_size=gi.SA_BLOCK, attn_sink=inp.get("attn_sink"))
            put_out(case, out)

    np.savez_compressed(os.path.join(HERE, "reference_golden.npz"), **store)
    with open(os.path.join(HERE, "reference_golden_inputs.json"), "w") as f:
        json.dump({"torch": torch.__version__, "sha256": meta}, f, indent=1, sort_keys=True)
    print(f"wrote {len(store)} arrays for {len(meta)} cases")


# Edge configurations of the integer index builders and the mean compressors:
# lengths 0 / 1 / just below, at and above a stride or window, strides 1 to 128,
# windows longer than every sequence, top_k above the slot count.
EDGE_LENS = [1, 2, 0, 3, 4, 5, 7, 8, 9, 127, 128, 129, 300]
EDGE_CSA_M = (1, 3, 4)
EDGE_HCA_M = (1, 5, 16, 128)
EDGE_NWIN = (1, 4, 130)
EDGE_CSA_IDX = ((4, 4, 6), (4, 1, 64), (3, 130, 16))     # (m, n_win, top_k)


def main_edges(ref_dir):
    """reference_edges.npz: inputs (fp16, seed 1) and the reference's own
    compress_kv_overlap / compress_kv_simple / build_hca_topk_idxs /
    build_csa_topk_idxs results on EDGE_LENS."""
    sys.path.insert(0, ref_dir)
    import csa as CSA
    import hca as HCA

    g = torch.Generator().manual_seed(1)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(EDGE_LENS)]), dtype=torch.int32)
    T = int(cu[-1])
    k = torch.randn(T, 1, 8, generator=g).half()
    v = torch.randn(T, 1, 8, generator=g).half()
    q = torch.randn(T, 2, 8, generator=g).half()
    store = {"cu_seqlens": cu.numpy(), "k": k.numpy(), "v": v.numpy(), "q": q.numpy()}
    for m in EDGE_CSA_M:
        ck, cv, offs = CSA.compress_kv_overlap(k, v, cu, m)
        store[f"csa_m{m}/ck"], store[f"csa_m{m}/cv"], store[f"csa_m{m}/comp_offsets"] = \
            ck.numpy(), cv.numpy(), offs.numpy()
    for mp in EDGE_HCA_M:
        ck, cv, offs = HCA.compress_kv_simple(k, v, cu, mp)
        store[f"hca_m{mp}/ck"], store[f"hca_m{mp}/cv"], store[f"hca_m{mp}/comp_offsets"] = \
            ck.numpy(), cv.numpy(), offs.numpy()
        if mp > 1:
            for nw in EDGE_NWIN:
                store[f"hca_m{mp}/topk_idxs_w{nw}"] = HCA.build_hca_topk_idxs(cu, offs, T, nw, mp).numpy()
    for m, nw, tk in EDGE_CSA_IDX:
        ck, _, offs = CSA.compress_kv_overlap(k, v, cu, m)
        store[f"csa_idx_m{m}_w{nw}_k{tk}"] = CSA.build_csa_topk_idxs(q, ck, cu, offs, nw, tk, m).numpy()
    _attention_edges(store, g)
    np.savez_compressed(os.path.join(HERE, "reference_edges.npz"), **store)
    print(f"wrote {len(store)} edge arrays")


def _attention_edges(store, g):
    """The reference's torch attention functions on edge lengths: sequences of
    0, 1, 2 and 63-65 / 129 tokens (prefill, causal and not); contexts of 1,
    P - 1, P, P + 1 and whole tables (paged decode, P = 16); -1 padding, an
    all -1 row, with and without sinks (sparse prefill); contexts below the
    window and compressed rows (sparse decode).  fp16, GQA 4 / 2 or MQA."""
    import flash_attention_prefill as FP
    import paged_attention_decode as PD
    import sparse_attn_fwd as SA

    lens = [1, 2, 0, 63, 64, 65, 129]
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)
    T = int(cu[-1])
    q, k, v = (torch.randn(T, h, 16, generator=g).half() for h in (4, 2, 2))
    store.update({"fp/cu_seqlens": cu.numpy(), "fp/q": q.numpy(), "fp/k": k.numpy(), "fp/v": v.numpy()})
    for causal in (True, False):
        store[f"fp/out_c{int(causal)}"] = FP.torch_prefill_tnd_reference(q, k, v, cu, causal=causal).numpy()

    P = 16
    ctx = torch.tensor([1, 15, 16, 17, 48, 96], dtype=torch.int32)
    kc, vc = (torch.randn(40, 2, P, 16, generator=g).half() for _ in range(2))
    bt = torch.randperm(40, generator=g)[:36].view(6, 6).to(torch.int32)
    qd = torch.randn(6, 4, 16, generator=g).half()
    store.update({"pd/q": qd.numpy(), "pd/k_cache": kc.numpy(), "pd/v_cache": vc.numpy(),
                  "pd/block_tables": bt.numpy(), "pd/context_lens": ctx.numpy()})
    store["pd/out"] = PD.torch_paged_attention_reference(qd, kc, vc, bt, ctx, P).numpy()

    rows, n_tok = 50, 5
    ks = torch.randn(rows, 1, 16, generator=g).half()
    qs = torch.randn(n_tok, 4, 16, generator=g).half()
    idx = torch.stack([torch.sort(torch.randperm(rows, generator=g)[:12]).values for _ in range(n_tok)])
    idx = idx.to(torch.int32)
    idx[1, 6:] = -1
    idx[2, :] = -1
    sink = torch.randn(4, generator=g)
    store.update({"sap/q": qs.numpy(), "sap/k": ks.numpy(), "sap/topk_idxs": idx.numpy(),
                  "sap/attn_sink": sink.numpy()})
    cu_s = torch.tensor([0, n_tok], dtype=torch.int32)
    for s_on in (0, 1):
        store[f"sap/out_s{s_on}"] = SA.torch_sparse_prefill_reference(
            qs, ks, ks, idx, cu_s, attn_sink=sink if s_on else None).numpy()

    ctx_d = torch.tensor([1, 3, 16, 17], dtype=torch.int32)
    n_win, n_comp, K = 4, 9, 10
    kcd, vcd = (torch.randn(12, 1, P, 16, generator=g).half() for _ in range(2))
    btd = torch.randperm(12, generator=g)[:8].view(4, 2).to(torch.int32)
    ck, cv = (torch.randn(n_comp, 1, 16, generator=g).half() for _ in range(2))
    qdd = torch.randn(4, 4, 16, generator=g).half()
    idd = torch.full((4, K), -1, dtype=torch.int32)
    for b in range(4):
        c = int(ctx_d[b])
        for i in range(n_win):
            if c - n_win + i >= 0:
                idd[b, i] = c - n_win + i
        pick = torch.sort(torch.randperm(n_comp, generator=g)[:K - n_win - b % 2]).values
        idd[b, n_win:n_win + pick.shape[0]] = c + pick.to(torch.int32)
    store.update({"sad/q": qdd.numpy(), "sad/k_cache": kcd.numpy(), "sad/v_cache": vcd.numpy(),
                  "sad/compressed_k": ck.numpy(), "sad/compressed_v": cv.numpy(), "sad/block_tables": btd.numpy(),
                  "sad/topk_idxs": idd.numpy(), "sad/context_lens": ctx_d.numpy(), "sad/attn_sink": sink.numpy()})
    for s_on in (0, 1):
        store[f"sad/out_s{s_on}"] = SA.torch_sparse_decode_reference(
            qdd, kcd, vcd, ck, cv, btd, idd, ctx_d, block_size=P, attn_sink=sink if s_on else None).numpy()


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout>/attention")
    ref = sys.argv[1]
    main(ref)
    main_edges(ref)

"""CPU-side checks of the boundary: the C-ABI library loads and exports every
symbol include/tak_attention.h declares, the ctypes signatures cover exactly
those symbols, and the drop-in modules keep the reference's call signatures
and refuse non-CUDA tensors the way the reference refuses non-NPU ones."""

import ctypes
import inspect
import os
import re

import pytest
import torch

import _tak_b200 as T

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "tak_attention.h")


def header_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tak_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    if not os.path.exists(T.LIB_PATH):
        pytest.skip("libtak_b200.so not built (run __graft_entry__.build())")
    h = ctypes.CDLL(T.LIB_PATH)
    syms = header_symbols()
    assert len(syms) >= 15
    for s in syms:
        assert hasattr(h, s), f"{s} declared in tak_attention.h but not exported"
    assert set(T._SIGS) == set(syms), "ctypes table and header disagree"
    assert T.lib().tak_version().decode().startswith("tak-b200")


def test_reference_signatures_kept():
    import flash_attention_prefill as FP
    import paged_attention_decode as PD
    import sparse_attn_fwd as SA
    import csa as CSA
    import hca as HCA

    def pos(fn):
        return [(p.name, p.default) for p in inspect.signature(fn).parameters.values()
                if p.kind == p.POSITIONAL_OR_KEYWORD]

    E = inspect.Parameter.empty
    assert pos(FP.flash_attention_prefill) == [("q", E), ("k", E), ("v", E), ("cu_seqlens", E), ("causal", True)]
    assert pos(PD.paged_attention_decode) == [("q", E), ("k_cache", E), ("v_cache", E), ("block_tables", E),
                                              ("context_lens", E), ("block_size", 16), ("block_n", 16)]
    assert pos(SA.sparse_attn_prefill) == [("q", E), ("k", E), ("v", E), ("topk_idxs", E), ("cu_seqlens", E),
                                           ("attn_sink", None)]
    assert [n for n, _ in pos(SA.sparse_attn_decode)] == [
        "q", "k_cache", "v_cache", "compressed_k", "compressed_v", "block_tables", "topk_idxs", "context_lens",
        "num_win", "block_size", "attn_sink"]
    assert [n for n, _ in pos(SA.build_token_to_seq)] == ["cu_seqlens", "total_tokens", "device"]
    assert [n for n, _ in pos(CSA.compress_kv_overlap)] == ["k", "v", "cu_seqlens", "m"]
    assert [n for n, _ in pos(CSA.build_csa_topk_idxs)] == ["q", "compressed_k", "cu_seqlens", "comp_offsets",
                                                           "n_win", "top_k", "m"]
    assert [n for n, _ in pos(CSA.csa_prefill_forward)] == ["q", "k", "v", "cu_seqlens", "n_win", "top_k", "m",
                                                           "attn_sink"]
    assert [n for n, _ in pos(CSA.csa_decode_forward)] == ["q", "k_cache", "v_cache", "block_tables",
                                                          "context_lens", "n_win", "top_k", "m", "block_size",
                                                          "attn_sink"]
    assert [n for n, _ in pos(HCA.compress_kv_simple)] == ["k", "v", "cu_seqlens", "m_prime"]
    assert [n for n, _ in pos(HCA.build_hca_topk_idxs)] == ["cu_seqlens", "comp_offsets", "total_tokens", "n_win",
                                                           "m_prime"]
    assert [n for n, _ in pos(HCA.hca_prefill_forward)] == ["q", "k", "v", "cu_seqlens", "n_win", "m_prime",
                                                           "attn_sink"]
    assert [n for n, _ in pos(HCA.hca_decode_forward)] == ["q", "k_cache", "v_cache", "block_tables",
                                                          "context_lens", "n_win", "m_prime", "block_size",
                                                          "attn_sink"]


def test_cpu_tensors_rejected_like_the_reference():
    import flash_attention_prefill as FP
    import paged_attention_decode as PD
    import sparse_attn_fwd as SA

    q = torch.zeros(4, 2, 8)
    with pytest.raises(AssertionError):
        FP.flash_attention_prefill(q, q[:, :1], q[:, :1], torch.tensor([0, 4], dtype=torch.int32))
    with pytest.raises(AssertionError):
        PD.paged_attention_decode(q, torch.zeros(2, 1, 16, 8), torch.zeros(2, 1, 16, 8),
                                  torch.zeros(4, 1, dtype=torch.int32), torch.ones(4, dtype=torch.int32))
    with pytest.raises(AssertionError):
        SA.sparse_attn_prefill(q, q[:, :1], q[:, :1], torch.zeros(4, 2, dtype=torch.int32), None)


def test_missing_library_raises(monkeypatch):
    """Without libtak_b200.so the first call raises: there is no fallback."""
    monkeypatch.setattr(T, "LIB_PATH", os.path.join(REPO, "no-such-dir", "libtak_b200.so"))
    monkeypatch.setattr(T, "_lib", None)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        T.lib()


def test_product_modules_do_not_use_the_oracle():
    """The drop-in modules and the C ABI sources neither import nor name the
    CPU oracle (it is test infrastructure only)."""
    pkg = os.path.join(REPO, "triton-ascend-kernels_b200")
    for root, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                src = open(os.path.join(root, f)).read()
                assert "oracle" not in src, f"{f} names the oracle"


def test_paged_decode_block_n_assertion():
    import paged_attention_decode as PD

    # PD:121-123: block_n must divide block_size and not exceed it
    q = torch.zeros(1, 1, 8)
    with pytest.raises(AssertionError):
        PD.paged_attention_decode(q, q, q, q, q, block_size=16, block_n=32)


def test_workspace_size_is_host_only():
    if not os.path.exists(T.LIB_PATH):
        pytest.skip("libtak_b200.so not built")
    n = T.lib().tak_paged_attention_decode_workspace_size(64, 32, 8, 128, 128, 64, 0)
    assert n > 64 * 32 * 130 * 4
    # one page per split: one partial per page
    n1 = T.lib().tak_paged_attention_decode_workspace_size(2, 4, 1, 128, 16, 10, 1)
    assert n1 >= 2 * 4 * 10 * 130 * 4


def test_comp_offsets_host_matches_oracle():
    from oracle import attention_oracle as O

    for lens, st in (([0, 3, 4, 5, 130], 4), ([256, 512, 384], 128), ([], 4), ([1], 128)):
        assert T.comp_offsets_host(lens, st) == O.comp_offsets_for(lens, st).tolist()


def test_indexer_workspace_size_is_host_only():
    if not os.path.exists(T.LIB_PATH):
        pytest.skip("libtak_b200.so not built")
    L = T.lib()
    # rows x max slots rounded up to 128 x element size (bf16 = 1, fp32 = 2)
    assert L.tak_csa_indexer_workspace_size(65536, 1024, 1) == 65536 * 1024 * 2
    assert L.tak_csa_indexer_workspace_size(64, 2042, 1) == 64 * 2048 * 2
    assert L.tak_csa_indexer_workspace_size(10, 1, 2) == 10 * 128 * 4
    assert L.tak_csa_indexer_workspace_size(0, 100, 1) == 0


def test_prefix_view_and_slot_bounds():
    kc = torch.zeros(6, 1, 16, 576)
    assert T.is_prefix_view(kc, kc)
    assert T.is_prefix_view(kc[..., :512], kc)              # MLA: V = the first 512 latent columns
    assert not T.is_prefix_view(kc[..., 64:], kc)           # another offset
    assert not T.is_prefix_view(torch.zeros(6, 1, 16, 512), kc)
    assert not T.is_prefix_view(kc[:3], kc)                 # fewer pages
    bt = torch.zeros(4, 64, dtype=torch.int32)
    assert T.max_slots_per_seq(bt, 128, 4) == 2048          # 64 pages x 128 rows / m
    assert T.max_slots_per_seq(bt, 128, 128) == 64
    assert T.max_slots_per_seq(torch.zeros(4, 0, dtype=torch.int32), 16, 4) == 1


def _header_params():
    """{entry point: [parameter names]} parsed from tak_attention.h."""
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for name, params in re.findall(r"\b(tak_\w+)\s*\(([^)]*)\)\s*;", src):
        ps = [p.strip() for p in params.split(",") if p.strip() and p.strip() != "void"]
        out[name] = [re.findall(r"(\w+)\s*$", p)[0] for p in ps]
    return out


# a host stride array for arguments whose values are copied before the checked one
# (the pointers given with it are never dereferenced: validation fails first)
_S4 = (ctypes.c_int64 * 4)(0, 0, 0, 0)


def _call_invalid(name, **vals):
    """Call entry point `name` with null pointers, zero sizes and `vals`."""
    params = _header_params()[name]
    argtypes = T._SIGS[name][0]
    assert len(params) == len(argtypes), name
    unknown = set(vals) - set(params)
    assert not unknown, (name, unknown)
    args = [vals.get(p, None if t is T._P else (1.0 if t is T._F32 else 0)) for p, t in zip(params, argtypes)]
    rc = getattr(T.lib(), name)(*args)
    return rc, T.lib().tak_last_error().decode()


@pytest.mark.skipif(torch.cuda.is_available(), reason="argument checks only, on a machine without a GPU")
@pytest.mark.parametrize("name,vals,msg", [
    ("tak_flash_attention_prefill", dict(dtype=5, num_q_heads=8, num_kv_heads=2, head_dim=128), "unknown dtype"),
    ("tak_flash_attention_prefill", dict(dtype=1, num_q_heads=8, num_kv_heads=3, head_dim=128), "heads"),
    ("tak_flash_attention_prefill", dict(dtype=1, num_q_heads=8, num_kv_heads=2, head_dim=1000), "head_dim"),
    ("tak_flash_attention_prefill", dict(dtype=1, num_q_heads=8, num_kv_heads=2, head_dim=128, num_seqs=1,
                                         total_tokens=4), "null"),
    ("tak_paged_attention_decode", dict(dtype=1, num_q_heads=32, num_kv_heads=8, head_dim=128, block_size=256,
                                        cache_rows=128), "block_size"),
    ("tak_paged_attention_decode", dict(dtype=1, num_q_heads=32, num_kv_heads=8, head_dim=128, block_size=16,
                                        cache_rows=16, num_seqs=2, max_blocks=4, num_blocks=8), "null"),
    ("tak_sparse_attn_prefill", dict(dtype=1, total_tokens=4, num_q_heads=64, num_kv_heads=1, head_dim=576,
                                     head_dim_v=0), "head dims"),
    ("tak_sparse_attn_decode", dict(dtype=1, num_seqs=2, num_q_heads=64, num_kv_heads=1, head_dim=512,
                                    head_dim_v=512, k_topk=-1), "negative"),
    ("tak_sparse_attn_decode", dict(dtype=1, num_seqs=2, num_q_heads=64, num_kv_heads=1, head_dim=512,
                                    head_dim_v=512, k_topk=4, topk_idxs=8, topk_strides=_S4, q=8, q_strides=_S4,
                                    out=8, out_strides=_S4, k_cache=8, k_strides=_S4, v_cache=8, v_strides=_S4,
                                    block_tables=8, bt_strides=_S4, context_lens=8, block_size=16, max_blocks=-1),
     "max_blocks"),
    ("tak_compress_kv", dict(dtype=1, stride=0, window=8, num_kv_heads=1, head_dim=512, num_compressed=4),
     "stride"),
    # no V given but a V head dim: the K-only form needs head_dim_v = 0
    ("tak_compress_kv_paged", dict(dtype=1, stride=4, window=8, num_kv_heads=1, head_dim=512, head_dim_v=512,
                                   num_compressed=4), "head sizes"),
    ("tak_compress_kv_paged", dict(dtype=1, stride=4, window=8, num_kv_heads=1, head_dim=512, num_compressed=4,
                                   k_cache=8, k_strides=_S4, comp_offsets=8, compressed_k=8, ck_strides=_S4,
                                   block_tables=8, bt_strides=_S4, context_lens=8, block_size=16, num_blocks=-1),
     "num_blocks"),
    ("tak_paged_attention_decode_static_scratch", dict(dtype=7, num_q_heads=32, num_kv_heads=8, head_dim=128),
     "unknown dtype"),
    ("tak_paged_attention_decode_static_scratch", dict(dtype=1, num_q_heads=32, num_kv_heads=8, head_dim=-4,
                                                       num_seqs=4096, max_blocks=64, block_size=128,
                                                       cache_rows=128), "head_dim"),
    ("tak_compress_kv_csa_hca", dict(dtype=1, m=0, m_prime=128, num_csa=4, num_kv_heads=1, head_dim=512,
                                     head_dim_v=512), "null v"),
    ("tak_build_window_idxs", dict(num_seqs=1, total_tokens=4, n_win=8, ld=4), "bad arguments"),
    ("tak_build_decode_topk_idxs", dict(num_seqs=1, n_win=8, n_comp_cols=4, ld=8), "decode idxs"),
    ("tak_comp_offsets", dict(num_seqs=1, stride=0), "comp offsets"),
    ("tak_csa_indexer_topk", dict(dtype=1, m=4, top_k=32, n_win=8, ld=16, num_q_heads=8, num_kv_heads=1,
                                  head_dim=512), "null pointer"),
    ("tak_build_token_to_seq", dict(num_seqs=-1, total_tokens=4), "token_to_seq"),
])
def test_c_abi_rejects_invalid_arguments(name, vals, msg):
    """Every entry point validates its arguments before touching the device:
    status 1 (invalid argument) and a message naming the problem, the C-side
    counterpart of the reference wrappers' asserts (FP:124-133, PD:120-129,
    SA:274-280, SA:337-343)."""
    if not os.path.exists(T.LIB_PATH):
        pytest.skip("libtak_b200.so not built")
    rc, err = _call_invalid(name, **vals)
    assert rc == 1, (name, rc, err)
    assert msg in err, (name, err)


@pytest.mark.skipif(torch.cuda.is_available(), reason="argument checks only, on a machine without a GPU")
@pytest.mark.parametrize("name,vals", [
    ("tak_sparse_attn_prefill", dict(total_tokens=0)),
    ("tak_sparse_attn_decode", dict(num_seqs=0)),
    ("tak_compress_kv", dict(num_compressed=0)),
    ("tak_compress_kv_paged", dict(num_compressed=0)),
    ("tak_compress_kv_csa_hca", dict(num_csa=0, num_hca=0)),
])
def test_c_abi_empty_inputs_succeed(name, vals):
    """Empty inputs (no tokens, requests or slots) return 0 with nothing
    launched and no pointer read, where the reference's host loops simply do
    nothing."""
    if not os.path.exists(T.LIB_PATH):
        pytest.skip("libtak_b200.so not built")
    rc, err = _call_invalid(name, **vals)
    assert rc == 0, (name, rc, err)

"""One-launch prefill + decode (mixed_step.prefill_and_decode) against the two
separate entry points and the CPU oracle.

The reference runs flash_attention_prefill (attention/flash_attention_prefill.py
:108-171) and paged_attention_decode (attention/paged_attention_decode.py
:104-151) as separate launches; the persistent kernel must return what they
return: prefill rows and LSE, decode outputs and LSE (split combines done by
the last split to finish).  Tolerances: bf16 max-abs <= 2e-2 of the float64
oracle, LSE <= 1e-3; against the separate launches 1e-2 (the same math,
compiled into another kernel).
"""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu

import _tak_b200 as T  # noqa: E402
import flash_attention_prefill as FP  # noqa: E402
import mixed_step as MS  # noqa: E402
import paged_attention_decode as PD  # noqa: E402

DEV = "cuda"
TOL16, TOL_LSE = 2e-2, 1e-3


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert T.read_device_error() == 0, "a kernel reported a timed-out wait"


def _prefill_case(lens, seed, H=64, Hkv=8, D=128):
    g = torch.Generator().manual_seed(seed)
    Tn = sum(lens)
    q = torch.randn(Tn, H, D, generator=g).to(DEV, torch.bfloat16)
    k = torch.randn(Tn, Hkv, D, generator=g).to(DEV, torch.bfloat16)
    v = torch.randn(Tn, Hkv, D, generator=g).to(DEV, torch.bfloat16)
    cu = torch.tensor([0] + np.cumsum(lens).tolist(), dtype=torch.int32, device=DEV)
    return q, k, v, cu


def _decode_case(ctx, seed, P=128, H=32, Hkv=8, D=128, max_ctx=8192):
    g = torch.Generator().manual_seed(seed)
    B = len(ctx)
    maxb = (max_ctx + P - 1) // P
    pool = sum((c + P - 1) // P for c in ctx) + 4
    perm = torch.randperm(pool, generator=g).to(torch.int32)
    bt = torch.zeros(B, maxb, dtype=torch.int32)
    i = 0
    for b, c in enumerate(ctx):
        n = (c + P - 1) // P
        bt[b, :n] = perm[i:i + n]
        i += n
    kc = torch.randn(pool, Hkv, P, D, generator=g).to(DEV, torch.bfloat16)
    vc = torch.randn(pool, Hkv, P, D, generator=g).to(DEV, torch.bfloat16)
    qd = torch.randn(B, H, D, generator=g).to(DEV, torch.bfloat16)
    return qd, kc, vc, bt.to(DEV), torch.tensor(ctx, dtype=torch.int32, device=DEV)


def _diff(a, b):
    return (a.float() - b.float()).abs().max().item() if a.numel() else 0.0


def _lse_diff(a, b):
    fin = torch.isfinite(b)
    assert torch.equal(torch.isfinite(a), fin)
    return (a[fin] - b[fin]).abs().max().item() if fin.any() else 0.0


@pytest.mark.parametrize("causal", [True, False])
def test_mixed_step_matches_separate_launches_and_oracle(causal):
    """Prefill of five sequences (64/8 heads, d 128; lengths past several
    256-row blocks, one off the grid) and decode of 40 requests (32/8 heads,
    page 128, contexts up to 8192: one to many splits, ctx 0 and 1) in one
    launch, twice in a row (the work-queue counters are cleared per call)."""
    lens = [300, 1000, 77, 2048, 513]
    q, k, v, cu = _prefill_case(lens, 11)
    g = torch.Generator().manual_seed(12)
    ctx = torch.randint(1, 8193, (40,), generator=g).tolist()
    ctx[3], ctx[7], ctx[9] = 0, 1, 8192
    qd, kc, vc, bt, cl = _decode_case(ctx, 13)
    ref_p, ref_pl = FP.flash_attention_prefill(q, k, v, cu, causal, return_lse=True)
    ref_d, ref_dl = PD.paged_attention_decode(qd, kc, vc, bt, cl, 128, 128, return_lse=True)
    for call in range(2):
        (op, opl), (od, odl) = MS.prefill_and_decode(q, k, v, cu, qd, kc, vc, bt, cl, 128, causal, return_lse=True)
        assert T.last_kernel() == "mixed_step"
        torch.cuda.synchronize()
        assert _diff(op, ref_p) <= 1e-2 and _lse_diff(opl, ref_pl) <= 1e-4, f"call {call}: prefill"
        assert _diff(od, ref_d) <= 1e-2 and _lse_diff(odl, ref_dl) <= 1e-4, f"call {call}: decode"
    # the oracle on every decode request and on the three shorter sequences
    rd, rdl = O.paged_decode(qd.float().cpu().numpy(), kc.float().cpu().numpy(), vc.float().cpu().numpy(),
                             bt.cpu(), cl.cpu(), 128, acc=np.float32)
    assert np.abs(od.float().cpu().numpy() - rd).max() <= TOL16
    fin = np.isfinite(rdl)
    assert np.abs(odl.cpu().numpy()[fin] - rdl[fin]).max() <= TOL_LSE
    short = [0, 1, 2]
    cuh = cu.cpu().tolist()
    for s in short:
        a, b = cuh[s], cuh[s + 1]
        rp, rpl = O.prefill(q[a:b].float().cpu().numpy(), k[a:b].float().cpu().numpy(),
                            v[a:b].float().cpu().numpy(), [0, b - a], causal, acc=np.float32)
        assert np.abs(op[a:b].float().cpu().numpy() - rp).max() <= TOL16
        assert np.abs(opl[a:b].cpu().numpy() - rpl).max() <= TOL_LSE


def test_mixed_step_long_contexts_and_many_splits():
    """Decode-heavy step: 96 requests with contexts up to 131072 tokens (up to
    64 splits each, merged by the last split) beside a short prefill."""
    q, k, v, cu = _prefill_case([700, 129], 21)
    g = torch.Generator().manual_seed(22)
    ctx = torch.randint(1, 131073, (96,), generator=g).tolist()
    qd, kc, vc, bt, cl = _decode_case(ctx, 23, max_ctx=131072)
    ref_p = FP.flash_attention_prefill(q, k, v, cu, True)
    ref_d, ref_dl = PD.paged_attention_decode(qd, kc, vc, bt, cl, 128, 128, return_lse=True)
    (op, _), (od, odl) = MS.prefill_and_decode(q, k, v, cu, qd, kc, vc, bt, cl, 128, True, return_lse=True)
    assert T.last_kernel() == "mixed_step"
    assert _diff(op, ref_p) <= 1e-2
    assert _diff(od, ref_d) <= 1e-2 and _lse_diff(odl, ref_dl) <= 1e-4
    pick = [0, 17, 50, 95]
    idx = torch.tensor(pick, device=DEV)
    rd, _ = O.paged_decode(qd[idx].float().cpu().numpy(), kc.float().cpu().numpy(), vc.float().cpu().numpy(),
                           bt[idx].cpu(), cl[idx].cpu(), 128, acc=np.float32)
    assert np.abs(od[idx].float().cpu().numpy() - rd).max() <= TOL16


def test_mixed_step_other_shapes_run_back_to_back():
    """Pages of 16 rows (not a multiple of the 64-row chunk the one-launch
    kernel streams): the two kernels run back to back with the same results;
    an empty decode batch runs the prefill alone."""
    q, k, v, cu = _prefill_case([300, 64], 31)
    qd, kc, vc, bt, cl = _decode_case([1, 500, 33], 32, P=16, max_ctx=512)
    op, od = MS.prefill_and_decode(q, k, v, cu, qd, kc, vc, bt, cl, 16, True)
    assert T.last_kernel() == "paged_decode_tc"
    assert _diff(op, FP.flash_attention_prefill(q, k, v, cu, True)) == 0.0
    assert _diff(od, PD.paged_attention_decode(qd, kc, vc, bt, cl, 16, 16)) <= 1e-2
    qd0 = qd[:0]
    op, od = MS.prefill_and_decode(q, k, v, cu, qd0, kc, vc, bt[:0], cl[:0], 16, True)
    assert od.shape[0] == 0 and T.last_kernel() == "prefill_tc"
    assert _diff(op, FP.flash_attention_prefill(q, k, v, cu, True)) == 0.0

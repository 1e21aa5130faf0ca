"""Benchmark of the attention hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|prefill|sparse|compress]

Default workload (the configuration the headline metric is quoted on): paged
decode, batch 64 requests x one query token, 32 query heads / 8 KV heads,
head_dim 128, bf16, context lengths U[1, 8192], page size 128, block tables
drawn from a random permutation of a 5000-page pool, K/V ~ N(0, 1).  A "step"
is one paged_attention_decode call over the whole batch.  The KV pool
(2 x 1.31 GB) and the bytes one step reads (~1.07 GB) are far larger than the
126 MB L2, so no flush is needed between steps.

N > 1 (torchrun, one process per GPU): every rank serves its own batch of 64
requests (seed + rank) -- weak scaling, no collective on the data path; the
outputs are all-gathered to every rank over NCCL after the timed region
(timed separately).  value = bytes of all ranks / max-over-ranks time.

--impl reference: the reference's math on the host CPU (the numpy oracle of
this repository, the reference being Python/PyTorch for an Ascend NPU that
cannot run here), all host threads, over a bounded sample of the same batch
per step; rank 0 only.
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "triton-ascend-kernels_b200", "attention"))

METRIC = "prefill/sparse TFLOP/s & decode HBM GB/s per B200 (% peak), 1/2/4/8 GPUs"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def profile_traffic(name):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu
    summary (line 'traffic_bytes_per_launch: <n>'), or None."""
    p = os.path.join(REPO, "profiles", name)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# paged decode workload (default)
# ---------------------------------------------------------------------------

DEC = dict(batch=64, q_heads=32, kv_heads=8, head_dim=128, page=128, pool=5000, max_ctx=8192)


def decode_inputs(seed, device):
    c = DEC
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(1, c["max_ctx"] + 1, (c["batch"],), generator=g, dtype=torch.int64).to(torch.int32)
    maxb = c["max_ctx"] // c["page"]
    perm = torch.randperm(c["pool"], generator=g).to(torch.int32)
    bt = torch.zeros(c["batch"], maxb, dtype=torch.int32)
    i = 0
    for b in range(c["batch"]):
        n = (int(ctx[b]) + c["page"] - 1) // c["page"]
        bt[b, :n] = perm[i:i + n]
        i += n
    q = torch.randn(c["batch"], c["q_heads"], c["head_dim"], generator=g).to(torch.bfloat16)
    shape = (c["pool"], c["kv_heads"], c["page"], c["head_dim"])
    if device is None:
        return q, None, None, bt, ctx
    kc = torch.empty(shape, dtype=torch.bfloat16, device=device)
    vc = torch.empty(shape, dtype=torch.bfloat16, device=device)
    gd = torch.Generator(device=device).manual_seed(seed + 1000)
    kc.normal_(generator=gd)
    vc.normal_(generator=gd)
    return q, kc, vc, bt, ctx


def decode_bytes(ctx):
    """Algorithmic HBM bytes of one step: every valid K and V row once
    (H_kv x D x 2 B each), q in, out written, block-table and length reads."""
    c = DEC
    kv = int(ctx.sum()) * c["kv_heads"] * c["head_dim"] * 2 * 2
    qo = 2 * c["batch"] * c["q_heads"] * c["head_dim"] * 2
    meta = int(((ctx + c["page"] - 1) // c["page"]).sum()) * 4 + c["batch"] * 4
    return kv + qo + meta


def cpu_decode_sample(q, ctx, pages, seconds, threads):
    """Time the oracle (numpy, fp32) on the sampled requests, cycling over them
    for about `seconds`; returns (GB/s of algorithmic bytes, requests, seconds)."""
    from concurrent.futures import ThreadPoolExecutor
    from threadpoolctl import threadpool_limits

    from oracle import attention_oracle as O

    c = DEC
    qn = q.float().numpy()
    sample = sorted(pages)

    def one(b):
        kc, vc = pages[b]
        O.paged_decode(qn[b:b + 1], kc, vc, np.arange(kc.shape[0])[None, :], ctx[b:b + 1].numpy(), c["page"],
                       acc=np.float32)
        return int(ctx[b]) * c["kv_heads"] * c["head_dim"] * 2 * 2 + 2 * c["q_heads"] * c["head_dim"] * 2

    done_bytes, n = 0, 0
    with threadpool_limits(limits=1), ThreadPoolExecutor(max_workers=threads) as ex:
        t0 = time.perf_counter()
        i = 0
        while time.perf_counter() - t0 < seconds:
            batch = [sample[(i + j) % len(sample)] for j in range(threads)]
            done_bytes += sum(ex.map(one, batch))
            n += len(batch)
            i += threads
        dt = time.perf_counter() - t0
    return done_bytes / dt / 1e9, n, dt


def host_pages(kc, vc, bt, ctx, sample):
    """Host copies of the sampled requests' pages (contiguous [n_pages, H_kv, P, D])."""
    c = DEC
    out = {}
    for b in sample:
        n = (int(ctx[b]) + c["page"] - 1) // c["page"]
        pages = bt[b, :n].long().to(kc.device)
        out[b] = (kc[pages].float().cpu().numpy(), vc[pages].float().cpu().numpy())
    return out


def run_decode_ours(args, rank, world, device):
    import paged_attention_decode as PD
    import _tak_b200 as T

    pk, pk_kind = peaks()
    q, kc, vc, bt, ctx = decode_inputs(1234 + rank, device)
    qd, btd, ctxd = q.to(device), bt.to(device), ctx.to(device)
    stream = torch.cuda.current_stream(device)

    def step():
        return PD.paged_attention_decode(qd, kc, vc, btd, ctxd, DEC["page"], DEC["page"])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    # launches per step: main kernel (+ split-KV combine when there are splits)
    L = T.lib()
    ws = L.tak_paged_attention_decode_workspace_size(DEC["batch"], DEC["q_heads"], DEC["kv_heads"], DEC["head_dim"],
                                                     DEC["page"], bt.shape[1], 0)
    launches_per_step = 2 if ws > 256 + DEC["batch"] * DEC["q_heads"] * (DEC["head_dim"] + 2) * 4 else 1

    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(device.index) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            out = step()
        ev1.record(stream)
        torch.cuda.synchronize(device)
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        torch.distributed.barrier()
    nbytes = decode_bytes(ctx)

    # end to end through the public API with host buffers: q / block tables /
    # context lengths copied in from pinned memory, output copied back, every step
    qh, bth, ctxh = q.pin_memory(), bt.pin_memory(), ctx.pin_memory()
    outh = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    qe, bte, ctxe = torch.empty_like(qd), torch.empty_like(btd), torch.empty_like(ctxd)

    def e2e_step():
        qe.copy_(qh, non_blocking=True)
        bte.copy_(bth, non_blocking=True)
        ctxe.copy_(ctxh, non_blocking=True)
        o = PD.paged_attention_decode(qe, kc, vc, bte, ctxe, DEC["page"], DEC["page"])
        outh.copy_(o, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = e0.elapsed_time(e1) / args.steps
    h2d = qh.numel() * qh.element_size() + bth.numel() * 4 + ctxh.numel() * 4
    d2h = outh.numel() * outh.element_size()

    gather_ms = None
    if world > 1:
        t = torch.tensor([ms, e2e_ms, float(nbytes)], dtype=torch.float64, device=device)
        mx = t.clone()
        torch.distributed.all_reduce(mx, op=torch.distributed.ReduceOp.MAX)
        tot = t.clone()
        torch.distributed.all_reduce(tot, op=torch.distributed.ReduceOp.SUM)
        ms, e2e_ms, nbytes_all = float(mx[0]), float(mx[1]), float(tot[2])
        outs = [torch.empty_like(out) for _ in range(world)]
        torch.cuda.synchronize(device)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        torch.distributed.all_gather(outs, out)
        g1.record(stream)
        torch.cuda.synchronize(device)
        gather_ms = g0.elapsed_time(g1)
    else:
        nbytes_all = float(nbytes)

    if rank != 0:
        return None
    gbs = nbytes_all / (ms * 1e-3) / 1e9
    per_launch_gbs = nbytes / (ms * 1e-3) / 1e9
    hbm = pk["hbm_gbs"]
    traffic = profile_traffic("paged_decode_cfg2.md")
    res = {
        "metric": METRIC,
        "value": round(gbs, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V and q, context lengths U[1,8192])",
        "config": {
            "workload": "paged decode: batch 64 x 1 token, 32 q heads / 8 KV heads, head_dim 128, bf16, "
                        "ctx U[1,8192], page 128, 5000-page pool, random-permutation block tables",
            "per_gpu_batch": DEC["batch"], "kv_pool_bytes": 2 * DEC["pool"] * DEC["kv_heads"] * DEC["page"]
            * DEC["head_dim"] * 2, "l2_policy": "inputs larger than L2 (1.07 GB read per step, 2.6 GB pool)",
            "parallelism": f"request sharding x{world} (weak scaling)",
            "pct_of_hbm_peak": round(100 * per_launch_gbs / hbm, 1), "pct_of_spec_8tbs": round(per_launch_gbs / 80, 1),
        },
        "roofline": {"bound": "hbm", "achieved": round(per_launch_gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(per_launch_gbs / hbm, 4), "traffic": traffic,
                     "peak_source": f"{pk_kind} hbm_gbs", "algorithmic_bytes_per_launch": nbytes,
                     "timed": "paged_decode_tc_kernel + split-KV combine per step, CUDA events"},
        "e2e": {"value": round(nbytes_all / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "note": "public paged_attention_decode() with q / block tables / context lengths copied from "
                        "pinned host memory and the output copied back every step; the KV cache is resident"},
        "gpu_launches": args.steps * launches_per_step,
        "clocks": clk.summary(),
    }
    if gather_ms is not None:
        res["config"]["output_all_gather_ms"] = round(gather_ms, 3)
    if not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        sample = list(range(0, DEC["batch"], 8))
        v, n, dt = cpu_decode_sample(q, ctx, host_pages(kc, vc, bt, ctx, sample), args.cpu_seconds, threads)
        res["cpu_baseline"] = {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                               "sample": f"requests {sample} of the batch, cycled {n} times through the numpy "
                                         f"oracle (the reference's math, fp32) for {dt:.1f} s on {threads} threads; "
                                         f"algorithmic bytes as the GPU figure"}
    return res


def run_decode_reference(args):
    """The reference math on the host CPU: the numpy oracle over a bounded
    sample of the batch each step (16 of the 64 requests), all host threads."""
    from concurrent.futures import ThreadPoolExecutor
    from threadpoolctl import threadpool_limits

    from oracle import attention_oracle as O

    c = DEC
    q, _, _, bt, ctx = decode_inputs(1234, None)
    threads = os.cpu_count() or 1
    g = np.random.default_rng(7)
    sample = list(range(0, c["batch"], 4))
    # host K/V for the sampled requests only (the full pool does not fit a quick CPU run)
    pages = {b: (g.standard_normal(((int(ctx[b]) + c["page"] - 1) // c["page"], c["kv_heads"], c["page"],
                                     c["head_dim"]), dtype=np.float32),
                 g.standard_normal(((int(ctx[b]) + c["page"] - 1) // c["page"], c["kv_heads"], c["page"],
                                    c["head_dim"]), dtype=np.float32)) for b in sample}
    qn = q.float().numpy()

    def one(b):
        kc, vc = pages[b]
        O.paged_decode(qn[b:b + 1], kc, vc, np.arange(kc.shape[0])[None, :], ctx[b:b + 1].numpy(), c["page"],
                       acc=np.float32)

    sample_bytes = sum(int(ctx[b]) * c["kv_heads"] * c["head_dim"] * 2 * 2 + 2 * c["q_heads"] * c["head_dim"] * 2
                       for b in sample)
    with threadpool_limits(limits=1), ThreadPoolExecutor(max_workers=threads) as ex:
        for _ in range(args.warmup):
            list(ex.map(one, sample))
        t0 = time.perf_counter()
        for _ in range(args.steps):
            list(ex.map(one, sample))
        dt = (time.perf_counter() - t0) / args.steps
    v = sample_bytes / dt / 1e9
    return {
        "impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "GB/s", "n_gpus": 0,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "paged decode: batch 64 x 1 token, 32 q heads / 8 KV heads, head_dim 128, "
                               "ctx U[1,8192], page 128 -- 16 of the 64 requests per step",
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"requests {sample[0]}..{sample[-1]} step 4 of the batch per step, numpy oracle "
                                   f"(the reference's math), fp32, {threads} threads"},
        "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["decode"], default="decode")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_decode_reference(args)), flush=True)
        return

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=device)
    res = run_decode_ours(args, rank, world, device)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()

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
import itertools
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


def timed_steps(run, steps, warmup, device):
    """Device ms per step of run(n), which executes exactly n steps: warm-up
    steps first, then one CUDA-event bracket around all timed steps."""
    run(warmup)
    torch.cuda.synchronize(device)
    st = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    run(steps)
    e1.record(st)
    torch.cuda.synchronize(device)
    return e0.elapsed_time(e1) / steps


def capture_graph(fn, device, warm=3):
    """CUDA graph of one step.  The step is first run on the capture stream so
    that everything it caches per stream (the decode workspace, for one) exists
    before capture; replays then launch exactly the step's kernels."""
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        for _ in range(warm):
            fn()
    torch.cuda.current_stream(device).wait_stream(s)
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        out = fn()
    torch.cuda.synchronize(device)
    return g, out


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


def decode_inputs(seed, device, world=1, rank=0):
    """One global batch of 64 x world requests from one seed, assigned to
    ranks by the longest-processing-time rule on context length
    (sharding.shard_requests: the bytes each request streams).  Weak scaling:
    the batch at N GPUs holds the 64 context lengths of the one-GPU batch N
    times over (fresh queries for every copy), so each GPU's share streams the
    same bytes as the one-GPU step.  Returns this rank's (q, k_cache, v_cache,
    block_tables, context_lens) and every rank's global request ids.  Each
    rank holds its own 5000-page pool; its requests' pages are drawn in order
    from one random permutation of it.  At world = 1 this is the single-GPU
    batch: requests 0..63 in order."""
    import sharding
    c = DEC
    g = torch.Generator().manual_seed(seed)
    n = c["batch"] * world
    ctx_all = torch.randint(1, c["max_ctx"] + 1, (c["batch"],), generator=g, dtype=torch.int64).to(torch.int32)
    ctx_all = ctx_all.repeat(world)
    maxb = c["max_ctx"] // c["page"]
    perm = torch.randperm(c["pool"], generator=g).to(torch.int32)
    q_all = torch.randn(n, c["q_heads"], c["head_dim"], generator=g).to(torch.bfloat16)
    ids = [sharding.shard_requests(ctx_all, world, r) for r in range(world)]
    mine = ids[rank]
    ctx, q = ctx_all[mine], q_all[mine]
    bt = torch.zeros(ctx.numel(), maxb, dtype=torch.int32)
    i = 0
    for b in range(ctx.numel()):
        npg = (int(ctx[b]) + c["page"] - 1) // c["page"]
        bt[b, :npg] = perm[i:i + npg]
        i += npg
    assert i <= c["pool"]
    shape = (c["pool"], c["kv_heads"], c["page"], c["head_dim"])
    if device is None:
        return q, None, None, bt, ctx, ids
    kc = torch.empty(shape, dtype=torch.bfloat16, device=device)
    vc = torch.empty(shape, dtype=torch.bfloat16, device=device)
    gd = torch.Generator(device=device).manual_seed(seed + 1000 + rank)
    kc.normal_(generator=gd)
    vc.normal_(generator=gd)
    return q, kc, vc, bt, ctx, ids


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


class PipelinedE2E:
    """End-to-end steps through a public API with host buffers, pipelined:
    step i's host-to-device copies run on a copy stream while step i - 1
    computes, and step i - 1's device-to-host copy on a second copy stream
    while step i computes (two device buffer sets, ordered by events).  The
    timed region starts before the first copy in and ends after the last copy
    back, so every step's copies are inside it.  `compute` takes the device
    copies of `host_inputs` and returns one output tensor or a tuple of them;
    `outputs` lists their (shape, dtype).  The copies back of consecutive
    steps are ordered on their stream, so one pinned host set receives them."""

    def __init__(self, host_inputs, compute, outputs, device, copy_back=True, post=None):
        self.hin = [t if t.is_pinned() else t.pin_memory() for t in host_inputs]
        self.sets = [[torch.empty(t.shape, dtype=t.dtype, device=device) for t in self.hin] for _ in range(2)]
        self.compute = compute
        self.post = post  # runs on the copy-back stream after compute (the NCCL output gather)
        self.copy_back = copy_back
        self.hout = [torch.empty(sh, dtype=dt).pin_memory() for sh, dt in outputs] if copy_back else None
        self.h2d = torch.cuda.Stream(device)
        self.d2h = torch.cuda.Stream(device)
        self.comp = torch.cuda.current_stream(device)
        self.ev_in = [torch.cuda.Event() for _ in range(2)]
        self.ev_done = [torch.cuda.Event() for _ in range(2)]
        self.device = device
        self.i = 0

    def h2d_bytes(self):
        return sum(t.numel() * t.element_size() for t in self.hin)

    def d2h_bytes(self):
        return sum(t.numel() * t.element_size() for t in self.hout) if self.copy_back else 0

    def step(self):
        b = self.i % 2
        with torch.cuda.stream(self.h2d):
            if self.i >= 2:
                self.h2d.wait_event(self.ev_done[b])  # step i - 2 has finished with this buffer set
            for d, h in zip(self.sets[b], self.hin):
                d.copy_(h, non_blocking=True)
            self.ev_in[b].record(self.h2d)
        self.comp.wait_event(self.ev_in[b])
        o = self.compute(*self.sets[b])
        outs = o if isinstance(o, (tuple, list)) else (o,)
        self.ev_done[b].record(self.comp)
        if self.copy_back or self.post is not None:
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.ev_done[b])
                res = outs
                if self.post is not None:
                    r = self.post(*outs)
                    res = r if isinstance(r, (tuple, list)) else (r,)
                if self.copy_back:
                    for h, d in zip(self.hout, res):
                        h.copy_(d, non_blocking=True)
            if not torch.cuda.is_current_stream_capturing():
                for d in outs:
                    d.record_stream(self.d2h)
        self.i += 1

    def capture(self, n):
        """One CUDA graph of n consecutive pipelined steps (copy streams and
        events included), so that the host's launch cost per step -- the
        public call's Python wrapper, the copies, the events -- cannot leave the
        device idle, as in a serving engine that replays its decode step from a
        graph.  n is even: the graph ends on the buffer set it starts on."""
        assert n % 2 == 0 and self.i % 2 == 0
        g = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(self.device)
        cap.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(cap):
            self.compute(*self.sets[0])  # per-stream caches (the decode workspace) exist before capture
        torch.cuda.synchronize(self.device)
        saved = self.comp
        with torch.cuda.graph(g, stream=cap):
            self.comp = cap
            self.h2d.wait_stream(cap)
            self.d2h.wait_stream(cap)
            i0 = self.i
            self.i = 0  # within the graph no step waits on a step before it
            for _ in range(n):
                self.step()
            cap.wait_stream(self.h2d)
            cap.wait_stream(self.d2h)
            self.i = i0
        self.comp = saved
        torch.cuda.synchronize(self.device)
        return g

    def timed(self, steps, warmup, world, graph_steps=0):
        """Device ms per step over exactly `steps` steps.  With graph_steps,
        whole graphs of that many steps are replayed (the remainder runs as
        plain steps)."""
        g = self.capture(graph_steps) if graph_steps else None
        for _ in range(warmup):
            self.step()
        torch.cuda.synchronize(self.device)
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(self.device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if g is None:
            e0.record(self.h2d)
            for _ in range(steps):
                self.step()
            e1.record(self.d2h if (self.copy_back or self.post is not None) else self.comp)
        else:
            st = torch.cuda.current_stream(self.device)
            e0.record(st)
            for _ in range(steps // graph_steps):
                g.replay()
            st.wait_stream(self.h2d)
            st.wait_stream(self.d2h)
            rem = steps % graph_steps
            if rem:
                self.h2d.wait_stream(st)
                self.d2h.wait_stream(st)
                self.comp.wait_stream(st)
                for _ in range(rem):
                    self.step()
                st.wait_stream(self.comp)
                st.wait_stream(self.d2h)
            e1.record(st)
        torch.cuda.synchronize(self.device)
        return e0.elapsed_time(e1) / steps


def run_decode_ours(args, rank, world, device):
    import paged_attention_decode as PD
    import _tak_b200 as T
    import sharding

    pk, pk_kind = peaks()
    q, kc, vc, bt, ctx, ids = decode_inputs(1234, device, world, rank)
    qd, btd, ctxd = q.to(device), bt.to(device), ctx.to(device)
    stream = torch.cuda.current_stream(device)
    B = q.shape[0]

    def step():
        return PD.paged_attention_decode(qd, kc, vc, btd, ctxd, DEC["page"], DEC["page"])

    run, graph = step, None
    if not args.no_graph:
        graph, out = capture_graph(step, device)
        run = graph.replay
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize(device)
    # launches per step: main kernel (+ split-KV combine when there are splits)
    L = T.lib()
    ws = L.tak_paged_attention_decode_workspace_size(B, DEC["q_heads"], DEC["kv_heads"], DEC["head_dim"],
                                                     DEC["page"], bt.shape[1], 0)
    launches_per_step = 2 if ws > 0 else 1

    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(device.index) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            if graph is None:
                out = step()
            else:
                run()
        ev1.record(stream)
        torch.cuda.synchronize(device)
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        torch.distributed.barrier()
    nbytes = decode_bytes(ctx)

    # the output gather over NCCL (N > 1): one all_gather_into_tensor of
    # fixed-size blocks, sizes and placement from the sharding plan
    gather = sharding.PlannedGather([len(i) for i in ids], ids) if world > 1 else None
    gather_ms = None
    if gather is not None:
        for _ in range(3):
            gather(out)
        torch.cuda.synchronize(device)
        torch.distributed.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 20
        g0.record(stream)
        for _ in range(reps):
            gather(out)
        g1.record(stream)
        torch.cuda.synchronize(device)
        gather_ms = g0.elapsed_time(g1) / reps

    # end to end through the public API with host buffers: q / block tables /
    # context lengths copied in from pinned memory every step, the output
    # (gathered from every rank at N > 1) copied back to rank 0's host
    def e2e_compute(qe, bte, ctxe):
        return PD.paged_attention_decode(qe, kc, vc, bte, ctxe, DEC["page"], DEC["page"])

    # the gather runs on the copy-back stream, so step i's gather overlaps step i + 1's kernels
    n_all = sum(len(i) for i in ids)
    e2e = PipelinedE2E([q, bt, ctx], e2e_compute, [((n_all,) + tuple(q.shape[1:]), q.dtype)], device,
                       copy_back=rank == 0, post=gather)
    # one GPU: eight pipelined steps per CUDA graph (host launch cost off the
    # device's critical path); more GPUs: plain steps (the NCCL gather stays
    # outside graphs)
    e2e_ms = e2e.timed(args.steps, args.warmup, world, graph_steps=8 if world == 1 and not args.no_graph else 0)
    h2d, d2h = e2e.h2d_bytes(), e2e.d2h_bytes()

    per_rank = None
    if world > 1:
        t = torch.tensor([ms, e2e_ms, float(nbytes), float(h2d), float(d2h), float(B)], dtype=torch.float64,
                         device=device)
        allv = torch.empty(world, t.numel(), dtype=torch.float64, device=device)
        torch.distributed.all_gather_into_tensor(allv, t)
        allv = allv.cpu()
        per_rank = [{"rank": r, "ms": round(float(allv[r, 0]), 4), "e2e_ms": round(float(allv[r, 1]), 4),
                     "gb": round(float(allv[r, 2]) / 1e9, 4), "requests": int(allv[r, 5])} for r in range(world)]
        ms, e2e_ms = float(allv[:, 0].max()), float(allv[:, 1].max())
        nbytes_all = float(allv[:, 2].sum())
        h2d, d2h = int(allv[:, 3].sum()), int(allv[:, 4].sum())
    else:
        nbytes_all = float(nbytes)

    if rank != 0:
        return None
    gbs = nbytes_all / (ms * 1e-3) / 1e9
    per_launch_gbs = nbytes / (ms * 1e-3) / 1e9
    hbm = pk["hbm_gbs"]
    traffic = profile_traffic("paged_decode_tc_kernel_decode_b64_ctx8k.md")
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
            "workload": "paged decode: batch 64 x 1 token per GPU, 32 q heads / 8 KV heads, head_dim 128, bf16, "
                        "ctx U[1,8192], page 128, 5000-page pool per GPU, random-permutation block tables",
            "per_gpu_batch": DEC["batch"], "kv_pool_bytes": 2 * DEC["pool"] * DEC["kv_heads"] * DEC["page"]
            * DEC["head_dim"] * 2, "l2_policy": "inputs larger than L2 (1.07 GB read per step, 2.6 GB pool)",
            "parallelism": (f"request sharding x{world}: one batch of {64 * world} requests from one seed, "
                            "assigned by longest-processing-time on context length (weak scaling)"
                            if world > 1 else "one GPU"),
            "pct_of_hbm_peak": round(100 * per_launch_gbs / hbm, 1), "pct_of_spec_8tbs": round(per_launch_gbs / 80, 1),
        },
        "roofline": {"bound": "hbm", "achieved": round(per_launch_gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(per_launch_gbs / hbm, 4), "traffic": traffic,
                     "peak_source": f"{pk_kind} hbm_gbs", "algorithmic_bytes_per_launch": nbytes,
                     "timed": "paged_decode_tc_kernel + split-KV combine per step, CUDA events"
                              + ("; each step a CUDA-graph replay of paged_attention_decode()" if graph is not None
                                 else "")},
        "e2e": {"value": round(nbytes_all / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "note": "public paged_attention_decode() with q / block tables / context lengths copied from pinned "
                        "host memory and the output copied back every step, copies on two copy streams overlapping "
                        "the neighbouring steps' kernels (two buffer sets); the KV cache is resident"
                        + ("; eight such steps (calls, copies and events) replayed per CUDA graph, as a serving "
                           "engine replays its decode step" if world == 1 and not args.no_graph else "")
                        + ("; includes the NCCL all-gather of every rank's output (on the copy-back stream, "
                           "overlapping the next step's kernels) and rank 0's copy of the whole result"
                           if world > 1 else "")},
        "gpu_launches": args.steps * launches_per_step,
        "clocks": clk.summary(),
    }
    if gather_ms is not None:
        res["config"]["output_all_gather_ms"] = round(gather_ms, 4)
        res["config"]["output_all_gather"] = (f"one all_gather_into_tensor of {max(len(i) for i in ids)}-request "
                                              "blocks (sizes from the sharding plan) + one index_select into "
                                              "request order, CUDA events over 20 calls")
        res["config"]["per_rank"] = per_rank
    if not args.no_cpu_baseline and world == 1:
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
    q, _, _, bt, ctx, _ = decode_inputs(1234, None)
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


# ---------------------------------------------------------------------------
# other workloads of the metric (prefill / sparse TFLOP/s, compression GB/s)
# ---------------------------------------------------------------------------

class Workload:
    """One hot-path workload: device-resident step, end-to-end step through the
    public API with host buffers, algorithmic work per step, and a bounded
    sample of it on host inputs through the numpy oracle (CPU baseline and the
    reference arm)."""
    name = unit = bound = peak_key = kernel = desc = ""
    # ncu summary under profiles/ whose capture is this workload's dominant
    # launch ("" = none: the roofline's traffic is then null)
    profile = ""
    graph_free = True  # steps run eagerly (set per run: False while CUDA graphs replay them)

    def reference_sample(self):
        """(step, work per step, text): one bounded oracle step on host inputs."""
        raise NotImplementedError

    def scale(self):
        return 1e12 if self.unit == "TFLOP/s" else 1e9

    def cpu_baseline(self, seconds, threads):
        step, work, text = self.reference_sample()
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds or n == 0:
            step()
            n += 1
        dt = time.perf_counter() - t0
        return n * work / dt / self.scale(), f"{n} x {text}, {dt:.1f} s, {threads} BLAS threads"

    def timed(self, fn, steps, warmup, device):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(device)
        st = torch.cuda.current_stream(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            fn()
        e1.record(st)
        torch.cuda.synchronize(device)
        return e0.elapsed_time(e1) / steps


def _loguniform_lengths(n, lo, hi, g):
    u = torch.rand(n, generator=g, dtype=torch.float64)
    return [int(round(math.exp(math.log(lo) + float(x) * (math.log(hi) - math.log(lo))))) for x in u]


class PrefillWL(Workload):
    name, unit, bound, peak_key, kernel = "prefill", "TFLOP/s", "tensor", "bf16_tflops", "prefill_tc_kernel"
    profile = "prefill_tc_kernel_varlen_32seq.md"
    desc = ("varlen causal prefill: 32 sequences (one GPU's share of 256), lengths log-uniform in [512, 32768], "
            "64 q heads / 8 KV heads, head_dim 128, bf16")

    def setup(self, rank, device):
        import flash_attention_prefill as FP
        import sharding
        self.FP = FP
        # one batch of 32 x world sequences from one seed, assigned to ranks by
        # longest-processing-time on causal attention cost L(L+1)/2
        g = torch.Generator().manual_seed(4321)
        lens_all = _loguniform_lengths((4 if SMALL else 32) * self.world, 512, 32768, g)
        owner = sharding.lpt_assign(sharding.prefill_costs(lens_all), self.world)
        self.lens = [L for L, o in zip(lens_all, owner) if o == rank]
        self.rows_per_rank = [sum(L for L, o in zip(lens_all, owner) if o == r) for r in range(self.world)]
        T = sum(self.lens)
        cu = [0]
        for L in self.lens:
            cu.append(cu[-1] + L)
        self.cu_h = torch.tensor(cu, dtype=torch.int32)
        gd = torch.Generator(device=device).manual_seed(99 + rank)
        self.q = torch.empty(T, 64, 128, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.k = torch.empty(T, 8, 128, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.v = torch.empty(T, 8, 128, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.cu = self.cu_h.to(device)
        self.work = 4.0 * 128 * 64 * sum(L * (L + 1) / 2 for L in self.lens)
        self.launches = 1
        self.config = {"sequences": len(self.lens), "total_tokens": T, "max_len": max(self.lens),
                       "l2_policy": f"inputs larger than L2 ({(T * 80 * 128 * 2) / 1e9:.2f} GB of q/k/v)"}
        if self.world > 1:
            self.config["assignment"] = (f"one batch of {len(lens_all)} sequences, longest-processing-time on "
                                         "L(L+1)/2 across ranks")

    def step(self):
        return self.FP.flash_attention_prefill(self.q, self.k, self.v, self.cu, True)

    def e2e_pipeline(self):
        """Host q / k / v / cu_seqlens in, the output back, through the public
        flash_attention_prefill()."""
        def fn(q, k, v, cu):
            return self.FP.flash_attention_prefill(q, k, v, cu, True)
        return [self.q.cpu(), self.k.cpu(), self.v.cpu(), self.cu_h], fn, [(tuple(self.q.shape), self.q.dtype)]

    def reference_sample(self):
        from oracle import attention_oracle as O
        L = 1024
        g = np.random.default_rng(1)
        q = g.standard_normal((L, 64, 128), dtype=np.float32)
        k = g.standard_normal((L, 8, 128), dtype=np.float32)
        v = g.standard_normal((L, 8, 128), dtype=np.float32)
        return (lambda: O.prefill(q, k, v, [0, L], True, acc=np.float32), 4.0 * 128 * 64 * L * (L + 1) / 2,
                "one causal 1024-token sequence (64/8 heads, d 128) through the numpy oracle, fp32")


class SparseWL(Workload):
    name, unit, bound, peak_key, kernel = "sparse", "TFLOP/s", "tensor", "bf16_tflops", "sparse_tc_kernel"
    profile = "sparse_tc_kernel_mla_16x4096_top2048.md"
    desc = ("top-k sparse attention with sinks: 16 sequences x 4096 query tokens over a 32768-token latent KV, "
            "MQA 64 heads, QK dim 576 (512 + 64 rope), V dim 512 (view of the latent), bf16, 2048 sorted unique "
            "causal indices per query, per-head sink logits")

    def setup(self, rank, device):
        import sparse_attn_fwd as SA
        self.SA = SA
        S, QT, KVL, K = (1 if SMALL else 16), 4096, 32768, 2048
        gd = torch.Generator(device=device).manual_seed(77 + rank)
        T = S * QT
        self.rows_per_rank = [T] * self.world  # every rank serves 16 equal sequences
        self.q = torch.empty(T, 64, 576, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.kv = torch.empty(S * KVL, 1, 576, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.sink = torch.empty(64, device=device).normal_(generator=gd)
        idx = torch.empty(T, K, dtype=torch.int32, device=device)
        pos_all = torch.arange(KVL - QT, KVL, device=device)
        ar = torch.arange(KVL, device=device)
        for s in range(S):
            for c0 in range(0, QT, 512):
                pos = pos_all[c0:c0 + 512]
                r = torch.rand(pos.numel(), KVL, device=device, generator=gd)
                r = torch.where(ar[None, :] <= pos[:, None], r, torch.full_like(r, 2.0))
                sel = torch.topk(r, K, dim=1, largest=False).indices.sort(dim=1).values
                idx[s * QT + c0:s * QT + c0 + pos.numel()] = (sel + s * KVL).to(torch.int32)
        self.idx = idx
        self.cu = torch.arange(0, T + 1, QT, dtype=torch.int32, device=device)
        self.work = 2.0 * 64 * (576 + 512) * T * K
        self.launches = 1
        self.config = {"tokens": T, "kv_rows": S * KVL, "top_k": K,
                       "l2_policy": "per-sequence latent KV (37.7 MB) fits L2 by design; q/out 9 GB stream"}

    def step(self):
        return self.SA.sparse_attn_prefill(self.q, self.kv, self.kv[..., :512], self.idx, self.cu, self.sink)

    def e2e_pipeline(self):
        """Host q / latent KV / index rows in, the output back, through the
        public sparse_attn_prefill()."""
        def fn(q, kv, idx):
            return self.SA.sparse_attn_prefill(q, kv, kv[..., :512], idx, self.cu, self.sink)
        return ([self.q.cpu(), self.kv.cpu(), self.idx.cpu()], fn,
                [((self.q.shape[0], 64, 512), self.q.dtype)])

    def reference_sample(self):
        from oracle import attention_oracle as O
        n_tok, KVL, K = 4, 32768, 2048
        g = np.random.default_rng(2)
        q = g.standard_normal((n_tok, 64, 576), dtype=np.float32)
        kv = g.standard_normal((KVL, 1, 576), dtype=np.float32)
        idx = np.stack([np.sort(g.choice(KVL - n_tok + i + 1, K, replace=False)) for i in range(n_tok)]).astype(np.int32)
        sink = g.standard_normal(64).astype(np.float32)
        return (lambda: O.sparse_prefill(q, kv, kv[..., :512], idx, None, sink, acc=np.float32),
                n_tok * 2.0 * 64 * 1088 * K,
                f"{n_tok} query tokens (64 heads, 2048 causal indices into a 32768-row latent, 576/512) "
                "through the numpy oracle, fp32")


class CompressWL(Workload):
    name, unit, bound, peak_key, kernel = "compress", "GB/s", "hbm", "hbm_gbs", "compress_dual_kernel"
    profile = "compress_dual_kernel_csa_hca_65536tok.md"
    desc = ("CSA + HCA KV compression: 65536 tokens (16 sequences x 4096) x 512 dims bf16 K and V plus per-token "
            "fp32 gate logits; CSA stride 4 (8-token windows, as the reference's csa.py) and HCA 128-token "
            "windows, gate-softmax-weighted sums")

    def setup(self, rank, device):
        import csa as CSA
        import hca as HCA
        self.CSA, self.HCA = CSA, HCA
        gd = torch.Generator(device=device).manual_seed(55 + rank)
        T = 65536
        self.rows_per_rank = [T // 4] * self.world  # CSA slots per rank (16 equal sequences)
        self.k = torch.empty(T, 1, 512, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.v = torch.empty(T, 1, 512, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.gate = torch.empty(T, device=device).normal_(generator=gd)
        self.cu_h = torch.arange(0, T + 1, 4096, dtype=torch.int32)
        # algorithmic bytes: read K, V and the gates once, write both compressed outputs
        self.work = 2 * T * 512 * 2 + T * 4 + 2 * (T // 4) * 512 * 2 + 2 * (T // 128) * 512 * 2
        self.launches = 1
        self.out_sets = 8
        self.config = {"tokens": T, "csa_slots": T // 4, "hca_slots": T // 128,
                       "l2_policy": "inputs (134 MB of K/V) larger than L2; each step writes one of 8 output sets "
                                    "(277 MB in all), so no step rewrites outputs still in L2",
                       "timed_path": "one tak_compress_kv_csa_hca launch (CSA and HCA outputs) per step through "
                                     "the C ABI"}

        # device step: one launch through the C ABI with the offsets, outputs
        # and argument list prepared once (the public wrapper sizes its outputs
        # on the host each call; the e2e leg below goes through it)
        import _tak_b200 as TK
        self.TK = TK
        dev = self.k.device
        self.cu_d = self.cu_h.to(dev)
        self.sets = []
        for _ in range(self.out_sets):
            bufs = []
            for stride in (4, 128):
                offs = TK.comp_offsets_host([4096] * 16, stride)
                nc = offs[-1]
                bufs.append((torch.tensor(offs, dtype=torch.int32, device=dev), nc,
                             torch.empty(nc, 1, 512, device=dev, dtype=torch.bfloat16),
                             torch.empty(nc, 1, 512, device=dev, dtype=torch.bfloat16)))
            (co, nc, ck, cv), (ho, nh, hk, hv) = bufs
            args = (TK.ptr(self.k), TK.strides(self.k), TK.ptr(self.v), TK.strides(self.v), TK.ptr(self.gate), 1,
                    TK.ptr(self.cu_d), 16, T, TK.ptr(co), nc, TK.ptr(ck), TK.strides(ck), TK.ptr(cv),
                    TK.strides(cv), TK.ptr(ho), nh, TK.ptr(hk), TK.strides(hk), TK.ptr(hv), TK.strides(hv), 1, 512,
                    512, 4, 128, 1)
            self.sets.append((bufs, args))
        self.set_i = 0
        self.use_outputs(0)
        self.fn = TK.lib().tak_compress_kv_csa_hca

    def use_outputs(self, i):
        self.outs, self.args = self.sets[i % self.out_sets]

    def step(self):
        self.TK.check(self.fn(*self.args, self.TK.stream_of(self.k)))
        out = self.outs[0][2]
        if self.graph_free:
            # eager steps rotate the output sets themselves
            self.set_i += 1
            self.use_outputs(self.set_i)
        return out

    def e2e_pipeline(self):
        """Host K / V / gates in, all four outputs (CSA K/V, HCA K/V) back,
        through the public compress_kv_csa_hca()."""
        def fn(k, v, g):
            (ck, cv, _), (hk, hv, _) = self.CSA.compress_kv_csa_hca(k, v, self.cu_h, 4, 128, gate=g)
            return ck, cv, hk, hv
        outs = [((n, 1, 512), torch.bfloat16) for n in (65536 // 4, 65536 // 4, 65536 // 128, 65536 // 128)]
        return [self.k.cpu(), self.v.cpu(), self.gate.cpu()], fn, outs

    def reference_sample(self):
        from oracle import attention_oracle as O
        T = 4096
        g = np.random.default_rng(3)
        k = g.standard_normal((T, 1, 512), dtype=np.float32)
        v = g.standard_normal((T, 1, 512), dtype=np.float32)
        gate = g.standard_normal(T).astype(np.float32)

        def one():
            O.compress_kv(k, v, [0, T], 4, 8, gate, acc=np.float32)
            O.compress_kv(k, v, [0, T], 128, 128, gate, acc=np.float32)

        return (one, 2 * T * 512 * 2 + T * 4 + 2 * (T // 4) * 512 * 2 + 2 * (T // 128) * 512 * 2,
                "one 4096-token sequence, CSA + HCA gated, through the numpy oracle, fp32")


class CsaWL(Workload):
    name, unit, bound, peak_key, kernel = "csa", "TFLOP/s", "tensor", "bf16_tflops", "sparse_tc_kernel"
    desc = ("CSA prefill forward over the compressed latent: 65536 tokens (16 sequences x 4096), 64 query heads on "
            "one 512-dim latent used as K and V, bf16; gated CSA compression (m = 4, 8-token windows), "
            "Lightning-indexer top-512 compressed slots + 128-token window per query, sparse attention with sinks")
    graphable = False  # the reference-compatible wrapper sizes outputs from host-side offsets each call

    def setup(self, rank, device):
        import csa as CSA
        self.CSA = CSA
        S, QT = (2 if SMALL else 16), 4096
        T = S * QT
        gd = torch.Generator(device=device).manual_seed(61 + rank)
        self.q = torch.empty(T, 64, 512, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.kv = torch.empty(T, 1, 512, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.gate = torch.empty(T, device=device).normal_(generator=gd)
        self.sink = torch.empty(64, device=device).normal_(generator=gd)
        self.cu_h = torch.arange(0, T + 1, QT, dtype=torch.int32)
        self.n_win, self.top_k, self.m = 128, 512, 4
        # attention work = every non-negative index (the reference also attends
        # the non-causal picks of a row that has fewer than top_k causal slots)
        ck, cv, offs = CSA.compress_kv_overlap(self.kv, self.kv, self.cu_h, self.m, gate=self.gate)
        idx = CSA.build_csa_topk_idxs(self.q, ck, self.cu_h, offs, self.n_win, self.top_k, self.m)
        n_idx = int((idx >= 0).sum())
        self.work = 2.0 * 64 * (512 + 512) * n_idx
        self.launches = 5
        self.config = {"tokens": T, "indices_per_query": self.n_win + self.top_k, "valid_indices": n_idx,
                       "l2_policy": "q (4.3 GB) and outputs stream; the 1.3 MB latent per sequence is L2-resident",
                       "timed_path": "csa_prefill_forward(): compression, window rows, Lightning indexer and "
                                     "sparse attention over the latent and compressed rows in place, every step"}

    def step(self):
        return self.CSA.csa_prefill_forward(self.q, self.kv, self.kv, self.cu_h, self.n_win, self.top_k, self.m,
                                            self.sink, gate=self.gate)

    def phases(self, device):
        """Device time of each stage of one forward (ms), eager."""
        CSA = self.CSA
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        torch.cuda.synchronize(device)
        ev[0].record()
        ck, cv, offs = CSA.compress_kv_overlap(self.kv, self.kv, self.cu_h, self.m, gate=self.gate)
        ev[1].record()
        idx = CSA.build_csa_topk_idxs(self.q, ck, self.cu_h, offs, self.n_win, self.top_k, self.m)
        ev[2].record()
        CSA.sparse_attn_prefill_two_sources(self.q, self.kv, self.kv, ck, ck, idx, attn_sink=self.sink)
        ev[3].record()
        torch.cuda.synchronize(device)
        return {"compress_ms": round(ev[0].elapsed_time(ev[1]), 3), "index_ms": round(ev[1].elapsed_time(ev[2]), 3),
                "attention_ms": round(ev[2].elapsed_time(ev[3]), 3)}

    def e2e_pipeline(self):
        """Host q / latent / gate logits in, the output back, through the
        public csa_prefill_forward() (which reads the compressed-slot offsets
        on the host each call, as the reference's does)."""
        def fn(q, kv, gate):
            return self.CSA.csa_prefill_forward(q, kv, kv, self.cu_h, self.n_win, self.top_k, self.m,
                                                self.sink, gate=gate)
        return ([self.q.cpu(), self.kv.cpu(), self.gate.cpu()], fn, [(tuple(self.q.shape), torch.bfloat16)])

    def reference_sample(self):
        from oracle import attention_oracle as O
        L = 512
        g = np.random.default_rng(4)
        q = g.standard_normal((L, 64, 512), dtype=np.float32)
        kv = g.standard_normal((L, 1, 512), dtype=np.float32)
        sink = g.standard_normal(64).astype(np.float32)
        idx = O.build_csa_topk_idxs(q, O.compress_kv(kv, kv, [0, L], 4, 8)[0], [0, L],
                                    O.comp_offsets_for([L], 4), 128, 512, 4)
        work = 2.0 * 64 * 1024 * int((idx >= 0).sum())
        return (lambda: O.csa_prefill_forward(q, kv, kv, [0, L], 128, 512, 4, sink),
                work, "one 512-token sequence through the numpy oracle's csa_prefill_forward (64 heads, 512-dim "
                      "latent, window 128 + top-512), fp32")


def csa_decode_bytes(ctx, n_idx, B, H, D, n_win, top_k, m):
    """Algorithmic HBM bytes of one CSA decode step over a latent cache (V a
    view of K, pooled once): every context row read once by the pooling, the
    compressed rows written, read once by the indexer and gathered once per
    valid index by the attention, plus q, out and the index rows."""
    slots = sum(max(1, -(-int(c) // m)) for c in ctx if c > 0)
    row = D * 2
    return (int(sum(int(c) for c in ctx)) * row + slots * row        # pooling: read context, write slots
            + B * row + slots * row + B * (n_win + top_k) * 4         # indexer: last-head q, slot rows, idx
            + n_idx * row + 2 * B * H * D * 2 + B * (n_win + top_k) * 4)  # attention: gathered rows, q, out, idx


class CsaDecodeWL(Workload):
    name, unit, bound, peak_key, kernel = "csa_decode", "GB/s", "hbm", "hbm_gbs", "compress_bulk_kernel"
    profile = "compress_bulk_kernel_csa_decode_64req.md"
    desc = ("CSA decode forward over a paged latent cache: 64 requests (one query token each, 64 query heads), "
            "one 512-dim latent KV head used as K and V, bf16, contexts uniform in [1, 8192], page 128; "
            "pooling straight from the pages (m = 4, 8-token windows), Lightning-indexer top-512 + 128-token "
            "window, sparse attention with sinks")

    def setup(self, rank, device):
        import csa as CSA
        self.CSA = CSA
        B, H, D, P = (16 if SMALL else 64), 64, 512, 128
        self.P, self.n_win, self.top_k, self.m = P, 128, 512, 4
        g = torch.Generator().manual_seed(71 + rank)
        ctx = torch.randint(1, 8192 + 1, (B,), generator=g, dtype=torch.int64).to(torch.int32)
        maxb = 8192 // P
        pool = B * maxb
        perm = torch.randperm(pool, generator=g).to(torch.int32)
        bt = torch.zeros(B, maxb, dtype=torch.int32)
        i = 0
        for b in range(B):
            n = (int(ctx[b]) + P - 1) // P
            bt[b, :n] = perm[i:i + n]
            i += n
        gd = torch.Generator(device=device).manual_seed(72 + rank)
        self.kc = torch.empty(pool, 1, P, D, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.q = torch.empty(B, H, D, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.sink = torch.empty(H, device=device).normal_(generator=gd)
        self.bt, self.ctx = bt.to(device), ctx.to(device)
        self.ctx_h, self.bt_h = ctx, bt
        # capacity of the compressed rows: the exact slot count, known from the
        # request lengths when the batch is formed (no host read per step)
        self.cap = sum(max(1, -(-int(c) // self.m)) for c in ctx.tolist())
        # valid attention indices: window positions < ctx plus every causal compressed slot picked (<= top_k)
        n_idx = sum(min(int(c), self.n_win) + min(-(-int(c) // self.m), self.top_k) for c in ctx.tolist())
        self.work = csa_decode_bytes(ctx.tolist(), n_idx, B, H, D, self.n_win, self.top_k, self.m)
        self.launches = 5  # slot offsets, pooling, window rows, indexer, sparse attention
        self.out_sets = 4  # four graphs, each with its own compressed rows (4 x 65 MB)
        self.config = {"requests": B, "context_tokens": int(ctx.sum()), "compressed_slots": self.cap,
                       "valid_indices": n_idx,
                       "l2_policy": "the context rows streamed by the pooling (261 MB) exceed L2; consecutive steps "
                                    "replay 4 graphs with separate compressed rows, so no step rewrites rows "
                                    "still in L2",
                       "timed_path": "csa_decode_forward(max_compressed=slots) per step: no host read, "
                                     "captured as one CUDA graph"}

    def step(self):
        return self.CSA.csa_decode_forward(self.q, self.kc, self.kc, self.bt, self.ctx, self.n_win, self.top_k,
                                           self.m, self.P, self.sink, max_compressed=self.cap)

    def phases(self, device):
        """Device time of each stage of one eager forward (ms)."""
        CSA, T = self.CSA, self.CSA._t
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        torch.cuda.synchronize(device)
        ev[0].record()
        ck, cv, offs, _, _ = T.compress_paged(self.kc, self.kc, self.bt, self.ctx, self.P, self.m, 2 * self.m,
                                              capacity=self.cap)
        ev[1].record()
        B = self.q.shape[0]
        K = self.n_win + self.top_k
        idx = torch.empty((B, K), dtype=torch.int32, device=device)
        L, st = T.lib(), T.stream_of(self.q)
        T.check(L.tak_build_decode_topk_idxs(T.ptr(self.ctx), T.ptr(offs), B, self.n_win, self.top_k, 0,
                                             T.ptr(idx), K, st))
        mc = min(T.max_slots_per_seq(self.bt, self.P, self.m), ck.shape[0])
        ws_bytes = L.tak_csa_indexer_workspace_size(B, mc, T.dtype_code(self.q))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
        T.check(L.tak_csa_indexer_topk(T.ptr(self.q), T.strides(self.q), T.ptr(ck), T.strides(ck), None,
                                       T.ptr(self.ctx), T.ptr(offs), B, B, 64, 1, 512, self.n_win, self.top_k,
                                       self.m, mc, T.ptr(idx), K, T.dtype_code(self.q), T.ptr(ws), ws_bytes,
                                       ck.shape[0], st))
        ev[2].record()
        CSA.sparse_attn_decode(self.q, self.kc, self.kc, ck, cv, self.bt, idx, self.ctx, self.n_win, self.P,
                               self.sink)
        ev[3].record()
        torch.cuda.synchronize(device)
        return {"pool_ms": round(ev[0].elapsed_time(ev[1]), 3), "index_ms": round(ev[1].elapsed_time(ev[2]), 3),
                "attention_ms": round(ev[2].elapsed_time(ev[3]), 3)}

    def kernel_roofline(self, device, reps=20):
        """The pooling launch alone (compress_bulk_kernel) through the C ABI,
        CUDA events over `reps` launches after warm-up: (algorithmic bytes
        per launch, ms per launch).  Bytes: every context row read once, every
        slot written once, block-table entries, lengths and offsets."""
        T = self.CSA._t
        offs = T.comp_offsets_device(self.ctx, self.m, self.cap)
        L = T.lib()
        # consecutive launches write different compressed rows (as the steps do)
        sets = []
        for _ in range(self.out_sets):
            ck = torch.empty(self.cap, 1, 512, device=device, dtype=torch.bfloat16)
            sets.append((ck, (T.ptr(self.kc), T.strides(self.kc), None, None, None, None, T.ptr(self.bt),
                              T.strides(self.bt), T.ptr(self.ctx), self.P, self.bt.shape[1], self.kc.shape[0],
                              T.ptr(offs), self.ctx.shape[0], self.cap,
                              T.ptr(ck), T.strides(ck), None, None, 1, 512, 0, self.m, 2 * self.m, T.dtype_code(ck),
                              T.stream_of(ck))))
        ring = itertools.cycle(sets)

        def launch():
            T.check(L.tak_compress_kv_paged(*next(ring)[1]))
        ms = self.timed(launch, reps, 3, device)
        rows = int(self.ctx_h.sum())
        pages = int(((self.ctx_h + self.P - 1) // self.P).sum())
        work = rows * 1024 + self.cap * 1024 + pages * 4 + 2 * self.ctx_h.numel() * 4
        return work, ms

    def e2e_pipeline(self):
        """Per step a serving engine sends the new queries, lengths and block
        tables and reads the output back; the paged latent cache stays
        resident.  The call is the timed step's (max_compressed = the slot
        bound, so it reads nothing back to the host)."""
        def fn(q, ctx, bt):
            return self.CSA.csa_decode_forward(q, self.kc, self.kc, bt, ctx, self.n_win, self.top_k,
                                               self.m, self.P, self.sink, max_compressed=self.cap)
        return ([self.q.cpu(), self.ctx_h, self.bt_h], fn, [(tuple(self.q.shape), torch.bfloat16)])

    def reference_sample(self):
        from oracle import attention_oracle as O
        g = np.random.default_rng(5)
        B, H, D, P = 2, 64, 512, 128
        ctx = np.array([4096, 4096], dtype=np.int32)
        maxb = 4096 // P
        bt = np.arange(B * maxb, dtype=np.int32).reshape(B, maxb)
        kc = g.standard_normal((B * maxb, 1, P, D), dtype=np.float32)
        q = g.standard_normal((B, H, D), dtype=np.float32)
        sink = g.standard_normal(H).astype(np.float32)
        n_idx = sum(min(int(c), 128) + min(-(-int(c) // 4), 512) for c in ctx)
        work = csa_decode_bytes(ctx.tolist(), n_idx, B, H, D, 128, 512, 4)
        return (lambda: O.csa_decode_forward(q, kc, kc, bt, ctx, 128, 512, 4, P, sink),
                work, "two 4096-token requests through the numpy oracle's csa_decode_forward (64 heads, 512-dim "
                      "latent, page 128, window 128 + top-512), fp32")


class MixedWL(Workload):
    """One GPU's share of the box-scale mixed serving step: the global problem
    at N GPUs is N/8 of the 8-GPU step (N x 32 prefill sequences, N x 512
    decode requests), drawn from one seed and assigned to ranks by a greedy
    longest-processing-time rule on estimated roofline time."""
    name, unit, bound, peak_key, kernel = "mixed", "% of roofline", "mixed", None, "mixed_step"
    desc = ("mixed serving step, one GPU's share of 8: varlen causal prefill of 32 sequences with lengths "
            "log-uniform in [512, 32768] (64 q heads / 8 KV heads, d 128, bf16) plus paged decode of 512 requests "
            "with contexts U[1, 131072] (32 q heads / 8 KV heads, d 128, page 128, bf16), requests and sequences "
            "balanced across GPUs by estimated time; the value is the roofline time of the step (prefill FLOPs at "
            "the measured bf16 peak + decode bytes at the measured HBM copy rate) over its measured time")
    world = 1
    POOL = 40960  # pages (21.5 GB of K/V); block tables alias it -- every read still comes from HBM

    def scale(self):
        return 0.01  # work is in roofline seconds: work / seconds / 0.01 = percent

    def setup(self, rank, device):
        import flash_attention_prefill as FP
        import paged_attention_decode as PD
        import sharding
        self.FP, self.PD = FP, PD
        pk, _ = peaks()
        tens, hbm = pk["bf16_tflops"] * 1e12, pk["hbm_gbs"] * 1e9
        world = self.world
        n_pre, n_dec = (4 if SMALL else 32) * world, (64 if SMALL else 512) * world
        g = torch.Generator().manual_seed(20261201)
        lens = _loguniform_lengths(n_pre, 512, 32768, g)
        ctx_all = torch.randint(1, 131072 + 1, (n_dec,), generator=g, dtype=torch.int64)
        pre_cost = [4.0 * 128 * 64 * L * (L + 1) / 2 / tens for L in lens]
        dec_cost = [int(c) * 8 * 128 * 2 * 2 / hbm for c in ctx_all]
        owner = sharding.lpt_assign(pre_cost + dec_cost, world)
        mine_p = [i for i in range(n_pre) if owner[i] == rank]
        mine_d = [b for b in range(n_dec) if owner[n_pre + b] == rank]
        # prefill share
        self.lens = [lens[i] for i in mine_p]
        self.rows_per_rank = [sum(lens[i] for i in range(n_pre) if owner[i] == r) for r in range(world)]
        T = sum(self.lens)
        cu = [0]
        for L in self.lens:
            cu.append(cu[-1] + L)
        gd = torch.Generator(device=device).manual_seed(1000 + rank)
        self.q = torch.empty(T, 64, 128, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.k = torch.empty(T, 8, 128, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.v = torch.empty(T, 8, 128, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.cu = torch.tensor(cu, dtype=torch.int32, device=device)
        # decode share: block tables drawn from the page pool (aliased across requests)
        self.ctx = ctx_all[mine_d].to(torch.int32)
        B = len(mine_d)
        maxb = 131072 // 128
        pool = self.POOL if not SMALL else 4096
        self.bt = torch.randint(0, pool, (max(B, 1), maxb), generator=g, dtype=torch.int32)[:B].contiguous()
        self.kc = torch.empty(pool, 8, 128, 128, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.vc = torch.empty(pool, 8, 128, 128, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.qd = torch.empty(B, 32, 128, device=device, dtype=torch.bfloat16).normal_(generator=gd)
        self.btd, self.ctxd = self.bt.to(device), self.ctx.to(device)
        self.pre_flops = 4.0 * 128 * 64 * sum(L * (L + 1) / 2 for L in self.lens)
        self.dec_bytes = int(self.ctx.to(torch.int64).sum()) * 8 * 128 * 2 * 2 + 2 * B * 32 * 128 * 2
        self.work = self.pre_flops / tens + self.dec_bytes / hbm
        self.launches = 3
        self.config = {"prefill_sequences": len(self.lens), "prefill_tokens": T, "decode_requests": B,
                       "decode_context_tokens": int(self.ctx.to(torch.int64).sum()),
                       "prefill_tflop": round(self.pre_flops / 1e12, 3), "decode_gb": round(self.dec_bytes / 1e9, 3),
                       "roofline_ms": round(self.work * 1e3, 3), "kv_pool_pages": pool,
                       "l2_policy": "inputs larger than L2 (aliased page pool of 21.5 GB)",
                       "assignment": f"LPT over {n_pre} sequences + {n_dec} requests on {world} GPU(s)"}

    def step(self):
        out = self.FP.flash_attention_prefill(self.q, self.k, self.v, self.cu, True)
        self.PD.paged_attention_decode(self.qd, self.kc, self.vc, self.btd, self.ctxd, 128, 128)
        return out

    def phases(self, device):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        torch.cuda.synchronize(device)
        ev[0].record()
        self.FP.flash_attention_prefill(self.q, self.k, self.v, self.cu, True)
        ev[1].record()
        self.PD.paged_attention_decode(self.qd, self.kc, self.vc, self.btd, self.ctxd, 128, 128)
        ev[2].record()
        torch.cuda.synchronize(device)
        pms, dms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
        pk, _ = peaks()
        return {"prefill_ms": round(pms, 3), "prefill_tflops": round(self.pre_flops / (pms * 1e-3) / 1e12, 1),
                "decode_ms": round(dms, 3), "decode_gbs": round(self.dec_bytes / (dms * 1e-3) / 1e9, 1)}

    def e2e_pipeline(self):
        """Host q / k / v of the prefill share and the decode queries, block
        tables and lengths in, both outputs back, through the public
        flash_attention_prefill() and paged_attention_decode(); the paged K/V
        cache stays resident, as in a serving engine."""
        def fn(q, k, v, qd, bt, ctx):
            o1 = self.FP.flash_attention_prefill(q, k, v, self.cu, True)
            o2 = self.PD.paged_attention_decode(qd, self.kc, self.vc, bt, ctx, 128, 128)
            return o1, o2
        return ([self.q.cpu(), self.k.cpu(), self.v.cpu(), self.qd.cpu(), self.bt, self.ctx], fn,
                [(tuple(self.q.shape), torch.bfloat16), (tuple(self.qd.shape), torch.bfloat16)])

    def reference_sample(self):
        from oracle import attention_oracle as O
        pk, _ = peaks()
        g = np.random.default_rng(5)
        L = 1024
        q = g.standard_normal((L, 64, 128), dtype=np.float32)
        k = g.standard_normal((L, 8, 128), dtype=np.float32)
        v = g.standard_normal((L, 8, 128), dtype=np.float32)
        ctx = np.array([4096, 65536], dtype=np.int32)
        npg = [(int(c) + 127) // 128 for c in ctx]
        kc = g.standard_normal((sum(npg), 8, 128, 128), dtype=np.float32)
        vc = g.standard_normal((sum(npg), 8, 128, 128), dtype=np.float32)
        bt = np.zeros((2, max(npg)), np.int32)
        bt[0, :npg[0]] = np.arange(npg[0])
        bt[1, :npg[1]] = np.arange(npg[0], npg[0] + npg[1])
        qd = g.standard_normal((2, 32, 128), dtype=np.float32)

        def one():
            O.prefill(q, k, v, [0, L], True, acc=np.float32)
            O.paged_decode(qd, kc, vc, bt, ctx, 128, acc=np.float32)

        work = 4.0 * 128 * 64 * L * (L + 1) / 2 / (pk["bf16_tflops"] * 1e12) + \
            int(ctx.sum()) * 8 * 128 * 2 * 2 / (pk["hbm_gbs"] * 1e9)
        return one, work, "one causal 1024-token prefill + decode of 2 requests (4096, 65536 tokens), numpy oracle"


WORKLOADS = {"prefill": PrefillWL, "sparse": SparseWL, "compress": CompressWL, "csa": CsaWL, "mixed": MixedWL,
             "csa_decode": CsaDecodeWL}
SMALL = False  # --small: a reduced instance of the workload (for ncu captures)


def run_workload_reference(args, W):
    """The reference math on the host CPU: the workload's bounded oracle step,
    timed over --steps after --warmup, on all host threads."""
    from threadpoolctl import threadpool_limits
    w = W()
    threads = os.cpu_count() or 1
    step, work, text = w.reference_sample()
    with threadpool_limits(limits=threads):
        for _ in range(args.warmup):
            step()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step()
        dt = (time.perf_counter() - t0) / args.steps
    v = work / dt / w.scale()
    return {
        "impl": "reference", "metric": METRIC, "workload": w.name, "value": round(v, 4), "unit": w.unit,
        "n_gpus": 0, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": w.desc, "sample_per_step": text, "parallelism": "host threads"},
        "cpu_baseline": {"value": round(v, 4), "unit": w.unit, "cores": threads, "kind": "port",
                         "sample": f"{text}, one per step, {threads} BLAS threads"},
        "e2e": {"value": round(v, 4), "unit": w.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_workload_ours(args, rank, world, device, W):
    pk, pk_kind = peaks()
    w = W()
    w.world = world
    w.setup(rank, device)
    if world > 1:
        torch.distributed.barrier()
    step_fn = w.step
    graph = None
    # out_sets > 1: consecutive steps write different output memory (one CUDA
    # graph per set, each with its own outputs), so a step never finds the
    # previous step's outputs still dirty in L2 -- a serving loop writes each
    # layer's outputs to fresh memory, and rewriting one buffer would absorb
    # its DRAM write-back
    out_sets = getattr(w, "out_sets", 1)
    w.graph_free = args.no_graph or not getattr(w, "graphable", True)
    multi = None
    if not w.graph_free:
        graphs = []
        for i in range(out_sets):
            if hasattr(w, "use_outputs"):
                w.use_outputs(i)
            graphs.append(capture_graph(w.step, device)[0])
        graph = graphs[0]
        ring = itertools.cycle(graphs)
        step_fn = lambda: next(ring).replay()  # noqa: E731
        if out_sets > 1:
            # the sets' steps back to back in one graph, as a serving loop
            # captures a whole layer stack: a graph boundary between steps
            # costs about 2 us of idle device time, which a step of a few tens
            # of us would otherwise carry.  Exactly K steps are still timed:
            # K // sets replays of it, then the remainder one set at a time.
            def all_sets():
                for i in range(out_sets):
                    if hasattr(w, "use_outputs"):
                        w.use_outputs(i)
                    w.step()
            multi = capture_graph(all_sets, device)[0]
    with Clocks(device.index) as clk:
        if multi is None:
            ms = w.timed(step_fn, args.steps, args.warmup, device)
        else:
            ms = timed_steps(lambda n: [multi.replay() for _ in range(n // out_sets)] +
                             [graphs[i].replay() for i in range(n % out_sets)], args.steps, args.warmup, device)
    if args.no_e2e:
        h2d = d2h = 0
        e2e_ms = float("nan")
    else:
        hin, fn, outs = w.e2e_pipeline()
        pe = PipelinedE2E(hin, fn, outs, device)
        del hin
        # each end-to-end step moves gigabytes over PCIe: a quarter of the
        # steps, at least 3 and at most 8, bounds the run at any --steps
        e2e_ms = pe.timed(min(8, max(3, args.steps // 4)), 2, world)
        h2d, d2h = pe.h2d_bytes(), pe.d2h_bytes()
        del pe
    work_all = float(w.work)
    gather_ms = None
    per_rank = None
    if world > 1:
        # outputs to rank 0 over NCCL, after and outside the timed regions:
        # one gather of fixed-size blocks whose sizes come from the sharding plan
        import sharding
        out = w.step()
        if hasattr(w, "rows_per_rank"):
            gather = sharding.PlannedGather(w.rows_per_rank, dst=0)
        else:
            gather = lambda x: sharding.concat_rows(x, dst=0)  # noqa: E731  (sizes exchanged first)
        gather(out)  # first use of the collective, untimed
        torch.distributed.barrier()
        torch.cuda.synchronize(device)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        gather(out)
        g1.record()
        torch.cuda.synchronize(device)
        gather_ms = g0.elapsed_time(g1)
        del out, gather
        t = torch.tensor([ms, e2e_ms, float(w.work)], dtype=torch.float64, device=device)
        allv = torch.empty(world, 3, dtype=torch.float64, device=device)
        torch.distributed.all_gather_into_tensor(allv, t)
        allv = allv.cpu()
        per_rank = [{"rank": r, "ms": round(float(allv[r, 0]), 4), "work": float(allv[r, 2])} for r in range(world)]
        ms, e2e_ms, work_all = float(allv[:, 0].max()), float(allv[:, 1].max()), float(allv[:, 2].sum())
    if rank != 0:
        return None
    scale = w.scale()
    val = work_all / (ms * 1e-3) / scale
    per_gpu = float(w.work) / (ms * 1e-3) / scale
    peak = pk[w.peak_key] if w.peak_key else 100.0
    res = {
        "metric": METRIC, "workload": w.name, "value": round(val, 1), "unit": w.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
        "config": dict({"workload": w.desc, "parallelism": f"sequence sharding x{world} (weak scaling)"}, **w.config),
        "roofline": {"bound": w.bound, "achieved": round(per_gpu, 1), "peak": peak, "unit": w.unit,
                     "frac": round(per_gpu / peak, 4), "traffic": profile_traffic(w.profile) if w.profile else None,
                     "peak_source": (f"{pk_kind} {w.peak_key} (burst)" if w.peak_key else
                                     f"{pk_kind} bf16_tflops (burst) for prefill + hbm_gbs for decode"),
                     "algorithmic_work_per_step": w.work,
                     "timed": f"{w.kernel} per step (public API, device-resident inputs), CUDA events"
                 + ("" if graph is None else
                    "; each step a CUDA-graph replay of the call" if multi is None else
                    f"; the {out_sets} output sets' steps back to back from one CUDA graph (exactly "
                    f"{args.steps} steps timed)")},
        "e2e": {"value": round(work_all / (e2e_ms * 1e-3) / scale, 2), "unit": w.unit, "ms_per_step": round(e2e_ms, 3),
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "note": ("public API with inputs copied from pinned host memory and outputs copied back every step"
                         + "; copies on two copy streams overlapping the neighbouring steps' kernels"
                         + ("; per GPU, each rank copying its own share" if world > 1 else ""))},
        "gpu_launches": args.steps * w.launches,
        "clocks": clk.summary(),
    }
    if args.no_e2e:
        res["e2e"] = None
    if gather_ms is not None:
        res["config"]["output_gather_to_rank0_ms"] = round(gather_ms, 3)
        res["config"]["per_rank"] = per_rank
    if hasattr(w, "phases"):
        res["config"]["phases"] = w.phases(device)
    if hasattr(w, "kernel_roofline"):
        # a multi-kernel step: the roofline is the dominant kernel timed alone
        kw, kms = w.kernel_roofline(device)
        ka = kw / (kms * 1e-3) / scale
        res["roofline"].update({"achieved": round(ka, 1), "frac": round(ka / peak, 4),
                                "algorithmic_work_per_launch": kw, "kernel_ms": round(kms, 4),
                                "step_achieved": round(per_gpu, 1), "step_frac": round(per_gpu / peak, 4),
                                "timed": f"{w.kernel} alone through the C ABI, CUDA events over 20 launches "
                                         "(the step figures above time the whole step)"})
    sus = pk.get(w.peak_key + "_sustained") if w.peak_key else None
    if sus:
        # the timed loop runs for seconds at the power cap: the sustained GEMM
        # figure of the same file is the matching denominator
        res["roofline"]["peak_sustained"] = sus
        res["roofline"]["frac_of_sustained"] = round(per_gpu / sus, 4)
    if not args.no_cpu_baseline and world == 1:
        from threadpoolctl import threadpool_limits
        threads = os.cpu_count() or 1
        with threadpool_limits(limits=threads):
            v, sample = w.cpu_baseline(args.cpu_seconds, threads)
        res["cpu_baseline"] = {"value": round(v, 4), "unit": w.unit, "cores": threads, "kind": "port",
                               "sample": sample}
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["decode"] + sorted(WORKLOADS), default="decode")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg (profiling)")
    ap.add_argument("--small", action="store_true", help="reduced workload instance (profiling captures)")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch each device-timed step eagerly instead of replaying a CUDA graph of it")
    ap.add_argument("--no-workloads", action="store_true",
                    help="decode only: skip the prefill / sparse / compression lines added to the default run")
    ap.add_argument("--workload-cpu-seconds", type=float, default=5.0,
                    help="CPU-baseline seconds of each added workload")
    args = ap.parse_args()
    global SMALL
    SMALL = args.small
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            if args.workload == "decode":
                print(json.dumps(run_decode_reference(args)), flush=True)
            else:
                print(json.dumps(run_workload_reference(args, WORKLOADS[args.workload])), flush=True)
        return

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=device)
    if args.workload == "decode":
        res = run_decode_ours(args, rank, world, device)
        if not args.no_workloads:
            # the metric's other figures (prefill / sparse TFLOP/s, compression
            # GB/s) and the mixed serving step (at 8 GPUs: the box-scale step),
            # each measured like the headline: same steps and warm-up, own
            # roofline, clocks, end-to-end leg and CPU baseline
            sub_args = argparse.Namespace(**vars(args))
            sub_args.cpu_seconds = args.workload_cpu_seconds
            wl = {}
            for name in ("prefill", "sparse", "compress", "mixed"):
                torch.cuda.empty_cache()
                r = run_workload_ours(sub_args, rank, world, device, WORKLOADS[name])
                if rank == 0:
                    for k in ("metric", "n_gpus", "steps", "warmup", "higher_is_better", "scaling", "vs_baseline",
                              "data"):
                        r.pop(k, None)
                    wl[name] = r
            if rank == 0:
                res["workloads"] = wl
    else:
        res = run_workload_ours(args, rank, world, device, WORKLOADS[args.workload])
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()

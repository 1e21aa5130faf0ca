"""The reference arm of bench.py (the numpy oracle on the host cores) prints
one JSON line with the keys the bench contract needs.  It runs on CPU with a
tiny sample per step; the GPU arm is covered by the bench runs themselves."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("workload", ["decode", "prefill", "sparse", "compress", "csa", "csa_decode", "mixed"])
def test_reference_arm_json_line(workload):
    cmd = [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--workload", workload,
           "--steps", "1", "--warmup", "1", "--cpu-seconds", "0.2"]
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=300, cwd=REPO)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, p.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "steps", "warmup", "ms_per_step", "higher_is_better", "config",
                "cpu_baseline", "e2e", "dtype"):
        assert key in d, key
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["higher_is_better"] is True
    assert d["warmup"] >= 3                              # at least three warm-up steps, whatever is asked
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == d["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def test_roofline_traffic_comes_from_the_workloads_own_capture():
    """Each workload's roofline `traffic` is read from the ncu summary of that
    workload's own dominant launch; a workload without one reports null."""
    sys.path.insert(0, REPO)
    import bench

    assert bench.profile_traffic("paged_decode_tc_kernel_decode_b64_ctx8k.md") > 1e9
    for name, w in bench.WORKLOADS.items():
        if not w.profile:
            continue
        path = os.path.join(REPO, "profiles", w.profile)
        assert os.path.exists(path), (name, w.profile)
        assert w.kernel in open(path).readline(), (name, w.profile)
        assert bench.profile_traffic(w.profile) > 0, (name, w.profile)
    assert not bench.WORKLOADS["csa"].profile     # its summary holds no per-launch traffic of the attention


def test_every_workload_times_a_pipelined_end_to_end_leg():
    """Every workload's `e2e` goes through PipelinedE2E: host inputs copied in
    on one copy stream while the previous step computes, outputs copied back
    on another, all inside the timed region."""
    sys.path.insert(0, REPO)
    import bench

    for name, w in bench.WORKLOADS.items():
        assert callable(getattr(w, "e2e_pipeline", None)), name

"""bench.py's reference arm on the CPU: the JSON line the driver reads.

The reference arm times the reference's own CPU loop (oracle/_ref when built,
else the C restatement) and needs no GPU, so its contract is checked here on
configuration 0 (N = 10k) with a one-second sample.
"""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
                        "tsne_10k", "--steps", "20", "--warmup", "3", "--cpu-seconds", "1"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, lines
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "tsne_iterations_per_second" and d["unit"] == "iterations/s"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["config"]["workload"] == "tsne_10k" and d["config"]["n"] == 10_000
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and "iterations" in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert 1 <= d["steps"] <= 750


def test_median_call_seconds_warms_once_then_takes_the_median():
    sys.path.insert(0, ROOT)
    import time

    import bench

    calls = []
    durations = iter([0.0, 0.03, 0.01, 0.02])  # the first (warm) call is not timed

    def call():
        calls.append(1)
        time.sleep(next(durations))

    secs = bench.median_call_seconds(call)
    assert len(calls) == 4
    assert 0.015 < secs < 0.05

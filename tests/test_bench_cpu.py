"""bench.py's reference arm on CPU (no GPU needed): the JSON line carries the
contract's keys, the reference arm measures the CPU port with the host's
threads, and ranks other than 0 print nothing."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def run_bench(*args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    r = subprocess.run([sys.executable, str(REPO / "bench.py"), *args], capture_output=True,
                       text=True, env=e, timeout=300, cwd=REPO)
    return r


def test_reference_arm_line():
    r = run_bench("--impl", "reference", "--steps", "1", "--warmup", "1",
                  "--ref-step-seconds", "0.5")
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["value"] > 0
    assert line["warmup"] >= 3  # the timing rules' minimum, whatever was asked
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert "simd" in cb and ("unavailable" in cb["simd"] or "not timed" in cb["simd"])
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_are_silent():
    r = run_bench("--impl", "reference", "--steps", "1", "--warmup", "1",
                  env={"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


def test_failing_rank_prints_a_json_error_line():
    # the B200 arm on a host without a usable GPU fails early: the failing
    # rank names itself and its phase on stdout, and exits non-zero
    r = run_bench("--steps", "1", "--warmup", "1", "--no-e2e", "--no-extra",
                  "--no-cpu-baseline", env={"CUDA_VISIBLE_DEVICES": "", "RANK": "3",
                                            "LOCAL_RANK": "0", "WORLD_SIZE": "1"})
    assert r.returncode != 0
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert lines, r.stdout[-2000:] + r.stderr[-2000:]
    err = json.loads(lines[-1])
    assert err["rank"] == 3 and err["where"] and err["error"] and err["impl"] == "b200"

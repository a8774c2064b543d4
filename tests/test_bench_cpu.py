"""bench.py's reference arm on CPU: the reference's CPU implementation of the path
(the oracle port) timed on a bounded sample, one JSON line with the driver's keys."""
from __future__ import annotations

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def _run(*args):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                       timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


def test_reference_arm_json_line():
    d = _run("--impl", "reference", "--steps", "1", "--warmup", "1")
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference" and d["unit"] == "Mtokens/s" and d["value"] > 0
    assert d["warmup"] >= 3  # the timing rules' minimum is enforced
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"] == "lowrank"


def test_reference_arm_headwise_workload():
    d = _run("--impl", "reference", "--workload", "headwise_hs32", "--steps", "1", "--warmup", "1")
    assert d["config"]["workload"] == "headwise_hs32" and d["value"] > 0

"""CPU: bench.py's reference arm (the oracle port of the decode sweep timed on
the host cores) prints one JSON line with the keys of the bench contract:
throughput, timing, the workload, the CPU baseline that describes the run, and
an end-to-end figure with no host-device copies.  About ten seconds."""
from __future__ import annotations

import json
import subprocess
import sys

from conftest import ROOT

CONTRACT_KEYS = ["metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                 "scaling", "vs_baseline", "dtype", "data", "config"]


def run_bench(*args: str) -> subprocess.CompletedProcess:
    return subprocess.run([sys.executable, "bench.py", *args], cwd=ROOT, capture_output=True, text=True,
                          timeout=300)


def test_reference_arm_prints_one_contract_line():
    r = run_bench("--impl", "reference", "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    for k in CONTRACT_KEYS:
        assert k in d, k
    assert d["impl"] == "reference"
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 0
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["higher_is_better"] is True
    assert isinstance(d["config"], dict) and "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_profiling_cases_are_listed():
    r = run_bench("--help")
    assert r.returncode == 0
    for case in ("decode-28", "prefill-32k", "gemm", "model-prefill", "tp-exchange"):
        assert case in r.stdout, case

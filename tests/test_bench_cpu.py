"""bench.py's reference arm on the CPU: it times the oracle restatement of the
reference's kernels on the host cores and prints the contract's JSON line
(impl, metric, value, unit, e2e with zero copy bytes, cpu_baseline); under a
multi-rank launch every rank but 0 exits 0 without output. Needs no GPU."""
from __future__ import annotations

import json
import os
import subprocess
import sys

from conftest import ROOT


def _run(extra_env=None, *args):
    env = dict(os.environ)
    env.update(extra_env or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", *args],
                          capture_output=True, text=True, cwd=ROOT, env=env, timeout=600)


def test_reference_arm_prints_contract_line():
    r = _run({"ONNXSHARP_THREADS": "4"}, "--workload", "gemm", "--warmup", "3", "--steps", "2")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "TFLOP/s" and d["value"] > 0
    assert d["higher_is_better"] is True and d["warmup"] >= 3
    assert d["config"]["workload"] and d["config"]["m"] == 2048
    assert d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert cb["reference_published"]["source"] == "bench.md:961-970"
    assert d["steps"] == 2


def test_reference_arm_other_ranks_are_silent():
    r = _run({"RANK": "1", "WORLD_SIZE": "2"}, "--workload", "gemm", "--warmup", "3", "--steps", "2")
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]

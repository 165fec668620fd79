"""The reference arm of bench.py on the host CPU (no GPU needed).

``bench.py --impl reference`` times the reference's contiguous decode (the
oracle restatement) on the host cores, prints one JSON line on rank 0 with the
same metric and config keys as the GPU arm, and exits 0 without output on the
other ranks.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys

from tests.conftest import ROOT

BENCH = str(ROOT / "bench.py")


def _run(*args: str, env: dict | None = None) -> subprocess.CompletedProcess:
    full_env = dict(os.environ)
    full_env.update(env or {})
    return subprocess.run([sys.executable, BENCH, "--impl", "reference", *args], cwd=ROOT,
                          env=full_env, capture_output=True, text=True, timeout=300)


def test_reference_arm_prints_one_contract_line():
    r = _run("--steps", "2", "--warmup", "1", "--batch", "4")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["value"] > 0 and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["warmup"] == 1 and d["n_gpus"] == 1
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "port" and cb["cores"] >= 1
    assert cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    r = _run("--gpus", "2", "--steps", "1", "--warmup", "1", "--batch", "4",
             env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_reference_arm_says_when_a_workload_has_no_cpu_arm():
    r = _run("--workload", "append", "--steps", "1", "--warmup", "1")
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d["impl"] == "reference" and "unavailable" in d

"""The benchmark's reference arm (CPU only): one JSON line with the contract's
keys on rank 0, nothing from other ranks."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(extra_env=None):
    env = dict(os.environ, **(extra_env or {}))
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], cwd=ROOT, env=env, capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    return [l for l in out.stdout.splitlines() if l.strip()]


def test_reference_arm_prints_one_contract_line():
    lines = _run()
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["value"] > 0 and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["warmup"] >= 3 and d["steps"] == 1
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert "workload" in d["config"]


def test_reference_arm_other_ranks_print_nothing():
    assert _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}) == []


def test_reference_arm_decode_workload_reports_tokens_per_second():
    env = dict(os.environ)
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", "step8b",
                          "--steps", "1", "--warmup", "3"], cwd=ROOT, env=env,
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads(out.stdout.strip().splitlines()[-1])
    assert d["impl"] == "reference" and d["unit"] == "tok/s" and d["value"] > 0
    assert d["warmup"] >= 3 and d["cpu_baseline"]["unit"] == "tok/s"
    assert d["e2e"]["h2d_bytes_per_step"] == 0


def test_reference_arm_prefill_workload_reports_prompt_tokens_per_second():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", "prefill8b",
                          "--steps", "1", "--warmup", "3"], cwd=ROOT, env=dict(os.environ),
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "tok/s" and d["value"] > 0
    assert d["config"]["prompt_tokens"] == 2048 and d["scaling"] == "strong"
    assert d["cpu_baseline"]["kind"] == "port" and "scaled to" in d["cpu_baseline"]["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}

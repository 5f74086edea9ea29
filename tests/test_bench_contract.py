"""The reference arm of bench.py, run on the host cores: one JSON line with the contract's keys.

`bench.py --impl reference` times the reference's op sequence (the oracle) on the CPU, so it
runs here without a GPU. Under torchrun only rank 0 works and prints; the other ranks exit 0.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
KEYS = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e")


def run_bench(*args, env=None, timeout=300):
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, capture_output=True, text=True,
                         timeout=timeout, env={**os.environ, **(env or {})})
    assert res.returncode == 0, res.stderr[-2000:]
    return [json.loads(line) for line in res.stdout.splitlines() if line.startswith("{")]


@pytest.mark.parametrize("workload", ["gpt2-xl", "operator"])
def test_reference_arm_prints_one_contract_line(workload):
    lines = run_bench("--impl", "reference", "--workload", workload, "--steps", "1", "--warmup", "0")
    assert len(lines) == 1
    d = lines[0]
    for key in KEYS:
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["metric"] == "candidate seqs scored+selected/sec" and d["unit"] == "candidates/s"
    assert d["higher_is_better"] is True and d["scaling"] == "weak" and d["n_gpus"] == 1
    assert d["steps"] == 1 and d["warmup"] == 0
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_exit_quietly():
    lines = run_bench("--impl", "reference", "--steps", "1", "--warmup", "0", env={"RANK": "1", "WORLD_SIZE": "2"},
                      timeout=120)
    assert lines == []

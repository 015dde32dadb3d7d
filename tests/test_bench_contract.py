"""bench.py's reference arm, run on the CPU: one JSON line with the contract's keys, the reference's CPU
path timed on a bounded sample (the oracle port), and no output from ranks other than 0."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_bench(*args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    res = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                         timeout=600, cwd=ROOT, env=env)
    assert res.returncode == 0, res.stderr[-2000:]
    return [json.loads(line) for line in res.stdout.splitlines() if line.startswith("{")]


@pytest.mark.parametrize("workload,unit", [("cfg1", "TFLOP/s"), ("gemv1", "GB/s")])
def test_reference_arm_prints_one_contract_line(workload, unit):
    lines = run_bench("--impl", "reference", "--workload", workload, "--steps", "1", "--warmup", "0")
    assert len(lines) == 1
    d = lines[0]
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == unit and d["value"] > 0 and d["n_gpus"] == 1
    assert d["higher_is_better"] is True and d["steps"] == 1 and d["warmup"] == 0
    assert d["config"]["workload"].startswith(workload)
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["unit"] == unit
    assert "rows" in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_runs_on_rank_zero_only():
    assert run_bench("--impl", "reference", "--steps", "1", "--warmup", "0", env_extra={"RANK": "1"}) == []

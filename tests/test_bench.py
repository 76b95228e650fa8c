"""bench.py's reference arm (no GPU needed): one JSON line with the fields the
benchmark contract names, for both workloads, and the N > 1 rule that only
rank 0 prints it."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT

CONTRACT = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
            "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e", "impl"}


def run_bench(*args, env=None):
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                          timeout=600, env=dict(os.environ, **(env or {})))
    assert proc.returncode == 0, proc.stderr[-2000:]
    return [json.loads(line) for line in proc.stdout.splitlines() if line.startswith("{")]


@pytest.mark.parametrize("workload", ["c2", "stdp"])
def test_reference_arm_line(workload):
    lines = run_bench("--impl", "reference", "--workload", workload, "--steps", "1", "--warmup", "3")
    assert len(lines) == 1
    line = lines[0]
    assert CONTRACT <= set(line), CONTRACT - set(line)
    assert line["impl"] == "reference" and line["metric"] == "synaptic events/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] == 1
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["config"]["workload"]


def test_reference_arm_prints_on_rank_zero_only():
    assert run_bench("--impl", "reference", "--steps", "1", "--warmup", "3", env={"RANK": "1", "WORLD_SIZE": "2"}) == []

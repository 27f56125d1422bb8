# SPDX-License-Identifier: MIT
"""bench.py's command-line contract on a machine without a GPU: the reference arm prints
one JSON line with the keys the driver reads; ranks other than 0 print nothing and exit
0; the GPU arm fails loudly instead of measuring anything on the CPU."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def _run(args, env_extra=None, timeout=600):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=env, capture_output=True,
                          text=True, timeout=timeout)


def _json_lines(out):
    return [json.loads(l) for l in out.splitlines() if l.startswith("{")]


def test_reference_arm_prints_one_contract_line():
    p = _run(["--impl", "reference", "--workload", "cfg1", "--steps", "2", "--warmup", "1"])
    assert p.returncode == 0, p.stderr[-2000:]
    lines = _json_lines(p.stdout)
    assert len(lines) == 1, p.stdout
    d = lines[0]
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["steps"] == 2 and d["n_gpus"] == 1
    assert d["warmup"] == 3  # warm-up is raised to the contract's minimum of three steps
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert "workload" in d["config"]


def test_reference_arm_other_ranks_exit_quietly():
    p = _run(["--impl", "reference", "--workload", "cfg1", "--steps", "1", "--warmup", "1"],
             {"RANK": "1", "WORLD_SIZE": "2"})
    assert p.returncode == 0, p.stderr[-2000:]
    assert _json_lines(p.stdout) == []


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the behaviour without a GPU")
def test_gpu_arm_fails_without_a_gpu():
    p = _run(["--workload", "cfg1", "--steps", "1", "--warmup", "1", "--no-e2e", "--no-cpu-baseline"], timeout=300)
    assert p.returncode != 0
    assert _json_lines(p.stdout) == []

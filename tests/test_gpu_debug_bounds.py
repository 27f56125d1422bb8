# SPDX-License-Identifier: MIT
"""The bounds-checked build (librmsnorm_b200_debug.so: every load, store and copy of every
kernel checks its bytes against the ranges the API call registered, and a failed check is
reported and skipped, never trapped) runs the odd-shape matrix of tests/debug_bounds_matrix.py
-- unaligned-free odd widths, ragged row counts, per-head rows, split rows in both exchange
modes and chunk counts, the generic kernels, TMEM and register backwards, the no-allocation
entry point, LayerNorm -- with zero failed checks and parity with the oracle; and the
checker catches a planted range error (an output registered one row short)."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device"),
]

HERE = Path(__file__).resolve().parent
DEBUG_LIB = HERE.parent / "rmsnorm-h100_b200" / "rmsnorm" / "lib" / "librmsnorm_b200_debug.so"


def test_odd_shape_matrix_is_clean_under_the_bounds_checked_build():
    assert DEBUG_LIB.exists(), "librmsnorm_b200_debug.so is missing: run __graft_entry__.build()"
    env = dict(os.environ, RMSNORM_B200_LIBRARY=str(DEBUG_LIB))
    r = subprocess.run([sys.executable, str(HERE / "debug_bounds_matrix.py")], env=env, capture_output=True,
                       text=True, timeout=1200)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert lines, f"no summary (exit {r.returncode}):\n{r.stdout[-3000:]}\n{r.stderr[-3000:]}"
    summary = json.loads(lines[-1])
    assert summary["cases"] >= 80, summary["cases"]
    assert not summary["failures"], json.dumps(summary["failures"][:5], indent=1)
    assert summary["device_status"][0] == 0, summary["device_status"]
    clip = summary["clip"]
    assert clip["violations"] > 0 and clip["site"] == 2, clip  # vector stores to the clipped row
    assert clip["in_clipped_row"] and clip["last_row_untouched"] and clip["rest_ok"], clip
    assert r.returncode == 0, r.stderr[-2000:]

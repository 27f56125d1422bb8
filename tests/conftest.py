# SPDX-License-Identifier: MIT
"""Shared pytest configuration: the `gpu` marker, import paths, golden-vector loader."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "rmsnorm-h100_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"
_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name: str) -> dict:
    """Tensors (and 'meta') from tests/golden/<name>.npz, in their original dtypes."""
    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(z["__meta__"]))
    out = {"meta": meta}
    for k, code in meta["dtypes"].items():
        a = torch.from_numpy(z[k].copy())
        out[k] = a.view(_DT[code]) if code in ("f16", "bf16") else a
    return out


@pytest.fixture
def golden():
    return load_golden


def cuda_available() -> bool:
    return torch.cuda.is_available()

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


@pytest.fixture(autouse=True)
def _nan_poisoned_device_memory(request):
    """Before every GPU test, the caching allocator's free device memory is filled with 0xFF
    bytes -- NaN as fp16, bf16 and fp32 -- so an output element a kernel fails to write
    reads NaN instead of a value an earlier test left in the same block. One large segment
    (a quarter of the free memory, at most 16 GiB) serves the tensors the API allocates;
    a few small ones serve allocations under 1 MiB, which the allocator keeps apart."""
    if request.node.get_closest_marker("gpu") is None or not torch.cuda.is_available():
        yield
        return
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    free, _ = torch.cuda.mem_get_info()
    big = torch.empty(min(free // 4, 16 << 30), dtype=torch.uint8, device="cuda")
    big.fill_(0xFF)
    small = [torch.empty((1 << 20) - 512, dtype=torch.uint8, device="cuda") for _ in range(16)]
    for t in small:
        t.fill_(0xFF)
    torch.cuda.synchronize()
    del big, small
    yield

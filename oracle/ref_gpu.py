# SPDX-License-Identifier: MIT
"""GPU COMPARATOR -- benchmark infrastructure only; the product never loads it.

Loads the reference's own CUDA extension (its Hopper kernels recompiled for sm_100a by
oracle/build_ref.py into oracle/_ref/) and calls it the way the reference's Python layer
does for each BASELINE workload (rmsnorm/rmsnorm.py:274-528 of Int21-AI/RMSNorm-H100):

  cfg1            fwd_fast(x, w, eps)                          (py:323-348)
  cfg2            fwd_(x, w, b, res, out, ro_fp32, None, 1, eps) (bias -> general path, py:350-387)
  cfg3            bwd_fast(x, w, dout, rstd)                   (py:420-441)
  cfg4 forward    fwd_(x, w, b, None, out, None, rstd, 32, eps) (per-head, store_rstd under autograd)
  cfg4 backward   bwd_(x, w, dout, rstd, dx, dw, db, None, None, 32, 1e-6)
  cfg5 forward    fwd_(x, w, None, None, out, None, rstd, 1, eps) (store_rstd under autograd)
  cfg5 backward   bwd_fast(x, w, dout, rstd)

The extension is located relative to this file (the reference checkout is not needed at
run time). Used by `bench.py --impl refgpu`.
"""

from __future__ import annotations

import importlib.machinery
import importlib.util
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
NAME = "rmsnorm_ref_ext"


def load():
    for suf in importlib.machinery.EXTENSION_SUFFIXES:
        path = HERE / "_ref" / f"{NAME}{suf}"
        if path.exists():
            break
    else:
        raise FileNotFoundError("reference extension not built (oracle/build_ref.py)")
    spec = importlib.util.spec_from_file_location(NAME, str(path))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def make_step(ext, kind, t, heads=1, ro_dtype=None, store_rstd=False, has_bias=False):
    """Returns a zero-argument callable running one step of the reference's path on the
    device tensors `t` (keys as in bench.py: x, w, b, res, dy, rstd)."""
    x, w = t["x"], t["w"]
    if kind == "fwd":
        b, res = t.get("b"), t.get("res")
        if b is None and res is None and not store_rstd and heads == 1:
            return lambda: ext.fwd_fast(x, w, 1e-6)
        out = torch.empty_like(x)
        ro = torch.empty(x.shape, dtype=ro_dtype, device=x.device) if (res is not None and ro_dtype) else None
        rstd = torch.empty(x.shape[0], dtype=torch.float32, device=x.device) if store_rstd else None
        return lambda: ext.fwd_(x, w, b, res, out, ro, rstd, heads, 1e-6)
    dy, rstd = t["dy"], t["rstd"]
    if heads == 1 and not has_bias:
        return lambda: ext.bwd_fast(x, w, dy, rstd)
    dx = torch.empty_like(x)
    dw = torch.empty(w.shape, dtype=torch.float32, device=x.device)
    db = torch.empty(w.shape, dtype=torch.float32, device=x.device) if has_bias else None
    return lambda: ext.bwd_(x, w, dy, rstd, dx, dw, db, None, None, heads, 1e-6)

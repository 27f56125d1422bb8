# SPDX-License-Identifier: MIT
"""ORACLE build recipe -- test infrastructure only.

Compiles oracle/rmsnorm_ref.c (the C restatement of the reference's CPU loops) into
oracle/_build/liboracle_c.so with gcc, and exposes a ctypes wrapper. Run by
`__graft_entry__.build()`; tests build it on demand if it is missing.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
SRC = HERE / "rmsnorm_ref.c"
OUT = HERE / "_build" / "liboracle_c.so"


def build(force: bool = False) -> Path:
    if OUT.exists() and not force and OUT.stat().st_mtime >= SRC.stat().st_mtime:
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    cmd = ["gcc", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-o", str(OUT), str(SRC), "-lm"]
    subprocess.run(cmd, check=True)
    return OUT


_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        _LIB = ctypes.CDLL(str(build()))
        p = ctypes.c_void_p
        i64 = ctypes.c_int64
        _LIB.oracle_fwd.argtypes = [p, p, p, p, i64, i64, i64, ctypes.c_float, p, p, p]
        _LIB.oracle_bwd.argtypes = [p, p, p, p, p, i64, i64, i64, p, p, p]
    return _LIB


def _f32(t):
    return None if t is None else t.detach().cpu().float().contiguous()


def _p(t):
    return None if t is None else t.data_ptr()


def fwd(x, weight=None, bias=None, residual=None, eps=1e-6, heads=1):
    """Returns fp32 (y, h, rstd) for a [rows, n] problem."""
    xf, rf, wf, bf = _f32(x), _f32(residual), _f32(weight), _f32(bias)
    rows, n = xf.shape
    y = torch.empty_like(xf)
    h = torch.empty_like(xf)
    rstd = torch.empty(rows, dtype=torch.float32)
    lib().oracle_fwd(_p(xf), _p(rf), _p(wf), _p(bf), rows, n, heads, eps, _p(y), _p(h), _p(rstd))
    return y, h, rstd


def bwd(x, weight, dout, rstd, dresidual_out=None, has_bias=False, heads=1):
    """Returns fp32 (dx, dweight [heads*n] or None, dbias [heads*n] or None)."""
    xf, wf, df, rf, af = _f32(x), _f32(weight), _f32(dout), _f32(rstd), _f32(dresidual_out)
    rows, n = xf.shape
    dx = torch.empty_like(xf)
    dw = torch.zeros(heads * n, dtype=torch.float32) if weight is not None else None
    db = torch.zeros(heads * n, dtype=torch.float32) if has_bias else None
    lib().oracle_bwd(_p(xf), _p(wf), _p(df), _p(af), _p(rf), rows, n, heads, _p(dx), _p(dw), _p(db))
    return dx, dw, db


if __name__ == "__main__":
    print(build(force=True))

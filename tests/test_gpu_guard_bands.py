# SPDX-License-Identifier: MIT
"""Out-of-bounds and unwritten-element checks without a device sanitizer.

Every tensor handed to the C ABI here is a view into a larger NaN-filled buffer, with
GUARD elements of guard band on each side (16-byte aligned, so the streaming kernels
still take their vectorised paths):
  * outputs start as NaN: an element the kernel leaves unwritten fails the parity check;
  * output guard bands must still be NaN afterwards: a write past either end is caught;
  * input guard bands are NaN: a read past either end poisons a result, which then
    fails the parity check.
The cases cover every plan the library picks (row mode, pipelined rows, segments,
per-head column mode, rows split over a cluster or a cooperative grid, chunked slices,
the generic kernels, LayerNorm) and compare against the CPU oracle."""

from __future__ import annotations

import math

import pytest
import torch

from oracle import rmsnorm_oracle as oracle

from rmsnorm import _lib

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device"),
]

DEV = torch.device("cuda")
F16, BF16, F32 = torch.float16, torch.bfloat16, torch.float32
GUARD = 4096  # elements on each side (8 KB or more: 16-byte aligned for every dtype)


class Guarded:
    """A tensor of `shape` at offset GUARD inside a NaN-filled buffer."""

    def __init__(self, shape, dtype, value=None):
        self.n = math.prod(shape)
        self.buf = torch.full((self.n + 2 * GUARD,), float("nan"), dtype=dtype, device=DEV)
        self.t = self.buf[GUARD:GUARD + self.n].view(shape)
        if value is not None:
            self.t.copy_(value)

    def guards_intact(self):
        return bool(torch.isnan(self.buf[:GUARD]).all()) and bool(torch.isnan(self.buf[GUARD + self.n:]).all())


def _env(monkeypatch, env):
    for k, v in (env or {}).items():
        monkeypatch.setenv(k, v)


FWD_CASES = [
    # rows, n, dtype, residual dtype, residual_out dtype, bias, heads, env, expected plan
    (37, 4096, BF16, BF16, F32, True, 1, None, "fwd_stream mode=row"),
    (1000, 1024, F16, None, None, False, 1, None, "fwd_stream mode=row"),
    (9, 24, F32, F32, F32, True, 1, None, "mode=seg"),
    (37 * 32, 128, F16, None, None, True, 32, None, "cols=1"),
    (21 * 32, 256, BF16, None, None, True, 32, None, "cols=2"),
    (3, 262144, BF16, None, None, False, 1, None, "fwd_stream"),
    (5, 262144, F32, F32, F32, True, 1, None, "fwd_stream"),
    (40, 65536, BF16, BF16, F32, True, 1, {"RMSNORM_B200_XMODE": "1", "RMSNORM_B200_FORCE_CLUSTER": "4"},
     "x=global"),
    (9, 65536, F32, F32, F32, False, 1, {"RMSNORM_B200_FORCE_CLUSTER": "8", "RMSNORM_B200_FORCE_K": "2"}, "K=2"),
    (6, 100, BF16, BF16, F32, True, 1, None, "fwd_generic"),
]


@pytest.mark.parametrize("rows,n,dt,rdt,rodt,bias,heads,env,expect", FWD_CASES)
def test_fwd_guard_bands(monkeypatch, rows, n, dt, rdt, rodt, bias, heads, env, expect):
    _env(monkeypatch, env)
    aff = (heads, n) if heads > 1 else (n,)
    xv = oracle.gen((rows, n), dt, 1)
    rv = oracle.gen((rows, n), rdt, 2) if rdt is not None else None
    wv = oracle.gen(aff, F32, 3, "weight")
    bv = oracle.gen(aff, F32, 4, "bias") if bias else None
    x = Guarded((rows, n), dt, xv)
    res = Guarded((rows, n), rdt, rv) if rdt is not None else None
    w = Guarded(aff, F32, wv)
    b = Guarded(aff, F32, bv) if bias else None
    out = Guarded((rows, n), dt)
    ro = Guarded((rows, n), rodt) if rodt is not None else None
    rstd = Guarded((rows,), F32)
    _lib.fwd(x.t, res.t if res else None, w.t, heads, b.t if b else None, heads, out.t, ro.t if ro else None,
             rstd.t, heads, 1e-6)
    torch.cuda.synchronize()
    plan = _lib.last_plan()
    assert expect in plan, plan
    xs = xv.view(rows // heads, heads, n) if heads > 1 else xv
    rs = rv.view(xs.shape) if rv is not None else None
    _, o_ro, o_rstd, y = oracle.fwd(xs, wv, bv, rs, residual_dtype=rodt)
    oracle.check_close(out.t.view(xs.shape), y, dt, f"out [{plan}]")
    assert torch.allclose(rstd.t.cpu().view(o_rstd.shape), o_rstd, rtol=1e-5, atol=0), plan
    if ro is not None:
        assert torch.equal(ro.t.cpu().view(o_ro.shape), o_ro), plan
    for g in (out, ro, rstd):
        if g is not None:
            assert g.guards_intact(), f"write outside an output [{plan}]"
    assert _lib.device_status(DEV) == (0, 0)


BWD_CASES = [
    # rows, n, x dtype, dout dtype, dresidual_out, dbias, heads, env, expected plan
    (37, 4096, BF16, BF16, False, True, 1, None, "bwd_stream"),
    (300, 2048, F32, BF16, True, True, 1, None, "bwd_stream"),
    (9, 24, F16, F16, False, True, 1, None, "mode=seg"),
    (37 * 32, 128, F16, F16, False, True, 32, None, "cols=1"),
    (3, 262144, BF16, BF16, False, False, 1, None, "bwd_stream"),
    (4, 262144, F32, F32, False, False, 1, None, "bwd_stream"),
    (4, 262144, F32, F32, False, True, 1, None, "bwd_generic"),  # dbias rows wider than 16 CTAs hold
    (70, 65536, BF16, BF16, False, True, 1, {"RMSNORM_B200_XMODE": "1", "RMSNORM_B200_FORCE_CLUSTER": "8"},
     "x=global"),
    (37, 16384, F32, BF16, False, True, 1, None, "acc=tmem"),  # dweight / dbias sums in TMEM
    (301, 12288, BF16, BF16, True, True, 1, None, "acc=tmem"),  # last vector of the slice ragged
    (37, 16384, F32, BF16, False, True, 1, {"RMSNORM_B200_TMEM_ACC": "0"}, "P=2"),
    (6, 100, BF16, BF16, True, True, 1, None, "bwd_generic"),
]


@pytest.mark.parametrize("rows,n,dt,gdt,dro,dbias,heads,env,expect", BWD_CASES)
def test_bwd_guard_bands(monkeypatch, rows, n, dt, gdt, dro, dbias, heads, env, expect):
    _env(monkeypatch, env)
    aff = (heads, n) if heads > 1 else (n,)
    xv = oracle.gen((rows, n), dt, 11)
    gv = oracle.gen((rows, n), gdt, 12)
    wv = oracle.gen(aff, F32, 13, "weight")
    xs = xv.view(rows // heads, heads, n) if heads > 1 else xv
    _, _, rv, _ = oracle.fwd(xs, wv)
    dv = oracle.gen((rows, n), dt, 14) if dro else None
    x = Guarded((rows, n), dt, xv)
    g = Guarded((rows, n), gdt, gv)
    w = Guarded(aff, F32, wv)
    rstd = Guarded((rows,), F32, rv.reshape(-1))
    d = Guarded((rows, n), dt, dv) if dro else None
    dx = Guarded((rows, n), gdt if dt == F32 and gdt != F32 else dt)
    dres = Guarded((rows, n), dx.t.dtype) if dro else None
    dw = Guarded(aff, F32)
    db = Guarded(aff, F32) if dbias else None
    a = _lib.bwd_args(x.t, g.t, rstd.t, w.t, heads, d.t if d else None, dx.t, dres.t if dres else None, dw.t,
                      db.t if db else None, heads, heads)
    nbytes = _lib.bwd_workspace_bytes(a, DEV)
    ws = Guarded((max(nbytes // 4, 4),), F32)  # workspace: NaN inside too (partials must all be written)
    _lib.bwd(a, DEV, ws.t.view(torch.uint8))
    torch.cuda.synchronize()
    plan = _lib.last_plan()
    assert expect in plan, plan
    gs = gv.view(xs.shape)
    o_dx, o_dw, o_db, s_dw, s_db = oracle.bwd(xs, wv, gs, rv, dresidual_out=dv.view(xs.shape) if dro else None,
                                              has_bias=dbias)
    oracle.check_close(dx.t.view(xs.shape), o_dx, dx.t.dtype if dx.t.dtype != F32 else dt, f"dx [{plan}]",
                       rtol=oracle.y_tolerance(gdt) if dt == F32 else None)
    if dres is not None:
        assert torch.equal(dres.t, dx.t), plan
    oracle.check_reduction(dw.t, o_dw, s_dw, f"dweight [{plan}]")
    if db is not None:
        oracle.check_reduction(db.t, o_db, s_db, f"dbias [{plan}]")
    for t in (dx, dres, dw, db, ws):
        if t is not None:
            assert t.guards_intact(), f"write outside an output or the workspace [{plan}]"
    assert _lib.device_status(DEV) == (0, 0)


@pytest.mark.parametrize("rows,n,dt,bias,expect", [(1000, 4096, BF16, True, "ln_stream mode=row"),
                                                   (70, 128, F32, True, "ln_stream mode=seg"),
                                                   (17, 65536, BF16, False, "ln_generic")])
def test_layernorm_guard_bands(rows, n, dt, bias, expect):
    xv = oracle.gen((rows, n), dt, 21)
    wv = oracle.gen((n,), F32, 22, "weight")
    bv = oracle.gen((n,), F32, 23, "bias") if bias else None
    x = Guarded((rows, n), dt, xv)
    w = Guarded((n,), F32, wv)
    b = Guarded((n,), F32, bv) if bias else None
    out = Guarded((rows, n), dt)
    mean = Guarded((rows,), F32)
    rstd = Guarded((rows,), F32)
    _lib.layernorm_fwd(x.t, n, w.t, b.t if b else None, out.t, mean.t, rstd.t, 1e-6)
    torch.cuda.synchronize()
    plan = _lib.last_plan()
    assert expect in plan, plan
    _, o_rstd, o_mean, y = oracle.layernorm_fwd(xv, wv, bv, 1e-6)
    oracle.check_close(out.t, y, dt, f"ln out [{plan}]")
    assert torch.isfinite(mean.t).all() and torch.allclose(rstd.t.cpu(), o_rstd, rtol=1e-5, atol=0), plan
    for t in (out, mean, rstd):
        assert t.guards_intact(), f"write outside an output [{plan}]"

# SPDX-License-Identifier: MIT
"""Test helper: fp32 PyTorch reference of the same math, evaluated on the GPU in row
chunks, for full-size checks where the CPU oracle would take minutes. Everything else is
checked against the CPU oracle (oracle/rmsnorm_oracle.py); both are test infrastructure."""

from __future__ import annotations

import torch


@torch.no_grad()
def fwd_max_err(x, weight, bias, residual, out, ro, rstd, eps, rtol, chunk=1024, heads=1):
    """Max over rows of |out - ref| / (rtol * (rms(ref) + |ref|)) (<= 1 passes), plus exact
    residual_out and rstd checks, on 2-D [rows, n] views; per-head when heads > 1."""
    worst = 0.0
    n = x.shape[-1]
    rows = x.shape[0]
    rms_all = None
    w = weight.float() if weight is not None else None
    b = bias.float() if bias is not None else None
    for s in range(0, rows, chunk):
        e = min(rows, s + chunk)
        h = x[s:e].float()
        if residual is not None:
            h = h + residual[s:e].float()
        r = torch.rsqrt(h.square().mean(-1, keepdim=True) + eps)
        y = h * r
        if heads > 1:
            hidx = torch.arange(s, e, device=x.device) % heads
            if w is not None:
                y = y * (w[hidx] if w.dim() == 2 else w)
            if b is not None:
                y = y + (b[hidx] if b.dim() == 2 else b)
        else:
            if w is not None:
                y = y * w
            if b is not None:
                y = y + b
        if rms_all is None:
            rms_all = y.square().mean().sqrt().item()
        err = (out[s:e].float() - y).abs() / (rtol * (rms_all + y.abs()))
        worst = max(worst, err.max().item())
        if ro is not None:
            assert torch.equal(ro[s:e], h.to(ro.dtype)), f"residual_out rows {s}:{e} differ"
        if rstd is not None:
            rel = ((rstd[s:e].float() - r.squeeze(-1)).abs() / r.squeeze(-1)).max().item()
            assert rel <= 1e-5, f"rstd rows {s}:{e} rel err {rel}"
    return worst


@torch.no_grad()
def bwd_check(x, weight, dout, rstd, dx, dw, rtol, chunk=512, heads=1):
    """Returns (max normalised dx error, max normalised dweight error) against an fp32
    (dx) / fp64-accumulated (dweight) reference; dweight bound is 1e-3 * sum|dy * xhat|."""
    rows, n = x.shape
    worst = 0.0
    acc = torch.zeros(weight.shape if weight is not None else (n,), dtype=torch.float64, device=x.device)
    acc_abs = torch.zeros_like(acc)
    w = weight.float() if weight is not None else None
    rms_all = None
    for s in range(0, rows, chunk):
        e = min(rows, s + chunk)
        r = rstd[s:e].float().unsqueeze(-1)
        xh = x[s:e].float() * r
        g = dout[s:e].float()
        if w is not None and heads > 1:
            ww = w[torch.arange(s, e, device=x.device) % heads]
        else:
            ww = w
        wdy = g * ww if ww is not None else g
        c = (xh * wdy).mean(-1, keepdim=True)
        ref = (wdy - xh * c) * r
        if rms_all is None:
            rms_all = ref.square().mean().sqrt().item()
        err = (dx[s:e].float() - ref).abs() / (rtol * (rms_all + ref.abs()))
        worst = max(worst, err.max().item())
        t = (g * xh).double()
        if heads > 1:
            acc.index_add_(0, torch.arange(s, e, device=x.device) % heads, t)
            acc_abs.index_add_(0, torch.arange(s, e, device=x.device) % heads, t.abs())
        else:
            acc += t.sum(0)
            acc_abs += t.abs().sum(0)
    dw_err = 0.0
    if dw is not None:
        dw_err = ((dw.double() - acc).abs() / (1e-3 * acc_abs + 1e-6)).max().item()
    return worst, dw_err

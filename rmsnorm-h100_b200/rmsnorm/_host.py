# SPDX-License-Identifier: MIT
"""Host-tensor semantics of the reference package, in plain PyTorch.

These functions restate the reference's fp32 math for tensors that live on the host
(rmsnorm/rmsnorm.py:230-271 `rmsnorm_ref` / `_fallback_fwd`, :390-399 `rmsnorm_bwd_ref`,
:443-468 the backward fallback, :651-686 LayerNorm helpers). `rmsnorm.rmsnorm*` only
calls them for tensors that are not on a CUDA device; CUDA tensors always go to the
native library, which fails loudly if it is missing.
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor


def sum_to_affine_shape(values: Tensor, affine_shape: torch.Size) -> Tensor:
    """Sums the leading dimensions away so `values` takes the affine parameter's shape
    (rmsnorm/rmsnorm.py:196-204)."""
    extra = values.dim() - len(affine_shape)
    if extra < 0:
        raise ValueError(
            f"affine shape {tuple(affine_shape)} cannot be larger than input shape {tuple(values.shape)}"
        )
    return values if extra == 0 else values.sum(dim=tuple(range(extra)))


def _normalise(x: Tensor, residual: Optional[Tensor], eps: float):
    h = x.float()
    if residual is not None:
        h = h + residual.float()
    rstd = torch.rsqrt(h.square().mean(dim=-1, keepdim=True) + eps)
    return h, rstd


def _affine(y: Tensor, weight: Optional[Tensor], bias: Optional[Tensor]) -> Tensor:
    if weight is not None:
        y = y * weight.float()
    if bias is not None:
        y = y + bias.float()
    return y


def rmsnorm_ref(x: Tensor, w: Optional[Tensor] = None, bias=None, residual=None, eps=1e-6):
    """fp32 reference forward (rmsnorm/rmsnorm.py:230-243): returns out, or
    (out, x + residual in residual.dtype) when a residual is given."""
    h, rstd = _normalise(x, residual, eps)
    out = _affine(h * rstd, w, bias).to(x.dtype)
    if residual is None:
        return out
    return out, h.to(residual.dtype)


def fallback_fwd(x, weight, bias, residual, out_dtype, residual_dtype, eps, store_rstd):
    """(out, residual_out, rstd) for host tensors (rmsnorm/rmsnorm.py:246-271)."""
    h, rstd = _normalise(x, residual, eps)
    out = _affine(h * rstd, weight, bias).to(out_dtype)
    rstd_out = rstd.squeeze(-1).contiguous() if store_rstd else None
    if residual is None:
        residual_out = x if residual_dtype in (None, x.dtype) else x.to(residual_dtype)
    else:
        residual_out = h.to(residual_dtype or residual.dtype)
    return out, residual_out, rstd_out


def rmsnorm_bwd_ref(x, w, dout, rstd, eps=1e-6):
    """fp32 reference backward (rmsnorm/rmsnorm.py:390-399): (dx in x.dtype, dweight in
    w.dtype or None). `eps` is unused, as in the reference."""
    r = rstd.unsqueeze(-1)
    xhat = x.float() * r
    g = dout.float()
    wdy = g * w.float() if w is not None else g
    c = (xhat * wdy).mean(dim=-1, keepdim=True)
    dx = (wdy - xhat * c) * r
    if w is None:
        return dx.to(x.dtype), None
    return dx.to(x.dtype), sum_to_affine_shape(g * xhat, w.shape).to(w.dtype)


def fallback_bwd(x, weight, dout, rstd, dresidual_out, has_bias, has_residual, bias):
    """(dx, dweight, dbias, dresidual) for host tensors (rmsnorm/rmsnorm.py:450-468)."""
    dx, dw = rmsnorm_bwd_ref(x, weight, dout, rstd)
    if dresidual_out is not None:
        dx = (dx.float() + dresidual_out.float()).to(x.dtype)
    db = None
    if has_bias:
        if bias is not None:
            db_dtype, db_shape = bias.dtype, bias.shape
        elif weight is not None:
            db_dtype, db_shape = weight.dtype, weight.shape
        else:
            db_dtype, db_shape = x.dtype, torch.Size((x.shape[-1],))
        db = sum_to_affine_shape(dout.float(), db_shape).to(db_dtype)
    return dx, dw, db, (dx if has_residual else None)


def layernorm_ref(x: Tensor, w: Tensor, eps: float = 1e-6) -> Tensor:
    return torch.nn.functional.layer_norm(x.float(), w.shape, w.float(), None, eps).to(x.dtype)


def layernorm_fwd(x, weight, bias=None, eps=1e-6, return_rstd=False, return_mean=False):
    """LayerNorm forward with optional rstd / mean outputs (rmsnorm/rmsnorm.py:655-676)."""
    xf = x.float()
    out = torch.nn.functional.layer_norm(
        xf, weight.shape, weight.float(), bias.float() if bias is not None else None, eps
    ).to(x.dtype)
    mean = xf.mean(dim=-1) if (return_rstd or return_mean) else None
    rstd = None
    if return_rstd:
        var = (xf - mean.unsqueeze(-1)).square().mean(dim=-1)
        rstd = torch.rsqrt(var + eps)
    if return_rstd and return_mean:
        return out, rstd, mean
    if return_rstd:
        return out, rstd
    if return_mean:
        return out, mean
    return out


def layernorm_rstd_ref(x: Tensor, eps: float = 1e-6) -> Tensor:
    xf = x.float()
    var = (xf - xf.mean(dim=-1, keepdim=True)).square().mean(dim=-1)
    return torch.rsqrt(var + eps)


def layernorm_mean_ref(x: Tensor) -> Tensor:
    return x.float().mean(dim=-1)

# SPDX-License-Identifier: MIT
"""torch.library custom ops so that `torch.compile` keeps the native kernels.

The reference bypassed its extension while tracing and ran PyTorch ops instead
(rmsnorm/rmsnorm.py:611). Here `rmsnorm()` under compilation calls two opaque custom ops
(`rmsnorm_b200::fwd`, `rmsnorm_b200::bwd`) with fake-tensor shape functions and an
autograd formula equivalent to RMSNormFunction (rmsnorm/rmsnorm.py:531-595).
Outputs that the eager API aliases (residual_out is x; dresidual is dx) are returned as
empty placeholders by the ops and re-aliased by the Python wrapper, since custom ops may
not return views of their inputs or of each other.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor

# The submodule, not the package attribute `rmsnorm` (the package re-exports the function
# of that name, which shadows the submodule).
import importlib

_api = importlib.import_module(__package__ + ".rmsnorm")

_EMPTY = (0,)


def _ro_dtype(x: Tensor, residual: Optional[Tensor], residual_dtype: Optional[torch.dtype]):
    if residual is not None:
        return residual_dtype or residual.dtype
    if residual_dtype is not None and residual_dtype != x.dtype:
        return residual_dtype
    return None


@torch.library.custom_op("rmsnorm_b200::fwd", mutates_args=(), device_types="cuda")
def fwd_op(
    x: Tensor,
    weight: Optional[Tensor],
    bias: Optional[Tensor],
    residual: Optional[Tensor],
    out_dtype: torch.dtype,
    residual_dtype: Optional[torch.dtype],
    eps: float,
    store_rstd: bool,
) -> Tuple[Tensor, Tensor, Tensor]:
    out, ro, rstd = _api.rmsnorm_fwd(x, weight, bias, residual, out_dtype, residual_dtype, eps, store_rstd)
    if _ro_dtype(x, residual, residual_dtype) is None:
        ro = x.new_empty(_EMPTY)
    if rstd is None:
        rstd = x.new_empty(_EMPTY, dtype=torch.float32)
    return out, ro, rstd


@fwd_op.register_fake
def _(x, weight, bias, residual, out_dtype, residual_dtype, eps, store_rstd):
    out = x.new_empty(x.shape, dtype=out_dtype)
    rdt = _ro_dtype(x, residual, residual_dtype)
    ro = x.new_empty(x.shape, dtype=rdt) if rdt is not None else x.new_empty(_EMPTY)
    rstd = x.new_empty(x.shape[:-1], dtype=torch.float32) if store_rstd else x.new_empty(_EMPTY, dtype=torch.float32)
    return out, ro, rstd


@torch.library.custom_op("rmsnorm_b200::bwd", mutates_args=(), device_types="cuda")
def bwd_op(
    x: Tensor,
    weight: Optional[Tensor],
    dout: Tensor,
    rstd: Tensor,
    dresidual_out: Optional[Tensor],
    bias: Optional[Tensor],
    has_bias: bool,
    has_residual: bool,
    dx_dtype: torch.dtype,
    dresidual_dtype: Optional[torch.dtype],
) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    h = _api._head_count(weight, bias, x.shape)
    dx, dw, db, dres = _api._bwd_cuda(
        x, weight, dout, rstd, dresidual_out, has_bias, has_residual, bias, h,
        dx_dtype=dx_dtype, dresidual_dtype=dresidual_dtype,
    )
    def empty():  # a fresh placeholder each time: returns may not alias one another
        return x.new_empty(_EMPTY, dtype=torch.float32)

    return (
        dx,
        dw if dw is not None else empty(),
        db if db is not None else empty(),
        dres if (dres is not None and dres is not dx) else empty(),
    )


@bwd_op.register_fake
def _(x, weight, dout, rstd, dresidual_out, bias, has_bias, has_residual, dx_dtype, dresidual_dtype):
    h = _api._head_count(weight, bias, x.shape)

    def empty():
        return x.new_empty(_EMPTY, dtype=torch.float32)

    dx = x.new_empty(x.shape, dtype=dx_dtype)
    dw = weight.new_empty(weight.shape) if weight is not None else empty()
    if has_bias:
        db_dtype, db_shape, _ = _api._db_layout(bias, weight, x, h)
        db = x.new_empty(db_shape, dtype=db_dtype)
    else:
        db = empty()
    separate = dresidual_out is not None or (
        has_residual and dresidual_dtype is not None and dresidual_dtype != dx_dtype
    )
    dres = x.new_empty(x.shape, dtype=dresidual_dtype or x.dtype) if separate else empty()
    return dx, dw, db, dres


def _setup_context(ctx, inputs, output):
    x, weight, bias, residual, out_dtype, residual_dtype, eps, store_rstd = inputs
    out, ro, rstd = output
    ctx.x_dtype = x.dtype
    ctx.residual_dtype = residual.dtype if residual is not None else None
    ctx.has_bias = bias is not None
    ctx.has_residual = residual is not None
    ctx.save_for_backward(x if residual is None else ro, weight, bias, rstd)


def _backward(ctx, g_out, g_ro, g_rstd):
    x, weight, bias, rstd = ctx.saved_tensors
    dro = g_ro if (ctx.has_residual and g_ro is not None) else None
    if g_out is None:
        dx = dro.to(ctx.x_dtype) if dro is not None else None
        dres = dro.to(ctx.residual_dtype) if (dro is not None and ctx.residual_dtype is not None) else None
        return dx, None, None, dres, None, None, None, None
    dx, dw, db, dres = bwd_op(
        x, weight, g_out.contiguous(), rstd, dro.contiguous() if dro is not None else None, bias,
        ctx.has_bias, ctx.has_residual, ctx.x_dtype, ctx.residual_dtype,
    )
    dw = dw if weight is not None else None
    db = db if ctx.has_bias else None
    if ctx.has_residual:
        dres = dres if dres.numel() > 0 or x.numel() == 0 else dx
    else:
        dres = None
    return dx, dw, db, dres, None, None, None, None


fwd_op.register_autograd(_backward, setup_context=_setup_context)


def rmsnorm_compiled(x, weight, bias, residual, out_dtype, residual_dtype, eps, prenorm):
    """`rmsnorm()` as traced by torch.compile: the same flattening and prenorm contract."""
    h = _api._head_count(weight, bias, x.shape)
    x_shape = x.shape
    flatten = h == 1
    xa = x.reshape(-1, x.shape[-1]) if flatten else x
    ra = residual.reshape(-1, residual.shape[-1]) if (flatten and residual is not None) else residual
    need = torch.is_grad_enabled() and any(
        t is not None and t.requires_grad for t in (x, weight, bias, residual)
    )
    out, ro, _ = fwd_op(xa, weight, bias, ra, out_dtype, residual_dtype, float(eps), bool(need))
    if flatten:
        out = out.reshape(x_shape)
    if residual is not None and prenorm:
        return out, (ro.reshape(x_shape) if flatten else ro)
    return out

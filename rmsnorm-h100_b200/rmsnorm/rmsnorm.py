# SPDX-License-Identifier: MIT
"""QuACK-compatible RMSNorm API backed by the B200 (sm_100a) kernels of librmsnorm_b200.

Same public surface as the reference package (rmsnorm/rmsnorm.py of Int21-AI/RMSNorm-H100):
`rmsnorm`, `rmsnorm_fwd`, `rmsnorm_bwd` (+ `_tuned` aliases), `rmsnorm_ref`,
`rmsnorm_bwd_ref`, `RMSNormFunction`, `QuackRMSNorm` and the LayerNorm helpers, with the
same argument meaning, return conventions and exception types/messages.

Routing differs from the reference on purpose: every CUDA tensor goes through the native
library (the reference sent bias, fp32-residual, mixed-dtype, mixed 1-D/2-D affine and
non-vectorisable shapes to PyTorch ops, rmsnorm/rmsnorm.py:207-227, 443-468). Tensors on
the host follow the reference's PyTorch semantics (module `_host`). There is no other path.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor

from . import _host
from . import _lib

_SUPPORTED_DTYPES = {torch.float16, torch.bfloat16, torch.float32}
_SUPPORTED_DTYPE_NAMES = "float32, float16 or bfloat16"


# ---------------------------------------------------------------------------------------
# Validation (messages and exception types as pinned by the reference's tests,
# tests/test_rmsnorm_correctness.py:102-203; checks follow rmsnorm/rmsnorm.py:51-179)
# ---------------------------------------------------------------------------------------
def _check_x_shape(x_shape: torch.Size) -> None:
    if len(x_shape) == 0:
        raise ValueError("RMSNorm input must have at least one dimension")
    if x_shape[-1] == 0:
        raise ValueError("RMSNorm hidden dimension must be nonzero")


def _affine_head_count(name: str, tensor: Optional[Tensor], x_shape: torch.Size) -> int:
    """1 for a shared (N,) parameter, H for a per-head (H, N) one (rmsnorm.py:58-81)."""
    if tensor is None:
        return 1
    n = x_shape[-1]
    if tensor.dim() == 1:
        if tensor.shape[0] != n:
            raise ValueError(
                f"{name} shape must be (N,) or (H, N) with N={n}, got {tuple(tensor.shape)}"
            )
        return 1
    if tensor.dim() == 2:
        if len(x_shape) < 2:
            raise ValueError(f"per-head {name} requires x to have at least two dimensions")
        if tensor.shape[1] != n:
            raise ValueError(
                f"{name} shape must be (N,) or (H, N) with N={n}, got {tuple(tensor.shape)}"
            )
        if tensor.shape[0] != x_shape[-2]:
            raise ValueError(
                f"per-head {name} expected x.shape[-2] == {tensor.shape[0]}, got {x_shape[-2]}"
            )
        return int(tensor.shape[0])
    raise ValueError(f"{name} shape must be (N,) or (H, N), got {tuple(tensor.shape)}")


def _check_same_device(name: str, tensor: Optional[Tensor], device: torch.device) -> None:
    if tensor is not None and tensor.device != device:
        raise ValueError(f"{name} must be on the same device as x")


def _check_tensor_dtype(name: str, tensor: Optional[Tensor]) -> None:
    if tensor is not None and tensor.dtype not in _SUPPORTED_DTYPES:
        raise AssertionError(f"{name} must be {_SUPPORTED_DTYPE_NAMES}")


def _check_optional_dtype(name: str, dtype: Optional[torch.dtype]) -> None:
    if dtype is not None and dtype not in _SUPPORTED_DTYPES:
        raise AssertionError(f"{name} must be {_SUPPORTED_DTYPE_NAMES}")


def _validate_fwd_dtypes(x, weight, bias, residual, out_dtype, residual_dtype) -> None:
    if x.dtype not in _SUPPORTED_DTYPES:
        raise AssertionError("Unsupported dtype")
    _check_tensor_dtype("Weight", weight)
    _check_tensor_dtype("Bias", bias)
    _check_tensor_dtype("Residual", residual)
    _check_optional_dtype("out_dtype", out_dtype)
    _check_optional_dtype("residual_dtype", residual_dtype)


def _head_count(weight: Optional[Tensor], bias: Optional[Tensor], x_shape: torch.Size) -> int:
    _check_x_shape(x_shape)
    wh = _affine_head_count("weight", weight, x_shape)
    bh = _affine_head_count("bias", bias, x_shape)
    if wh > 1 and bh > 1 and wh != bh:
        raise ValueError(f"weight and bias head counts must match, got {wh} and {bh}")
    return max(wh, bh)


def _validate_fwd_shapes(x, weight, bias, residual) -> int:
    _check_same_device("weight", weight, x.device)
    _check_same_device("bias", bias, x.device)
    _check_same_device("residual", residual, x.device)
    h = _head_count(weight, bias, x.shape)
    if residual is not None and residual.shape != x.shape:
        raise ValueError(
            f"residual shape must match x shape {tuple(x.shape)}, got {tuple(residual.shape)}"
        )
    return h


def _validate_bwd_shapes(x, weight, bias, dout, rstd, dresidual_out) -> int:
    for name, t in (("weight", weight), ("bias", bias), ("dout", dout), ("rstd", rstd),
                    ("dresidual_out", dresidual_out)):
        _check_same_device(name, t, x.device)
    h = _head_count(weight, bias, x.shape)
    if dout.shape != x.shape:
        raise ValueError(f"dout shape must match x shape {tuple(x.shape)}, got {tuple(dout.shape)}")
    if rstd.dtype != torch.float32:
        raise ValueError("rstd must be float32")
    rows = x.numel() // x.shape[-1]
    if rstd.numel() != rows:
        raise ValueError(f"rstd must have one element per row, got {rstd.numel()} for {rows} rows")
    if dresidual_out is not None and dresidual_out.shape != x.shape:
        raise ValueError(
            f"dresidual_out shape must match x shape {tuple(x.shape)}, "
            f"got {tuple(dresidual_out.shape)}"
        )
    return h


def _contig(t: Optional[Tensor]) -> Optional[Tensor]:
    """Contiguous, 16-byte aligned view (or copy) the kernels can stream with TMA.
    Misaligned storage offsets still work (the library takes its generic path); a copy
    is made only for non-contiguous tensors, as the reference did (rmsnorm.py:42-43)."""
    if t is None:
        return None
    return t if t.is_contiguous() else t.contiguous()


def _heads_of(t: Optional[Tensor], h: int) -> int:
    return h if (t is not None and t.dim() == 2 and h > 1) else 1


# ---------------------------------------------------------------------------------------
# References (fp32 math, rmsnorm/rmsnorm.py:230-243 and 390-399), device-agnostic
# ---------------------------------------------------------------------------------------
rmsnorm_ref = _host.rmsnorm_ref
rmsnorm_bwd_ref = _host.rmsnorm_bwd_ref


# ---------------------------------------------------------------------------------------
# Forward
# ---------------------------------------------------------------------------------------
def rmsnorm_fwd(
    x: Tensor,
    weight: Optional[Tensor] = None,
    bias: Optional[Tensor] = None,
    residual: Optional[Tensor] = None,
    out_dtype: Optional[torch.dtype] = None,
    residual_dtype: Optional[torch.dtype] = None,
    eps: float = 1e-6,
    store_rstd: bool = False,
) -> Tuple[Tensor, Tensor, Optional[Tensor]]:
    """Returns (out, residual_out, rstd) like the reference (rmsnorm/rmsnorm.py:274-387).

    residual_out is x itself (same storage) when there is no residual and residual_dtype is
    None or x.dtype; rstd (fp32, shape x.shape[:-1]) only when store_rstd."""
    out_dtype = x.dtype if out_dtype is None else out_dtype
    _validate_fwd_dtypes(x, weight, bias, residual, out_dtype, residual_dtype)
    h = _validate_fwd_shapes(x, weight, bias, residual)
    if not x.is_cuda:
        return _host.fallback_fwd(x, weight, bias, residual, out_dtype, residual_dtype, eps, store_rstd)

    x_c = _contig(x)
    res_c = _contig(residual)
    n = x.shape[-1]
    rows = x_c.numel() // n
    out = torch.empty(x_c.shape, dtype=out_dtype, device=x.device)
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device) if store_rstd else None
    if residual is not None:
        residual_out = torch.empty(x_c.shape, dtype=residual_dtype or residual.dtype, device=x.device)
    elif residual_dtype is not None and residual_dtype != x.dtype:
        residual_out = torch.empty(x_c.shape, dtype=residual_dtype, device=x.device)
    else:
        residual_out = None
    _lib.fwd(
        x_c, res_c,
        _contig(weight), _heads_of(weight, h),
        _contig(bias), _heads_of(bias, h),
        out, residual_out, rstd, h, float(eps),
    )
    if residual_out is None:
        residual_out = x_c
    return out, residual_out, (rstd.reshape(x_c.shape[:-1]) if rstd is not None else None)


# ---------------------------------------------------------------------------------------
# Backward
# ---------------------------------------------------------------------------------------
def _db_layout(bias, weight, x, h):
    """(dtype, shape, heads) of dbias, as rmsnorm/rmsnorm.py:489-498 and 519-525 pick them."""
    if bias is not None:
        return bias.dtype, bias.shape, _heads_of(bias, h)
    if weight is not None:
        return weight.dtype, weight.shape, _heads_of(weight, h)
    return x.dtype, torch.Size((h, x.shape[-1]) if h > 1 else (x.shape[-1],)), h


def _bwd_cuda(x, weight, dout, rstd, dresidual_out, has_bias, has_residual, bias, h,
              dx_dtype=None, dresidual_dtype=None, dw_out=None, db_out=None, peer_group=None):
    """dw_out / db_out: caller buffers (any float dtype, the affine shapes) that receive
    dweight / dbias instead of new tensors in the affine dtypes. peer_group: a native peer
    group handle; dweight / dbias are then summed over its ranks in the same launch."""
    x_c = _contig(x)
    dout_c = _contig(dout)
    dro_c = _contig(dresidual_out)
    rstd_c = rstd.contiguous().reshape(-1)
    dx = torch.empty(x_c.shape, dtype=dx_dtype or x.dtype, device=x.device)
    w_c = _contig(weight)
    dw = None
    if weight is not None:
        dw = dw_out if dw_out is not None else torch.empty(weight.shape, dtype=weight.dtype, device=x.device)
    db = None
    db_heads = 1
    if has_bias:
        db_dtype, db_shape, db_heads = _db_layout(bias, weight, x, h)
        db = db_out if db_out is not None else torch.empty(db_shape, dtype=db_dtype, device=x.device)
    dresidual = None
    if dresidual_out is not None or (
        has_residual and dresidual_dtype is not None and dresidual_dtype != dx.dtype
    ):
        dresidual = torch.empty(x_c.shape, dtype=dresidual_dtype or x.dtype, device=x.device)
    a = _lib.bwd_args(
        x_c, dout_c, rstd_c, w_c, _heads_of(weight, h), dro_c, dx, dresidual, dw, db, db_heads, h
    )
    _lib.bwd(a, x.device, peer_group=peer_group)
    if has_residual and dresidual is None:
        dresidual = dx
    return dx, dw, db, dresidual


def rmsnorm_bwd(
    x: Tensor,
    weight: Optional[Tensor],
    dout: Tensor,
    rstd: Tensor,
    dresidual_out: Optional[Tensor] = None,
    has_bias: bool = False,
    has_residual: bool = False,
    bias: Optional[Tensor] = None,
) -> Tuple[Tensor, Optional[Tensor], Optional[Tensor], Optional[Tensor]]:
    """Returns (dx, dweight, dbias, dresidual) like the reference (rmsnorm/rmsnorm.py:402-528).

    dx has x.dtype and includes dresidual_out; dweight/dbias follow the affine tensors'
    dtypes and shapes (per-head (H, N) stays per-head); dresidual is dx when has_residual
    and no dresidual_out is given, a separate tensor with the same values otherwise."""
    if x.dtype not in _SUPPORTED_DTYPES:
        raise AssertionError("Unsupported dtype")
    _check_tensor_dtype("Weight", weight)
    _check_tensor_dtype("Bias", bias)
    _check_tensor_dtype("dout", dout)
    _check_tensor_dtype("dresidual_out", dresidual_out)
    h = _validate_bwd_shapes(x, weight, bias, dout, rstd, dresidual_out)
    if not x.is_cuda:
        return _host.fallback_bwd(x, weight, dout, rstd, dresidual_out, has_bias, has_residual, bias)
    dx, dw, db, dresidual = _bwd_cuda(x, weight, dout, rstd, dresidual_out, has_bias, has_residual, bias, h)
    return dx, dw, db, dresidual


def _grad_layout(x: Tensor, weight: Optional[Tensor], bias: Optional[Tensor], has_bias: bool):
    """Shapes of dweight and dbias (None when absent), as rmsnorm_bwd returns them."""
    h = _head_count(weight, bias, x.shape)
    dw_shape = weight.shape if weight is not None else None
    db_shape = _db_layout(bias, weight, x, h)[1] if has_bias else None
    return dw_shape, db_shape


def _rmsnorm_bwd_fp32_grads(x, weight, dout, rstd, dresidual_out, has_bias, has_residual, bias, dw32, db32,
                            peer_group=None):
    """rmsnorm_bwd, except that dweight / dbias are written in fp32 into dw32 / db32
    (fp32 tensors of the shapes _grad_layout gives) whatever the affine dtypes. A
    row-sharded backward sums these per-rank fp32 values across ranks and rounds once to
    the parameters' dtypes (with `peer_group`, a native peer group handle, the library does
    that sum itself, in the launch that reduces them). Returns (dx, dresidual)."""
    if x.dtype not in _SUPPORTED_DTYPES:
        raise AssertionError("Unsupported dtype")
    _check_tensor_dtype("Weight", weight)
    _check_tensor_dtype("Bias", bias)
    _check_tensor_dtype("dout", dout)
    _check_tensor_dtype("dresidual_out", dresidual_out)
    h = _validate_bwd_shapes(x, weight, bias, dout, rstd, dresidual_out)
    for t in (dw32, db32):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous() or t.device != x.device):
            raise ValueError("gradient buffers must be contiguous float32 tensors on x's device")
    if not x.is_cuda:
        dx, _, _, dres = _host.fallback_bwd(x, weight, dout, rstd, dresidual_out, False, has_residual, bias)
        g = dout.float()
        if dw32 is not None:
            dw32.copy_(_host.sum_to_affine_shape(g * (x.float() * rstd.float().unsqueeze(-1)), dw32.shape))
        if db32 is not None:
            db32.copy_(_host.sum_to_affine_shape(g, db32.shape))
        return dx, dres
    dx, _, _, dres = _bwd_cuda(x, weight, dout, rstd, dresidual_out, has_bias, has_residual, bias, h,
                               dw_out=dw32, db_out=db32, peer_group=peer_group)
    return dx, dres


# ---------------------------------------------------------------------------------------
# Autograd (rmsnorm/rmsnorm.py:531-595)
# ---------------------------------------------------------------------------------------
class RMSNormFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias=None, residual=None, out_dtype=None, residual_dtype=None,
                eps=1e-6, prenorm=False):
        need_grad = any(ctx.needs_input_grad[:4])
        out, residual_out, rstd = rmsnorm_fwd(
            x, weight, bias=bias, residual=residual, out_dtype=out_dtype,
            residual_dtype=residual_dtype, eps=eps, store_rstd=need_grad,
        )
        ctx.x_dtype = x.dtype
        ctx.residual_dtype = residual.dtype if residual is not None else None
        ctx.save_for_backward(x if residual is None else residual_out, weight, bias, rstd)
        ctx.has_bias = bias is not None
        ctx.has_residual = residual is not None
        ctx.prenorm = prenorm
        if residual is not None and prenorm:
            return out, residual_out
        return out

    @staticmethod
    def backward(ctx, dout, *args):
        x, weight, bias, rstd = ctx.saved_tensors
        dresidual_out = args[0] if ctx.prenorm and ctx.has_residual else None
        if dout is None:
            dx = dresidual_out.to(ctx.x_dtype) if dresidual_out is not None else None
            dresidual = (
                dresidual_out.to(ctx.residual_dtype)
                if dresidual_out is not None and ctx.residual_dtype is not None
                else None
            )
            return dx, None, None, dresidual, *([None] * 4)
        dout = dout.contiguous()
        dresidual_out = dresidual_out.contiguous() if dresidual_out is not None else None
        if x.is_cuda:
            h = _head_count(weight, bias, x.shape)
            # dx and dresidual are written directly in the dtypes autograd returns, so the
            # reference's extra casts (rmsnorm/rmsnorm.py:587-594) become no-ops
            dx, dw, db, dresidual = _bwd_cuda(
                x, weight, dout, rstd, dresidual_out, ctx.has_bias, ctx.has_residual, bias, h,
                dx_dtype=ctx.x_dtype, dresidual_dtype=ctx.residual_dtype,
            )
        else:
            dx, dw, db, dresidual = rmsnorm_bwd(
                x, weight, dout, rstd, dresidual_out, ctx.has_bias,
                has_residual=ctx.has_residual, bias=bias,
            )
        if dx is not None and dx.dtype != ctx.x_dtype:
            dx = dx.to(ctx.x_dtype)
        if dresidual is not None and ctx.residual_dtype is not None and dresidual.dtype != ctx.residual_dtype:
            dresidual = dresidual.to(ctx.residual_dtype)
        return dx, dw, db, dresidual, *([None] * 4)


def rmsnorm(
    x: Tensor,
    weight: Optional[Tensor] = None,
    bias: Optional[Tensor] = None,
    residual: Optional[Tensor] = None,
    out_dtype: Optional[torch.dtype] = None,
    residual_dtype: Optional[torch.dtype] = None,
    eps: float = 1e-6,
    prenorm: bool = False,
) -> Tensor:
    """RMSNorm with autograd (rmsnorm/rmsnorm.py:598-638). Returns out, or
    (out, residual_out) when a residual is given and prenorm is True."""
    out_dtype = out_dtype or x.dtype
    _validate_fwd_dtypes(x, weight, bias, residual, out_dtype, residual_dtype)
    h = _validate_fwd_shapes(x, weight, bias, residual)
    if not x.is_cuda:
        out, residual_out, _ = _host.fallback_fwd(
            x, weight, bias, residual, out_dtype, residual_dtype, eps, False
        )
        if residual is None or not prenorm:
            return out
        return out, residual_out
    if torch.compiler.is_compiling():
        from . import _compile

        return _compile.rmsnorm_compiled(x, weight, bias, residual, out_dtype, residual_dtype, eps, prenorm)

    x_shape = x.shape
    x_c = _contig(x)
    res_c = _contig(residual)
    flatten = h == 1
    x_arg = x_c.reshape(-1, x_c.shape[-1]) if flatten else x_c
    res_arg = res_c.reshape(-1, res_c.shape[-1]) if (flatten and res_c is not None) else res_c
    result = RMSNormFunction.apply(x_arg, weight, bias, res_arg, out_dtype, residual_dtype, eps, prenorm)
    if not flatten:
        return result
    if isinstance(result, tuple):
        return tuple(t.reshape(x_shape) for t in result)
    return result.reshape(x_shape)


class QuackRMSNorm(torch.nn.RMSNorm):
    """torch.nn.RMSNorm whose forward runs the B200 kernels (rmsnorm/rmsnorm.py:641-648)."""

    def __init__(self, dim: int, eps: float = 1e-6, elementwise_affine: bool = True, device=None, dtype=None):
        super().__init__(dim, eps, elementwise_affine, device=device, dtype=dtype)

    def forward(self, x: Tensor) -> Tensor:
        return rmsnorm(x, self.weight, eps=self.eps)


# ---------------------------------------------------------------------------------------
# LayerNorm. The reference computes these with PyTorch ops (rmsnorm/rmsnorm.py:651-686);
# here layernorm_fwd on CUDA tensors runs the library's LayerNorm kernels. The *_ref
# helpers stay the reference's PyTorch formulas.
# ---------------------------------------------------------------------------------------
layernorm_ref = _host.layernorm_ref
layernorm_rstd_ref = _host.layernorm_rstd_ref
layernorm_mean_ref = _host.layernorm_mean_ref

_LN_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def layernorm_fwd(
    x: Tensor,
    weight: Tensor,
    bias: Optional[Tensor] = None,
    eps: float = 1e-6,
    return_rstd: bool = False,
    return_mean: bool = False,
):
    """LayerNorm forward (rmsnorm/rmsnorm.py:655-676): `out` normalises over weight's shape
    (the trailing weight.dim() dimensions of x, as torch.nn.functional.layer_norm does) and
    is returned in x.dtype; `rstd` and `mean` (fp32) are over the last dimension, as the
    reference returns them. Returns out, (out, rstd), (out, mean) or (out, rstd, mean)."""
    if not x.is_cuda:
        return _host.layernorm_fwd(x, weight, bias, eps, return_rstd, return_mean)
    nshape = tuple(weight.shape)
    if x.dim() < len(nshape) or tuple(x.shape[x.dim() - len(nshape):]) != nshape:
        raise RuntimeError(
            f"Given normalized_shape={list(nshape)}, expected input with shape "
            f"[*, {', '.join(str(d) for d in nshape)}], but got input of size{list(x.shape)}"
        )
    if bias is not None and tuple(bias.shape) != nshape:
        raise RuntimeError(f"Expected bias to be of same shape as normalized_shape, but got bias of shape "
                           f"{list(bias.shape)} and normalized_shape = {list(nshape)}")
    for t in (weight, bias):
        if t is not None and t.device != x.device:
            raise RuntimeError("Expected all tensors to be on the same device")
    if x.dtype not in _LN_DTYPES or weight.dtype not in _LN_DTYPES or (bias is not None and bias.dtype not in _LN_DTYPES):
        raise TypeError("layernorm_fwd supports float16, bfloat16 and float32 tensors on CUDA")
    xc = x.contiguous()
    out = torch.empty_like(xc)
    need_stats = return_rstd or return_mean
    mean = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device) if need_stats else None
    rstd = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device) if return_rstd else None
    if x.numel() > 0:
        w = weight.contiguous()
        b = bias.contiguous() if bias is not None else None
        if weight.dim() == 1:
            _lib.layernorm_fwd(xc, x.shape[-1], w, b, out, mean, rstd, eps)
        else:
            _lib.layernorm_fwd(xc, weight.numel(), w, b, out, None, None, eps)
            if need_stats:
                _lib.layernorm_fwd(xc, x.shape[-1], None, None, None, mean, rstd, eps)
    if return_rstd and return_mean:
        return out, rstd, mean
    if return_rstd:
        return out, rstd
    if return_mean:
        return out, mean
    return out

rmsnorm_fwd_tuned = rmsnorm_fwd
rmsnorm_bwd_tuned = rmsnorm_bwd

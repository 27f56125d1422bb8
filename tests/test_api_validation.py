# SPDX-License-Identifier: MIT
"""Drop-in contract of the Python API that needs no GPU: exported names, signatures,
exception types and messages (the reference pins them in
tests/test_rmsnorm_correctness.py:102-203), host-tensor semantics of out_dtype /
residual_dtype / prenorm / bias-only / dresidual_out / rank-3 and per-head reductions
(:49-366), and the LayerNorm helpers (:369-430)."""

from __future__ import annotations

import inspect

import pytest
import torch

import rmsnorm
from rmsnorm import layernorm_fwd, rmsnorm_bwd, rmsnorm_fwd

REFERENCE_EXPORTS = [
    "QuackRMSNorm", "layernorm_fwd", "layernorm_mean_ref", "layernorm_ref", "layernorm_rstd_ref",
    "rmsnorm", "rmsnorm_bwd", "rmsnorm_bwd_ref", "rmsnorm_bwd_tuned", "rmsnorm_fwd",
    "rmsnorm_fwd_tuned", "rmsnorm_ref",
]


def test_exports_match_reference():
    assert sorted(rmsnorm.__all__) == sorted(REFERENCE_EXPORTS)
    for name in REFERENCE_EXPORTS:
        assert hasattr(rmsnorm, name)
    assert rmsnorm.rmsnorm_fwd_tuned is rmsnorm.rmsnorm_fwd
    assert rmsnorm.rmsnorm_bwd_tuned is rmsnorm.rmsnorm_bwd


@pytest.mark.parametrize("fn,params", [
    ("rmsnorm", ["x", "weight", "bias", "residual", "out_dtype", "residual_dtype", "eps", "prenorm"]),
    ("rmsnorm_fwd", ["x", "weight", "bias", "residual", "out_dtype", "residual_dtype", "eps", "store_rstd"]),
    ("rmsnorm_bwd", ["x", "weight", "dout", "rstd", "dresidual_out", "has_bias", "has_residual", "bias"]),
    ("rmsnorm_ref", ["x", "w", "bias", "residual", "eps"]),
    ("rmsnorm_bwd_ref", ["x", "w", "dout", "rstd", "eps"]),
])
def test_signatures_match_reference(fn, params):
    assert list(inspect.signature(getattr(rmsnorm, fn)).parameters) == params


def _x():
    return torch.randn(2, 16, dtype=torch.float32)


def test_unsupported_dtypes_raise_assertion_errors():
    x = _x()
    with pytest.raises(AssertionError, match="Unsupported dtype"):
        rmsnorm.rmsnorm(torch.ones(2, 16, dtype=torch.int32))
    with pytest.raises(AssertionError, match="Weight must"):
        rmsnorm.rmsnorm(x, torch.ones(16, dtype=torch.int32))
    with pytest.raises(AssertionError, match="Bias must"):
        rmsnorm.rmsnorm(x, None, bias=torch.ones(16, dtype=torch.int32))
    with pytest.raises(AssertionError, match="Residual must"):
        rmsnorm.rmsnorm(x, None, residual=torch.ones_like(x, dtype=torch.int32))
    with pytest.raises(AssertionError, match="out_dtype must"):
        rmsnorm.rmsnorm(x, None, out_dtype=torch.int32)
    with pytest.raises(AssertionError, match="residual_dtype must"):
        rmsnorm.rmsnorm(x, None, residual_dtype=torch.int32)
    with pytest.raises(AssertionError, match="Weight must"):
        rmsnorm_fwd(x, torch.ones(16, dtype=torch.int32))
    with pytest.raises(AssertionError, match="Residual must"):
        rmsnorm_fwd(x, None, residual=torch.ones_like(x, dtype=torch.int32))


def test_shape_validation_messages():
    x = _x()
    with pytest.raises(ValueError, match="residual shape must match x shape"):
        rmsnorm.rmsnorm(x, torch.randn(16), residual=torch.randn(1, 16))
    with pytest.raises(ValueError, match="per-head weight expected"):
        rmsnorm.rmsnorm(torch.randn(2, 3, 16), torch.randn(2, 16))
    with pytest.raises(ValueError, match="at least one dimension"):
        rmsnorm.rmsnorm(torch.tensor(1.0))
    with pytest.raises(ValueError, match="hidden dimension must be nonzero"):
        rmsnorm.rmsnorm(torch.empty(2, 0))
    with pytest.raises(ValueError, match="weight shape must be"):
        rmsnorm.rmsnorm(x, torch.randn(8))
    with pytest.raises(ValueError, match="per-head bias requires x"):
        rmsnorm.rmsnorm(torch.randn(16), None, bias=torch.randn(1, 16))
    # a per-head bias whose head count differs from x.shape[-2] trips the bias's own check
    with pytest.raises(ValueError, match="per-head bias expected"):
        rmsnorm.rmsnorm(torch.randn(2, 3, 16), torch.randn(3, 16), bias=torch.randn(2, 16))


def test_backward_validation_messages():
    with pytest.raises(ValueError, match="at least one dimension"):
        rmsnorm_bwd(torch.tensor(1.0), None, torch.tensor(1.0), torch.tensor(1.0))
    with pytest.raises(ValueError, match="hidden dimension must be nonzero"):
        rmsnorm_bwd(torch.empty(2, 0), None, torch.empty(2, 0), torch.empty(2))
    x = _x()
    with pytest.raises(ValueError, match="rstd must be float32"):
        rmsnorm_bwd(x, None, torch.randn_like(x), torch.rsqrt(x.square().mean(-1) + 1e-6).half())
    rstd = torch.rsqrt(x.square().mean(-1) + 1e-6)
    with pytest.raises(AssertionError, match="dout must"):
        rmsnorm_bwd(x, None, torch.ones_like(x, dtype=torch.int32), rstd)
    with pytest.raises(AssertionError, match="dresidual_out must"):
        rmsnorm_bwd(x, None, torch.randn_like(x), rstd, dresidual_out=torch.ones_like(x, dtype=torch.int32))
    with pytest.raises(ValueError, match="rstd must have one element per row"):
        rmsnorm_bwd(x, None, torch.randn_like(x), rstd[:1])
    with pytest.raises(ValueError, match="dout shape must match"):
        rmsnorm_bwd(x, None, torch.randn(2, 8), rstd)


def test_host_semantics_out_and_residual_dtypes():
    torch.manual_seed(0)
    x = torch.randn(3, 16, dtype=torch.float16)
    res = torch.randn_like(x)
    w = torch.randn(16)
    out, ro = rmsnorm.rmsnorm(x, w, residual=res, residual_dtype=torch.float32, prenorm=True)
    assert out.dtype == torch.float16 and ro.dtype == torch.float32
    assert torch.equal(ro, x.float() + res.float())
    out = rmsnorm.rmsnorm(torch.randn(2, 16), w, out_dtype=torch.float16)
    assert out.dtype == torch.float16
    # residual_out aliases x without a residual, and is a cast copy with another residual_dtype
    xx = torch.randn(4, 16)
    _, ro, rstd = rmsnorm_fwd(xx, w)
    assert ro is xx and rstd is None
    _, ro, rstd = rmsnorm_fwd(xx, w, residual_dtype=torch.float16, store_rstd=True)
    assert ro.dtype == torch.float16 and rstd.shape == (4,)


def test_host_backward_dresidual_out_and_reductions():
    torch.manual_seed(10)
    x = torch.randn(2, 16)
    dout = torch.randn_like(x)
    dro = torch.randn_like(x)
    rstd = torch.rsqrt(x.square().mean(-1) + 1e-6)
    dx, dw, db, dres = rmsnorm_bwd(x, None, dout, rstd, dresidual_out=dro, has_residual=True)
    xhat = x * rstd[:, None]
    ref = (dout - xhat * (xhat * dout).mean(-1, keepdim=True)) * rstd[:, None] + dro
    assert torch.allclose(dx, ref, atol=1e-5, rtol=1e-5) and dres is dx and dw is None and db is None
    x3 = torch.randn(2, 3, 16)
    w = torch.randn(16)
    d3 = torch.randn_like(x3)
    r3 = torch.rsqrt(x3.square().mean(-1) + 1e-6)
    dx, dw, db, dres = rmsnorm_bwd(x3, w, d3, r3, has_bias=True)
    assert dw.shape == w.shape and db.shape == w.shape and dres is None
    assert torch.allclose(db, d3.sum(dim=(0, 1)), atol=1e-5)


def test_quack_module_is_torch_rmsnorm():
    m = rmsnorm.QuackRMSNorm(16)
    assert isinstance(m, torch.nn.RMSNorm) and m.eps == 1e-6
    x = torch.randn(2, 16)
    assert torch.allclose(m(x), rmsnorm.rmsnorm_ref(x, m.weight), atol=1e-6)


def test_layernorm_helpers():
    torch.manual_seed(5)
    x = torch.randn(3, 16, dtype=torch.float16)
    w = torch.randn(16)
    b = torch.randn(16)
    out, rstd = layernorm_fwd(x, w, bias=b, return_rstd=True)
    xf = x.float()
    mean = xf.mean(-1)
    var = ((xf - mean[:, None]) ** 2).mean(-1)
    assert out.dtype == x.dtype
    assert torch.allclose(rstd, torch.rsqrt(var + 1e-6), atol=1e-5, rtol=1e-5)
    ref = torch.nn.functional.layer_norm(xf, w.shape, w, b, 1e-6).to(x.dtype)
    assert torch.allclose(out.float(), ref.float(), atol=3e-2, rtol=3e-2)
    _, rstd2, mean2 = layernorm_fwd(x.float(), w, return_rstd=True, return_mean=True)
    assert torch.allclose(mean2, mean, atol=1e-6) and torch.allclose(rstd2, rstd, atol=1e-5)
    assert torch.allclose(rmsnorm.layernorm_mean_ref(x), mean)
    assert torch.allclose(rmsnorm.layernorm_rstd_ref(x), torch.rsqrt(var + 1e-6), atol=1e-5)

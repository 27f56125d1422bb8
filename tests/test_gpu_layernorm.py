# SPDX-License-Identifier: MIT
"""LayerNorm forward on the GPU (layernorm_fwd, rmsnorm/rmsnorm.py:655-676) against the
oracle and the reference's golden vectors. Tolerances as for RMSNorm: out within
rtol*(RMS(ref) + |ref|) with rtol bf16 1.6e-2, fp16 2e-3, fp32 1e-5; mean within
1e-6*(RMS(x) + |mean|); rstd within 1e-5 relative."""

from __future__ import annotations

import pytest
import torch

from conftest import load_golden
from oracle import rmsnorm_oracle as oracle

import rmsnorm
from rmsnorm import _lib

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]
DEV = torch.device("cuda")
BF16, F16, F32 = torch.bfloat16, torch.float16, torch.float32


def _check_stats(x, mean, rstd, ref_mean, ref_rstd, label):
    rms = x.float().square().mean(dim=-1).sqrt()
    if mean is not None:
        err = (mean.cpu() - ref_mean).abs()
        bound = 1e-6 * (rms.cpu() + ref_mean.abs())
        assert bool((err <= bound).all()), f"{label}: mean err {float((err / bound).max()):.2f} x bound"
    if rstd is not None:
        rel = ((rstd.cpu() - ref_rstd).abs() / ref_rstd).max()
        assert float(rel) <= 1e-5, f"{label}: rstd rel err {float(rel):.2e}"


def _case(rows, n, dtype, bias, expect=None, seed=0, outliers=0.0):
    x = oracle.gen((rows, n), dtype, seed, outliers=outliers).to(DEV)
    w = oracle.gen((n,), F32, seed + 1, "weight").to(DEV)
    b = oracle.gen((n,), F32, seed + 2, "bias").to(DEV) if bias else None
    out, rstd, mean = rmsnorm.layernorm_fwd(x, w, bias=b, eps=1e-6, return_rstd=True, return_mean=True)
    torch.cuda.synchronize()
    plan = _lib.last_plan()
    if expect is not None and rows > 0:
        assert expect in plan, plan
    r_out, r_rstd, r_mean, r_y = oracle.layernorm_fwd(x.cpu(), w.cpu(), b.cpu() if b is not None else None, 1e-6)
    assert out.dtype == dtype and out.shape == x.shape
    if rows > 0:
        oracle.check_close(out, r_y, dtype, f"ln out {rows}x{n} {dtype} [{plan}]")
        _check_stats(x, mean, rstd, r_mean, r_rstd, f"ln {rows}x{n} {dtype}")
    return plan


@pytest.mark.parametrize("rows,n,dtype,bias,expect", [
    (1000, 4096, BF16, True, "ln_stream mode=row"),
    (33, 16384, F16, False, "ln_stream mode=row"),
    (257, 2048, F32, True, "ln_stream mode=row"),
    (70, 128, F32, True, "ln_stream mode=seg"),
    (3, 8, BF16, False, "ln_stream mode=seg"),
    (300, 100, BF16, True, "ln_generic"),
    (17, 65536, BF16, True, "ln_generic"),
    (0, 256, F16, True, None),
])
def test_layernorm_matches_oracle(rows, n, dtype, bias, expect):
    _case(rows, n, dtype, bias, expect, seed=rows + n)


def test_layernorm_outliers_and_large_mean():
    # 1% x100 outliers and a shifted mean: the two-pass variance keeps rstd accurate
    x = (oracle.gen((64, 8192), BF16, 3, outliers=0.01).float() + 40.0).to(BF16).to(DEV)
    w = oracle.gen((8192,), F32, 4, "weight").to(DEV)
    out, rstd, mean = rmsnorm.layernorm_fwd(x, w, return_rstd=True, return_mean=True)
    r_out, r_rstd, r_mean, r_y = oracle.layernorm_fwd(x.cpu(), w.cpu(), None, 1e-6)
    oracle.check_close(out, r_y, BF16, "ln shifted out")
    _check_stats(x, mean, rstd, r_mean, r_rstd, "ln shifted")


def test_layernorm_unaligned_storage_takes_generic_path():
    base = oracle.gen((65 * 1024 + 8,), F16, 5).to(DEV)
    x = base[1:1 + 65 * 1024].view(65, 1024)  # storage offset of 2 bytes: not 16-byte aligned
    w = oracle.gen((1024,), F32, 6, "weight").to(DEV)
    out = rmsnorm.layernorm_fwd(x, w)
    assert "ln_generic" in _lib.last_plan()
    _, _, _, r_y = oracle.layernorm_fwd(x.cpu(), w.cpu(), None, 1e-6)
    oracle.check_close(out, r_y, F16, "ln unaligned")


@pytest.mark.parametrize("name", ["ln_fwd_bf16", "ln_fwd_2d_weight", "ln_fwd_f32_n100"])
def test_layernorm_matches_reference_golden(name):
    g = load_golden(name)
    x = g["x"].to(DEV)
    w = g["weight"].to(DEV)
    b = g["bias"].to(DEV) if "bias" in g else None
    has_mean = "mean" in g
    res = rmsnorm.layernorm_fwd(x, w, bias=b, eps=g["meta"]["eps"], return_rstd=True, return_mean=has_mean)
    _, _, _, r_y = oracle.layernorm_fwd(g["x"], g["weight"], g.get("bias"), g["meta"]["eps"])
    oracle.check_close(res[0], r_y, x.dtype, f"{name} out")
    # the reference's own output rounds the same fp32 value: at most one unit apart
    assert float((res[0].cpu().float() - g["out"].float()).abs().max()) <= float(
        (g["out"].float().abs().max()) * (2 ** -7 if x.dtype == BF16 else 2 ** -10 if x.dtype == F16 else 1e-5)), name
    _check_stats(x, res[2] if has_mean else None, res[1], g.get("mean"), g["rstd"], name)


def test_layernorm_two_dim_weight_semantics():
    # out over the last two dims (like torch layer_norm with a 2-D normalized_shape),
    # mean / rstd over the last dim, as the reference returns them
    x = oracle.gen((16, 8, 256), F32, 7).to(DEV)
    w = oracle.gen((8, 256), F32, 8, "weight").to(DEV)
    b = oracle.gen((8, 256), F32, 9, "bias").to(DEV)
    out, rstd, mean = rmsnorm.layernorm_fwd(x, w, bias=b, return_rstd=True, return_mean=True)
    r_out, r_rstd, r_mean, r_y = oracle.layernorm_fwd(x.cpu(), w.cpu(), b.cpu(), 1e-6)
    oracle.check_close(out, r_y, F32, "ln 2-D weight out")
    assert rstd.shape == (16, 8) and mean.shape == (16, 8)
    _check_stats(x, mean, rstd, r_mean, r_rstd, "ln 2-D weight")


def test_layernorm_shape_errors_match_torch():
    x = torch.randn(4, 64, device=DEV)
    with pytest.raises(RuntimeError):
        rmsnorm.layernorm_fwd(x, torch.ones(32, device=DEV))
    with pytest.raises(RuntimeError):
        rmsnorm.layernorm_fwd(x, torch.ones(64, device=DEV), bias=torch.zeros(32, device=DEV))


def test_layernorm_direct_c_abi_statistics_only():
    x = oracle.gen((40, 512), BF16, 10).to(DEV)
    mean = torch.full((40,), float("nan"), device=DEV)
    rstd = torch.full((40,), float("nan"), device=DEV)
    _lib.layernorm_fwd(x, 512, None, None, None, mean, rstd, 1e-6)
    torch.cuda.synchronize()
    _, r_rstd, r_mean, _ = oracle.layernorm_fwd(x.cpu(), torch.ones(512), None, 1e-6)
    _check_stats(x, mean, rstd, r_mean, r_rstd, "ln stats only")
    assert _lib.device_status(DEV) == (0, 0)

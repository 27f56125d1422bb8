# SPDX-License-Identifier: MIT
"""GPU parity: the CUDA path (public API -> ctypes -> C ABI -> sm_100a kernels) against the
CPU oracle on seeded inputs, the golden vectors of the reference, and -- at BASELINE's full
sizes -- an fp32 GPU reference in row chunks. Tolerances (stated by the task, applied as
|a - r| <= rtol * (RMS(r) + |r|)): y / dx rtol bf16 1.6e-2, fp16 2e-3, fp32 1e-5;
dweight / dbias |a - r| <= 1e-3 * sum_rows|term|; residual_out exact; rstd rel 1e-5."""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import load_golden
from oracle import rmsnorm_oracle as oracle

import rmsnorm
from rmsnorm import _lib

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device"),
]

DEV = "cuda"
F16, BF16, F32 = torch.float16, torch.bfloat16, torch.float32


def _g(shape, dtype, seed, kind="normal", outliers=0.0):
    return oracle.gen(shape, dtype, seed, kind, outliers).to(DEV)


def _fwd_case(M, N, dtype, *, residual=None, weight=True, bias=False, store_rstd=True, H=1,
              out_dtype=None, residual_dtype=None, wdtype=F32, seed=0, expect=None):
    shape = (M // H, H, N) if H > 1 else (M, N)
    x = _g(shape, dtype, seed)
    res = None
    if residual == "same":
        res = _g(shape, dtype, seed + 1)
    elif residual == "f32":
        res = _g(shape, F32, seed + 1)
    aff = (H, N) if H > 1 else (N,)
    w = _g(aff, wdtype, seed + 2, "weight") if weight else None
    b = _g(aff, wdtype, seed + 3, "bias") if bias else None
    out, ro, rstd = rmsnorm.rmsnorm_fwd(x, w, b, res, out_dtype=out_dtype, residual_dtype=residual_dtype,
                                        store_rstd=store_rstd)
    torch.cuda.synchronize()
    plan = _lib.last_plan()
    if expect is not None:
        assert expect in plan, plan
    o_out, o_ro, o_rstd, y = oracle.fwd(x.cpu(), None if w is None else w.cpu(), None if b is None else b.cpu(),
                                         None if res is None else res.cpu(), out_dtype=out_dtype,
                                         residual_dtype=residual_dtype)
    odt = out_dtype or dtype
    assert out.dtype == odt and out.shape == x.shape
    oracle.check_close(out, y, odt, f"out M={M} N={N} {dtype} H={H} [{plan}]",
                       rtol=max(oracle.y_tolerance(odt), oracle.y_tolerance(dtype)) if odt != dtype else None)
    if o_ro is None:
        assert ro.data_ptr() == x.data_ptr()
    else:
        assert ro.dtype == o_ro.dtype and torch.equal(ro.cpu(), o_ro), f"residual_out [{plan}]"
    if store_rstd:
        assert rstd.shape == x.shape[:-1]
        assert torch.allclose(rstd.cpu(), o_rstd, rtol=1e-5, atol=0), f"rstd [{plan}]"
    else:
        assert rstd is None
    return plan


# --------------------------------------------------------------------------------------
# forward
# --------------------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", [F16, BF16, F32])
@pytest.mark.parametrize("N", [8, 24, 128, 256, 1024, 4096, 5120, 16384, 32768, 65536])
def test_fwd_shapes(dtype, N):
    _fwd_case(5, N, dtype, expect="fwd_stream")


@pytest.mark.parametrize("dtype", [F16, BF16, F32])
@pytest.mark.parametrize("residual", ["same", "f32"])
@pytest.mark.parametrize("N", [256, 4096, 16384, 131072])
def test_fwd_residual_bias(dtype, residual, N):
    if residual == "f32" and dtype == F32:
        residual = "same"
    _fwd_case(7, N, dtype, residual=residual, bias=True, residual_dtype=F32)
    _fwd_case(3, N, dtype, residual=residual, bias=False, store_rstd=False)


@pytest.mark.parametrize("dtype", [F16, BF16, F32])
def test_fwd_very_long_rows_cluster_split(dtype):
    plan = _fwd_case(3, 262144, dtype, expect="fwd_")
    if "fwd_stream" in plan:
        assert "P=1 " not in plan  # the row is split across a cluster
    _fwd_case(2, 262144, dtype, residual="same", residual_dtype=F32 if dtype != F32 else None)


@pytest.mark.parametrize("M", [1, 2, 3, 17, 64, 1000])
def test_fwd_ragged_row_counts(M):
    _fwd_case(M, 512, BF16, residual="same", bias=True)
    _fwd_case(M, 4096, F16)


@pytest.mark.parametrize("N", [1, 7, 100, 1001, 4100])
def test_fwd_generic_hidden_sizes(N):
    for dt in (F16, BF16, F32):
        _fwd_case(4, N, dt, residual="same", bias=True, expect="fwd_generic")


def test_fwd_misaligned_storage_uses_generic_path():
    base = _g((4 * 256 + 1,), BF16, 40)
    x = base[1:].view(4, 256)  # storage offset of 2 bytes
    w = _g((256,), F32, 41, "weight")
    out, _, rstd = rmsnorm.rmsnorm_fwd(x, w, store_rstd=True)
    torch.cuda.synchronize()
    assert "generic" in _lib.last_plan()
    _, _, o_rstd, y = oracle.fwd(x.cpu(), w.cpu())
    oracle.check_close(out, y, BF16, "misaligned out")
    assert torch.allclose(rstd.cpu(), o_rstd, rtol=1e-5, atol=0)


@pytest.mark.parametrize("H,N,dtype,path", [(32, 128, F16, "mode=seg"), (3, 256, F16, "mode=seg"),
                                            (8, 64, BF16, "mode=seg"), (4, 96, F32, "generic"),
                                            (8, 512, BF16, "generic"), (2, 8, F32, "mode=seg")])
def test_fwd_per_head(H, N, dtype, path):
    _fwd_case(H * 6, N, dtype, H=H, bias=True, expect=path)
    _fwd_case(H * 5, N, dtype, H=H, weight=True, residual="same", residual_dtype=F32)


@pytest.mark.parametrize("H,N,dtype,tokens,cols", [
    (32, 128, F16, 37, "cols=1"),     # 4096-wide super-rows, ragged last tile
    (32, 128, BF16, 4099, "cols=1"),  # many tiles per CTA
    (32, 256, BF16, 21, "cols=2"),    # 8192-wide: two columns per thread
    (64, 128, F32, 9, "cols=2"),
    (8, 64, F32, 45, "cols=1"),       # 512-wide: eight groups of 64 threads
    (3, 256, F16, 29, "cols=1"),      # groups of 96 threads straddle warps
    (4, 16, BF16, 50, "cols=1"),      # segments of 2 lanes (fewer than the 4 values per thread)
    (2, 8, F32, 33, "cols=1"),        # segments of 1 lane
    (128, 128, F16, 5, "cols=4"),     # 16384-wide: four columns (the general kernel)
])
def test_fwd_per_head_column_mode(H, N, dtype, tokens, cols):
    """Per-head forward in column mode (several super-rows per thread per sweep): affine
    variants, rstd stored or not, ragged tiles."""
    _fwd_case(tokens * H, N, dtype, H=H, bias=True, expect=cols)
    _fwd_case(tokens * H, N, dtype, H=H, seed=7, expect=cols)
    _fwd_case(tokens * H, N, dtype, H=H, weight=False, bias=True, store_rstd=False, seed=9, expect=cols)


def test_fwd_per_head_column_mode_off(monkeypatch):
    monkeypatch.setenv("RMSNORM_B200_COL_MODE", "0")
    _fwd_case(37 * 32, 128, F16, H=32, bias=True, expect="cols=4")


def test_fwd_output_and_affine_dtypes():
    _fwd_case(6, 1024, BF16, out_dtype=F32, expect="fwd_stream")
    _fwd_case(6, 1024, F32, out_dtype=BF16)
    _fwd_case(6, 1024, F16, wdtype=BF16, bias=True)
    _fwd_case(6, 1024, BF16, weight=False, bias=True)
    _fwd_case(6, 1024, BF16, weight=False)
    _fwd_case(6, 1024, BF16, residual_dtype=F32)  # residual_out = x cast, no residual


def test_fwd_mixed_shared_and_per_head_affine():
    x = _g((4, 3, 256), F16, 50)
    w = _g((256,), F32, 51, "weight")
    b = _g((3, 256), F32, 52, "bias")
    out, _, rstd = rmsnorm.rmsnorm_fwd(x, w, b, store_rstd=True)
    _, _, o_rstd, y = oracle.fwd(x.cpu(), w.cpu(), b.cpu())
    oracle.check_close(out, y, F16, "mixed affine out")
    assert torch.allclose(rstd.cpu(), o_rstd, rtol=1e-5)


def test_fwd_empty_rows():
    x = torch.empty(0, 256, device=DEV, dtype=BF16)
    w = torch.ones(256, device=DEV)
    out, ro, rstd = rmsnorm.rmsnorm_fwd(x, w, store_rstd=True)
    assert out.shape == (0, 256) and rstd.shape == (0,)


# --------------------------------------------------------------------------------------
# backward
# --------------------------------------------------------------------------------------
def _bwd_case(M, N, dtype, *, H=1, weight=True, has_bias=False, dro=False, seed=100, dy_dtype=None,
              expect=None, repeat_check=True):
    shape = (M // H, H, N) if H > 1 else (M, N)
    x = _g(shape, dtype, seed)
    dy = _g(shape, dy_dtype or dtype, seed + 1)
    aff = (H, N) if H > 1 else (N,)
    w = _g(aff, F32, seed + 2, "weight") if weight else None
    _, _, rstd, _ = oracle.fwd(x.cpu(), w.cpu() if w is not None else None)
    rstd = rstd.to(DEV)
    dres_out = _g(shape, dtype, seed + 3) if dro else None
    dx, dw, db, dres = rmsnorm.rmsnorm_bwd(x, w, dy, rstd, dresidual_out=dres_out, has_bias=has_bias,
                                           has_residual=dro)
    torch.cuda.synchronize()
    plan = _lib.last_plan()
    if expect is not None:
        assert expect in plan, plan
    o_dx, o_dw, o_db, s_dw, s_db = oracle.bwd(x.cpu(), w.cpu() if w is not None else None, dy.cpu(), rstd.cpu(),
                                              dresidual_out=dres_out.cpu() if dro else None,
                                              has_bias=has_bias)
    assert dx.dtype == dtype
    oracle.check_close(dx, o_dx, dtype, f"dx M={M} N={N} {dtype} H={H} [{plan}]")
    if weight:
        assert dw.shape == w.shape and dw.dtype == w.dtype
        oracle.check_reduction(dw, o_dw, s_dw, f"dweight [{plan}]")
    else:
        assert dw is None
    if has_bias:
        oracle.check_reduction(db, o_db, s_db, f"dbias [{plan}]")
    else:
        assert db is None
    if dro:
        assert torch.equal(dres, dx)
    if repeat_check:  # deterministic: a second run is bitwise identical
        dx2, dw2, db2, _ = rmsnorm.rmsnorm_bwd(x, w, dy, rstd, dresidual_out=dres_out, has_bias=has_bias,
                                               has_residual=dro)
        assert torch.equal(dx, dx2)
        if weight:
            assert torch.equal(dw, dw2)
        if has_bias:
            assert torch.equal(db, db2)
    return plan


@pytest.mark.parametrize("dtype", [F16, BF16, F32])
@pytest.mark.parametrize("N", [8, 24, 256, 2048, 4096, 16384, 65536])
def test_bwd_shapes(dtype, N):
    _bwd_case(9, N, dtype, expect="bwd_stream")


@pytest.mark.parametrize("dtype", [F16, BF16, F32])
@pytest.mark.parametrize("N", [512, 8192, 32768])
def test_bwd_bias_and_dresidual(dtype, N):
    _bwd_case(11, N, dtype, has_bias=True, dro=True)
    _bwd_case(5, N, dtype, weight=False, has_bias=True)
    _bwd_case(4, N, dtype, weight=False)


@pytest.mark.parametrize("dtype", [F16, BF16, F32])
def test_bwd_very_long_rows(dtype):
    _bwd_case(3, 262144, dtype)


@pytest.mark.parametrize("M", [1, 3, 17, 300, 2000])
def test_bwd_ragged_and_many_rows(M):
    _bwd_case(M, 1024, BF16, has_bias=True)


@pytest.mark.parametrize("N", [1, 7, 100, 4100])
def test_bwd_generic_hidden_sizes(N):
    for dt in (F16, BF16, F32):
        _bwd_case(6, N, dt, has_bias=True, dro=True, expect="bwd_generic")


@pytest.mark.parametrize("H,N,dtype", [(32, 128, F16), (3, 256, F16), (8, 64, BF16), (4, 96, F32), (8, 512, BF16)])
def test_bwd_per_head(H, N, dtype):
    _bwd_case(H * 7, N, dtype, H=H, has_bias=True)


@pytest.mark.parametrize("H,N,dtype,tokens,cols", [
    (32, 128, F16, 37, "cols=1"),     # ragged last tile
    (32, 128, BF16, 2051, "cols=1"),  # many tiles per CTA (dweight / dbias over many rows)
    (32, 256, BF16, 21, "cols=2"),
    (64, 128, BF16, 9, "cols=2"),
    (64, 128, F32, 9, None),          # fp32: one column tile (2 rows) fills shared memory alone
    (8, 64, BF16, 45, "cols=1"),      # 32 rows per sweep
    (8, 64, F32, 45, None),           # fp32: one 32-row column tile fills shared memory alone
    (3, 256, F16, 29, "cols=1"),      # groups of 96 threads straddle warps
    (4, 16, BF16, 50, "cols=1"),      # segments of 2 lanes
    (2, 8, F16, 333, "cols=1"),       # segments of 1 lane, 1024 rows per sweep
])
def test_bwd_per_head_column_mode(H, N, dtype, tokens, cols):
    """Per-head backward in column mode: dweight / dbias accumulated over several rows per
    thread per sweep, the per-(row, head) rstd read from the staged block."""
    _bwd_case(tokens * H, N, dtype, H=H, has_bias=True, expect=cols)
    _bwd_case(tokens * H, N, dtype, H=H, seed=7, expect=cols)
    # without a per-head weight the rows are plain N-wide rows (no column mode)
    _bwd_case(tokens * H, N, dtype, H=H, weight=False, has_bias=True, seed=9)


def test_bwd_per_head_column_mode_off(monkeypatch):
    monkeypatch.setenv("RMSNORM_B200_COL_MODE", "0")
    plan = _bwd_case(37 * 32, 128, F16, H=32, has_bias=True)
    assert "cols=1" not in plan, plan


def test_bwd_mixed_dtypes_prenorm():
    # saved x is an fp32 residual_out, dout is half/bf16: the prenorm-with-fp32-residual case
    for dy in (F16, BF16):
        x = _g((13, 2048), F32, 60)
        g = _g((13, 2048), dy, 61)
        w = _g((2048,), F32, 62, "weight")
        _, _, rstd, _ = oracle.fwd(x.cpu(), w.cpu())
        dx, dw, _, _ = rmsnorm.rmsnorm_bwd(x, w, g, rstd.to(DEV))
        assert "bwd_stream" in _lib.last_plan()
        o_dx, o_dw, _, s_dw, _ = oracle.bwd(x.cpu(), w.cpu(), g.cpu(), rstd)
        oracle.check_close(dx, o_dx, F32, "mixed dx", rtol=oracle.y_tolerance(dy))
        oracle.check_reduction(dw, o_dw, s_dw, "mixed dweight")


# --------------------------------------------------------------------------------------
# autograd / module (ports of the reference's CUDA tests, tests/test_rmsnorm_correctness.py:433-981)
# --------------------------------------------------------------------------------------
def test_autograd_per_head_weight_and_bias():
    g = load_golden("perhead_cfg4")
    x = g["x"].to(DEV).requires_grad_(True)
    w = g["weight"].to(DEV).requires_grad_(True)
    b = g["bias"].to(DEV).requires_grad_(True)
    out = rmsnorm.rmsnorm(x, w, b)
    (out.float() * g["dout"].to(DEV).float()).sum().backward()
    _, _, rstd, y = oracle.fwd(g["x"], g["weight"], g["bias"])
    oracle.check_close(out, y, F16, "golden per-head out")
    o_dx, o_dw, o_db, s_dw, s_db = oracle.bwd(g["x"], g["weight"], g["dout"], rstd, has_bias=True,
                                              bias_shape=(32, 128))
    oracle.check_close(x.grad, o_dx, F16, "golden per-head dx")
    oracle.check_reduction(w.grad, o_dw, s_dw, "golden per-head dweight")
    oracle.check_reduction(b.grad, o_db, s_db, "golden per-head dbias")
    # and against the reference's own outputs
    assert (out.cpu().float() - g["out"].float()).abs().max() <= 2e-3 * 4
    assert torch.allclose(w.grad.cpu(), g["dweight"], rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("name", ["fwd_cfg1", "fwd_cfg2", "large_cfg5_f32", "large_cfg5_bf16"])
def test_golden_forward(name):
    g = load_golden(name)
    res = g.get("residual")
    out, ro, rstd = rmsnorm.rmsnorm_fwd(g["x"].to(DEV), g["weight"].to(DEV),
                                        g["bias"].to(DEV) if "bias" in g else None,
                                        res.to(DEV) if res is not None else None,
                                        residual_dtype=F32 if res is not None else None, store_rstd=True)
    dt = g["out"].dtype
    _, _, _, y = oracle.fwd(g["x"], g["weight"], g.get("bias"), res)
    oracle.check_close(out, y, dt, f"{name} vs oracle")
    # the reference's stored outputs: at most one rounding step apart
    diff = (out.cpu().float() - g["out"].float()).abs()
    assert (diff <= oracle.y_tolerance(dt) * (g["out"].float().abs() + 1e-3)).all(), name
    assert torch.allclose(rstd.cpu(), g["rstd"], rtol=1e-5, atol=0)
    if res is not None:
        assert torch.equal(ro.cpu(), g["residual_out"])


@pytest.mark.parametrize("name", ["bwd_cfg3", "large_cfg5_f32", "large_cfg5_bf16"])
def test_golden_backward(name):
    g = load_golden(name)
    dx, dw, _, _ = rmsnorm.rmsnorm_bwd(g["x"].to(DEV), g["weight"].to(DEV), g["dout"].to(DEV), g["rstd"].to(DEV))
    o_dx, o_dw, _, s_dw, _ = oracle.bwd(g["x"], g["weight"], g["dout"], g["rstd"])
    oracle.check_close(dx, o_dx, g["dx"].dtype, f"{name} dx")
    oracle.check_reduction(dw, g["dweight"], s_dw, f"{name} dweight vs reference")


def test_autograd_prenorm_fp32_residual():
    g = load_golden("prenorm_mixed")
    x = g["x"].to(DEV).requires_grad_(True)
    res = g["residual"].to(DEV).requires_grad_(True)
    w = g["weight"].to(DEV).requires_grad_(True)
    out, ro = rmsnorm.rmsnorm(x, w, residual=res, residual_dtype=F32, prenorm=True)
    ((out.float() * g["dout"].to(DEV).float()).sum() + (ro * g["dresidual_out"].to(DEV)).sum()).backward()
    assert ro.dtype == F32 and torch.equal(ro.cpu(), g["residual_out"])
    o_dx, o_dw, _, s_dw, _ = oracle.bwd(g["residual_out"], g["weight"], g["dout"],
                                        oracle.fwd(g["x"], g["weight"], residual=g["residual"])[2],
                                        dresidual_out=g["dresidual_out"])
    oracle.check_close(x.grad, o_dx, F16, "prenorm dx")
    oracle.check_close(res.grad, o_dx, F16, "prenorm dresidual")
    oracle.check_reduction(w.grad, o_dw, s_dw, "prenorm dweight")


def test_autograd_residual_only_and_bias_without_weight():
    x = _g((4, 256), F16, 70)
    res = _g((4, 256), F16, 71).requires_grad_(True)
    w = _g((256,), F32, 72, "weight")
    up = _g((4, 256), F16, 73)
    (rmsnorm.rmsnorm(x, w, residual=res) * up).sum().backward()
    h = x.cpu().float() + res.detach().cpu().float()
    _, _, rstd, _ = oracle.fwd(h, w.cpu())
    o_dx, _, _, _, _ = oracle.bwd(h, w.cpu(), up.cpu(), rstd)
    oracle.check_close(res.grad, o_dx, F16, "residual-only grad")

    x = _g((4, 256), F32, 74).requires_grad_(True)
    b = _g((256,), F32, 75, "bias").requires_grad_(True)
    up = _g((4, 256), F32, 76)
    (rmsnorm.rmsnorm(x, None, bias=b) * up).sum().backward()
    _, _, rstd, _ = oracle.fwd(x.detach().cpu())
    o_dx, _, o_db, _, s_db = oracle.bwd(x.detach().cpu(), None, up.cpu(), rstd, has_bias=True)
    oracle.check_close(x.grad, o_dx, F32, "bias-only dx")
    oracle.check_reduction(b.grad, o_db, s_db, "bias-only db")


def test_quack_module_matches_oracle():
    m = rmsnorm.QuackRMSNorm(1024, eps=1e-6, device=DEV, dtype=F32)
    with torch.no_grad():
        m.weight.copy_(_g((1024,), F32, 80, "weight"))
    x = _g((2, 3, 1024), BF16, 81)
    y = m(x)
    _, _, _, ref = oracle.fwd(x.cpu(), m.weight.detach().cpu())
    oracle.check_close(y, ref, BF16, "QuackRMSNorm")


def test_c_abi_direct_call():
    """Calls rmsnorm_b200_fwd through ctypes with a hand-filled argument struct."""
    lib = _lib.load_library()
    x = _g((33, 1024), BF16, 90)
    w = _g((1024,), F32, 91, "weight")
    out = torch.empty_like(x)
    rstd = torch.empty(33, device=DEV)
    a = _lib.FwdArgs(rows=33, hidden=1024, heads=1, x_dtype=_lib.BF16, x=x.data_ptr(),
                     weight_dtype=_lib.F32, weight=w.data_ptr(), weight_heads=1, out_dtype=_lib.BF16,
                     out=out.data_ptr(), rstd=rstd.data_ptr(), eps=1e-6)
    st = lib.rmsnorm_b200_fwd(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.rmsnorm_b200_strerror(st)
    torch.cuda.synchronize()
    _, _, o_rstd, y = oracle.fwd(x.cpu(), w.cpu())
    oracle.check_close(out, y, BF16, "direct ABI out")
    # invalid arguments come back as a status, not an exception or a fault
    bad = _lib.FwdArgs(rows=3, hidden=1024, heads=2, x_dtype=_lib.BF16, x=x.data_ptr(), out=out.data_ptr())
    assert lib.rmsnorm_b200_fwd(ctypes.byref(bad), None) == 1
    assert lib.rmsnorm_b200_fwd(None, None) == 1


def test_bounded_wait_reports_timeout_without_faulting():
    """Failure detection: a wait nothing completes runs out after its bound, the kernel
    records the timeout and returns, and the context stays usable."""
    dev = torch.device(DEV)
    assert _lib.device_status(dev, clear=True) == (0, 0)
    _lib.selftest_wait_timeout(dev, 20_000_000)  # 20 ms
    st, where = _lib.device_status(dev, clear=True)
    assert st == _lib.ERR_DEVICE_TIMEOUT and where == 8
    assert _lib.device_status(dev) == (0, 0)
    _fwd_case(8, 4096, BF16, expect="fwd_stream")  # still works afterwards


# --------------------------------------------------------------------------------------
# BASELINE configurations at full size
# --------------------------------------------------------------------------------------
def _gpu_gen(shape, dtype, seed, kind="normal", outliers=0.0):
    g = torch.Generator(device=DEV).manual_seed(oracle.BASE_SEED + seed)
    t = torch.randn(shape, generator=g, device=DEV, dtype=torch.float32)
    if kind == "weight":
        t = 1.0 + 0.1 * t
    elif kind == "bias":
        t = 0.02 * t
    if outliers > 0:
        t = torch.where(torch.rand(shape, generator=g, device=DEV) < outliers, t * 100.0, t)
    return t.to(dtype)


def _subset_vs_oracle(x, w, b, res, out, ro, rstd, dtype, nrows=128):
    rows = torch.randperm(x.shape[0], generator=torch.Generator().manual_seed(0))[:nrows].sort().values
    o_out, o_ro, o_rstd, y = oracle.fwd_rows_chunked(x, w.cpu() if w is not None else None,
                                                    b.cpu() if b is not None else None, res, rows=rows)
    oracle.check_close(out[rows.to(DEV)], y, dtype, "subset out")
    assert torch.allclose(rstd[rows.to(DEV)].cpu(), o_rstd, rtol=1e-5)


def test_baseline_cfg1_full():
    from gpu_ref import fwd_max_err
    x = _gpu_gen((8192, 4096), BF16, 1)
    w = _gpu_gen((4096,), F32, 2, "weight")
    out, ro, rstd = rmsnorm.rmsnorm_fwd(x, w, store_rstd=True)
    assert ro.data_ptr() == x.data_ptr()
    assert fwd_max_err(x, w, None, None, out, None, rstd, 1e-6, 1.6e-2) <= 1.0
    _subset_vs_oracle(x, w, None, None, out, None, rstd, BF16)


def test_baseline_cfg2_full():
    from gpu_ref import fwd_max_err
    x = _gpu_gen((32768, 16384), BF16, 3)
    res = _gpu_gen((32768, 16384), BF16, 4)
    w = _gpu_gen((16384,), F32, 5, "weight")
    b = _gpu_gen((16384,), F32, 6, "bias")
    out, ro, rstd = rmsnorm.rmsnorm_fwd(x, w, b, res, residual_dtype=F32, store_rstd=True)
    assert "fwd_stream" in _lib.last_plan()
    assert fwd_max_err(x, w, b, res, out, ro, rstd, 1e-6, 1.6e-2) <= 1.0
    _subset_vs_oracle(x, w, b, res, out, ro, rstd, BF16, nrows=32)


def test_baseline_cfg3_full():
    from gpu_ref import bwd_check
    x = _gpu_gen((32768, 65536), BF16, 7)
    dy = _gpu_gen((32768, 65536), BF16, 8)
    w = _gpu_gen((65536,), F32, 9, "weight")
    rstd = torch.rsqrt(torch.stack([x[i:i + 1024].float().square().mean(-1) for i in range(0, 32768, 1024)]).reshape(-1) + 1e-6)
    dx, dw, _, _ = rmsnorm.rmsnorm_bwd(x, w, dy, rstd)
    assert "bwd_stream" in _lib.last_plan()
    dx_err, dw_err = bwd_check(x, w, dy, rstd, dx, dw, 1.6e-2)
    assert dx_err <= 1.0 and dw_err <= 1.0, (dx_err, dw_err)
    dx2, dw2, _, _ = rmsnorm.rmsnorm_bwd(x, w, dy, rstd)
    assert torch.equal(dw, dw2) and torch.equal(dx, dx2)


def test_baseline_cfg4_full():
    from gpu_ref import bwd_check, fwd_max_err
    x = _gpu_gen((16384, 32, 128), F16, 10).requires_grad_(True)
    w = _gpu_gen((32, 128), F32, 11, "weight").requires_grad_(True)
    b = _gpu_gen((32, 128), F32, 12, "bias").requires_grad_(True)
    dy = _gpu_gen((16384, 32, 128), F16, 13)
    out = rmsnorm.rmsnorm(x, w, b)
    out.backward(dy)
    x2 = x.detach().reshape(-1, 128)
    _, _, rstd = rmsnorm.rmsnorm_fwd(x.detach(), w.detach(), b.detach(), store_rstd=True)
    assert fwd_max_err(x2, w.detach(), b.detach(), None, out.detach().reshape(-1, 128), None, rstd.reshape(-1),
                       1e-6, 2e-3, heads=32) <= 1.0
    dx_err, dw_err = bwd_check(x2, w.detach(), dy.reshape(-1, 128), rstd.reshape(-1), x.grad.reshape(-1, 128),
                               w.grad, 2e-3, heads=32)
    assert dx_err <= 1.0 and dw_err <= 1.0, (dx_err, dw_err)
    db_ref = dy.float().sum(0)
    db_abs = dy.float().abs().sum(0)
    assert ((b.grad - db_ref).abs() <= 1e-3 * db_abs + 1e-6).all()


@pytest.mark.parametrize("dtype", [F32, BF16])
def test_baseline_cfg5_full(dtype):
    from gpu_ref import bwd_check, fwd_max_err
    x = _gpu_gen((1024, 262144), dtype, 14, outliers=0.01)
    w = _gpu_gen((262144,), F32, 15, "weight")
    dy = _gpu_gen((1024, 262144), dtype, 16)
    out, _, rstd = rmsnorm.rmsnorm_fwd(x, w, store_rstd=True)
    tol = oracle.y_tolerance(dtype)
    assert fwd_max_err(x, w, None, None, out, None, rstd, 1e-6, tol, chunk=64) <= 1.0
    dx, dw, _, _ = rmsnorm.rmsnorm_bwd(x, w, dy, rstd)
    dx_err, dw_err = bwd_check(x, w, dy, rstd, dx, dw, tol, chunk=64)
    assert dx_err <= 1.0 and dw_err <= 1.0, (dx_err, dw_err)


@pytest.mark.parametrize("p", [2, 4, 16])
@pytest.mark.parametrize("dtype", [BF16, F32])
def test_split_row_global_exchange(monkeypatch, p, dtype):
    """Split rows whose totals go through tagged records in global memory (groups of P CTAs
    of a cooperative grid) give the same results as the cluster exchange; row counts below,
    at and above the group count of the grid, with and without the exchange lag."""
    monkeypatch.setenv("RMSNORM_B200_XMODE", "1")
    monkeypatch.setenv("RMSNORM_B200_FORCE_CLUSTER", str(p))
    N = 8192 * p if dtype == BF16 else 4096 * p
    for rows, lag in ((3, 1), (70, 1), (301, 0), (301, 1)):
        monkeypatch.setenv("RMSNORM_B200_FORCE_LAG", str(lag))
        plan = _fwd_case(rows, N, dtype, residual="same", bias=True, seed=rows)
        if "fwd_stream" in plan:
            assert f"P={p} x=global" in plan, plan
        plan = _bwd_case(rows, N, dtype, has_bias=(rows == 70), seed=rows + 7)
        if "bwd_stream" in plan and f"P={p}" in plan:
            assert "x=global" in plan, plan
    assert _lib.device_status(DEV) == (0, 0)


@pytest.mark.parametrize("k,lag", [(1, 0), (1, 1), (1, 2), (1, 3), (2, 0), (2, 1), (2, 3), (4, 0), (4, 1)])
@pytest.mark.parametrize("dtype", [BF16, F32])
def test_split_row_pipeline_variants(monkeypatch, k, lag, dtype):
    """Rows split across a cluster stream as K chunks per row slice, with an exchange lag of
    0 to 3 rows; results must not depend on either."""
    import re
    monkeypatch.setenv("RMSNORM_B200_FORCE_K", str(k))
    monkeypatch.setenv("RMSNORM_B200_FORCE_LAG", str(lag))
    p = 4 if dtype == BF16 else 8  # leaves room for two stages of x + residual slices
    monkeypatch.setenv("RMSNORM_B200_FORCE_CLUSTER", str(p))
    N = 65536
    plan = _fwd_case(9, N, dtype, residual="same", bias=True, residual_dtype=F32 if dtype != F32 else None)
    if "fwd_stream" in plan:
        stages = int(re.search(r" S=(\d+)", plan).group(1))
        want_lag = lag
        while want_lag > 0 and stages < (want_lag + 1) * k:
            want_lag -= 1
        assert f"P={p}" in plan and f"K={k} lag={want_lag}" in plan, plan
    for has_bias in (False, True):
        plan = _bwd_case(9, N, dtype, has_bias=has_bias)
        if "bwd_stream" in plan:
            assert "P=" in plan and f"K={k}" in plan, plan


@pytest.mark.parametrize("xmode", ["0", "1"])
@pytest.mark.parametrize("rows,n,dtype", [(1, 65536, BF16), (74, 65536, BF16), (111, 65536, BF16),
                                           (301, 65536, F16), (148, 32768, BF16), (222, 32768, F16),
                                           (1001, 65536, F16), (1, 262144, BF16), (2, 262144, BF16),
                                           (37, 262144, BF16), (300, 131072, F16), (55, 131072, BF16)])
def test_split_row_pairs_match_row_by_row(monkeypatch, xmode, rows, n, dtype):
    """Residual-free forwards with rows split over 2 to 16 CTAs take their rows in pairs (one
    CTA-wide sum, one exchange round and one record poll per two rows; with the global
    exchange warp 0 alone polls). With odd and even row counts per CTA (1, 2, 3 and more),
    cluster and global exchange, out and rstd must equal the row-by-row loop's bit for bit
    and match the oracle."""
    monkeypatch.setenv("RMSNORM_B200_XMODE", xmode)
    x = _g((rows, n), dtype, 400 + rows)
    w = _g((n,), F32, 401, "weight")
    b = _g((n,), F32, 402, "bias")
    out_p, _, rstd_p = rmsnorm.rmsnorm_fwd(x, w, b, None, store_rstd=True)
    torch.cuda.synchronize()
    plan = _lib.last_plan()
    assert "pairs" in plan and ("x=global" in plan) == (xmode == "1"), plan
    monkeypatch.setenv("RMSNORM_B200_XPAIR", "0")
    out_r, _, rstd_r = rmsnorm.rmsnorm_fwd(x, w, b, None, store_rstd=True)
    torch.cuda.synchronize()
    assert "pairs" not in _lib.last_plan(), _lib.last_plan()
    assert torch.equal(out_p.view(torch.int16), out_r.view(torch.int16)), plan
    assert torch.equal(rstd_p, rstd_r), plan
    idx = torch.arange(0, rows, max(1, rows // 16))
    _, _, o_rstd, y = oracle.fwd(x[idx].cpu(), w.cpu(), b.cpu(), None)
    oracle.check_close(out_p[idx], y, dtype, f"pairs out [{plan}]")
    assert torch.allclose(rstd_p[idx].cpu(), o_rstd, rtol=1e-5, atol=0), plan
    assert _lib.device_status(DEV) == (0, 0)


@pytest.mark.parametrize("rows,n,dtype", [(37, 262144, BF16), (300, 65536, F16), (3, 131072, BF16)])
def test_split_row_record_poll_by_one_warp_matches_all_warps(monkeypatch, rows, n, dtype):
    """Global-record exchange with warp 0 alone polling and posting the row total to the
    other warps through shared memory (the default for row slices of at most 32 KB) gives the
    same bits as every warp polling, forward and backward, and matches the oracle."""
    monkeypatch.setenv("RMSNORM_B200_XMODE", "1")
    x = _g((rows, n), dtype, 500 + rows)
    dy = _g((rows, n), dtype, 501 + rows)
    w = _g((n,), F32, 502, "weight")

    def run():
        out, _, rstd = rmsnorm.rmsnorm_fwd(x, w, None, None, store_rstd=True)
        torch.cuda.synchronize()
        pf = _lib.last_plan()
        dx, dw, _, _ = rmsnorm.rmsnorm_bwd(x, w, dy, rstd)
        torch.cuda.synchronize()
        return (out, rstd, dx, dw), pf, _lib.last_plan()

    one, pf1, pb1 = run()
    assert "bcast" in pf1 and "bcast" in pb1, (pf1, pb1)
    monkeypatch.setenv("RMSNORM_B200_XBCAST", "0")
    every, pf0, pb0 = run()
    assert "bcast" not in pf0 and "bcast" not in pb0, (pf0, pb0)
    for a, b in zip(one, every):
        assert torch.equal(a, b), (pf1, pb1)
    idx = torch.arange(0, rows, max(1, rows // 8))
    _, _, o_rstd, y = oracle.fwd(x[idx].cpu(), w.cpu())
    oracle.check_close(one[0][idx], y, dtype, f"out [{pf1}]")
    o_dx, _, _, _, _ = oracle.bwd(x[idx].cpu(), w.cpu(), dy[idx].cpu(), one[1][idx].cpu())
    oracle.check_close(one[2][idx], o_dx, dtype, f"dx [{pb1}]")
    assert _lib.device_status(DEV) == (0, 0)


def test_split_row_global_exchange_concurrent_streams(monkeypatch):
    """Two split-row launches with the global-memory exchange running at the same time on
    two streams (launch epochs pick different record sets) give the same bits as the same
    launches one after the other."""
    monkeypatch.setenv("RMSNORM_B200_XMODE", "1")
    monkeypatch.setenv("RMSNORM_B200_FORCE_CLUSTER", "4")
    n = 32768
    xs = [_g((40, n), BF16, 70 + i) for i in range(2)]
    w = _g((n,), F32, 72, "weight")
    seq = [rmsnorm.rmsnorm_fwd(x, w, store_rstd=True) for x in xs]
    torch.cuda.synchronize()
    assert "x=global" in _lib.last_plan()
    streams = [torch.cuda.Stream() for _ in range(2)]
    outs = [None, None]
    for rep in range(3):
        for i, st in enumerate(streams):
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                outs[i] = rmsnorm.rmsnorm_fwd(xs[i], w, store_rstd=True)
        torch.cuda.synchronize()
        for i in range(2):
            assert torch.equal(outs[i][0], seq[i][0]) and torch.equal(outs[i][2], seq[i][2]), (rep, i)
    assert _lib.device_status(DEV) == (0, 0)


@pytest.mark.parametrize("pipe", ["0", "1"])
@pytest.mark.parametrize("rows,n", [(8192, 4096), (4096, 8192), (2048, 16384)])
def test_row_pipelining_on_and_off(monkeypatch, pipe, rows, n):
    """Row-mode rows with and without the one-tile-deep pipeline (split-phase row-group
    reductions), at sizes with many tiles per CTA so warps drift apart: forward with and
    without residual (rstd checked row by row) and backward."""
    from gpu_ref import bwd_check, fwd_max_err
    monkeypatch.setenv("RMSNORM_B200_PIPE_ROWS", pipe)
    x = _gpu_gen((rows, n), BF16, 80 + n)
    r = _gpu_gen((rows, n), BF16, 81 + n)
    w = _gpu_gen((n,), F32, 82, "weight")
    b = _gpu_gen((n,), F32, 83, "bias")
    out, _, rstd = rmsnorm.rmsnorm_fwd(x, w, store_rstd=True)
    plan = _lib.last_plan()
    assert "mode=row" in plan, plan
    assert fwd_max_err(x, w, None, None, out, None, rstd, 1e-6, 1.6e-2) <= 1.0, plan
    out, ro, rstd = rmsnorm.rmsnorm_fwd(x, w, b, r, residual_dtype=F32, store_rstd=True)
    assert fwd_max_err(x, w, b, r, out, ro, rstd, 1e-6, 1.6e-2) <= 1.0, _lib.last_plan()
    dy = _gpu_gen((rows, n), BF16, 84 + n)
    dx, dw, _, _ = rmsnorm.rmsnorm_bwd(x, w, dy, rstd)
    dx_err, dw_err = bwd_check(x, w, dy, rstd, dx, dw, 1.6e-2, chunk=512)
    assert dx_err <= 1.0 and dw_err <= 1.0, (dx_err, dw_err, _lib.last_plan())
    assert _lib.device_status(DEV) == (0, 0)


@pytest.mark.parametrize("xmode", [None, "1"])
@pytest.mark.parametrize("rows,n,dtype", [(64, 65536, BF16), (24, 262144, BF16), (20, 262144, F32)])
def test_split_row_graph_replay_with_new_inputs(monkeypatch, xmode, rows, n, dtype):
    """Split rows (cfg 3- and cfg 5-shaped: P CTAs per row, by default the global-memory
    exchange on a cooperative grid) captured once into a CUDA graph and replayed three times
    with new inputs written in place between replays. Every replay must match the oracle on
    its own inputs: an exchange record left by the previous replay (same launch parameters)
    is never taken for this one's. Outputs are NaN-filled before each replay."""
    if xmode is not None:
        monkeypatch.setenv("RMSNORM_B200_XMODE", xmode)
    dev = torch.device(DEV)
    x = torch.empty((rows, n), dtype=dtype, device=DEV)
    dy = torch.empty_like(x)
    w = _g((n,), F32, 300, "weight")
    out = torch.empty_like(x)
    rstd = torch.empty(rows, dtype=F32, device=DEV)
    rstd_in = torch.empty(rows, dtype=F32, device=DEV)
    dx = torch.empty_like(x)
    dw = torch.empty(n, dtype=F32, device=DEV)
    args = _lib.bwd_args(x, dy, rstd_in, w, 1, None, dx, None, dw, None, 1, 1)
    ws = torch.empty(max(16, _lib.bwd_workspace_bytes(args, dev)), dtype=torch.uint8, device=DEV)

    def step():
        _lib.fwd(x, None, w, 1, None, 1, out, None, rstd, 1, 1e-6)
        _lib.bwd(args, dev, ws)

    x.copy_(_g((rows, n), dtype, 301))
    dy.copy_(_g((rows, n), dtype, 302))
    step()  # eager warm-up (kernel attributes, plans)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    plan = _lib.last_plan()
    assert "P=1 " not in plan, plan
    if xmode == "1":
        assert "x=global" in plan, plan
    tol = oracle.y_tolerance(dtype)
    for rep in range(3):
        xs = oracle.gen((rows, n), dtype, 310 + rep)
        dys = oracle.gen((rows, n), dtype, 320 + rep)
        _, _, o_rstd, y = oracle.fwd(xs, w.cpu())
        x.copy_(xs.to(DEV))
        dy.copy_(dys.to(DEV))
        rstd_in.copy_(o_rstd.to(DEV))
        for t in (out, dx, dw, rstd):
            t.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        oracle.check_close(out, y, dtype, f"replay {rep} out [{plan}]", rtol=tol)
        assert torch.allclose(rstd.cpu(), o_rstd, rtol=1e-5, atol=0), f"replay {rep} rstd"
        o_dx, o_dw, _, s_dw, _ = oracle.bwd(xs, w.cpu(), dys, o_rstd)
        oracle.check_close(dx, o_dx, dtype, f"replay {rep} dx", rtol=tol)
        oracle.check_reduction(dw, o_dw, s_dw, f"replay {rep} dweight")
    del graph
    assert _lib.device_status(dev) == (0, 0)


@pytest.mark.parametrize("M,N,dtype,dro", [(7, 8192, F32, False), (300, 4096, BF16, True), (33, 12288, F16, False),
                                          (2000, 1024, F16, False), (1, 16384, BF16, True)])
def test_bwd_dbias_sums_in_tmem(monkeypatch, M, N, dtype, dro):
    """dbias backwards whose rows fit one CTA keep the dweight / dbias sums in tensor memory
    (4 vectors per thread, no cluster split): results match the oracle and repeat bitwise;
    the register-accumulator kernel (TMEM off) matches the oracle as well."""
    plan = _bwd_case(M, N, dtype, has_bias=True, dro=dro, seed=400 + M, expect="acc=tmem")
    assert "P=1 " in plan, plan
    monkeypatch.setenv("RMSNORM_B200_TMEM_ACC", "0")
    plan = _bwd_case(M, N, dtype, has_bias=True, dro=dro, seed=400 + M)
    assert "acc=tmem" not in plan, plan
    assert _lib.device_status(DEV) == (0, 0)

# SPDX-License-Identifier: MIT
"""The odd-shape matrix run through the bounds-checked build (librmsnorm_b200_debug.so,
selected with RMSNORM_B200_LIBRARY by tests/test_gpu_debug_bounds.py, which starts this
script as a child process). Every case runs through the public API against the CPU oracle
with the tolerances of the parity tests, with the free device memory NaN-filled first, and
then reads the build's report and the device status word (both cleared after every case):
any failed bounds check or device-side timeout fails the run and names its case. A last case checks
the checker itself: the output tensor of one forward is registered one row short
(RMSNORM_B200_DEBUG_CLIP_OUT), so the kernel's stores to that row -- in bounds of the real
allocation -- must be reported and skipped, leaving the row NaN. Prints one JSON summary
line; exits non-zero on any failure."""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
for p in (str(ROOT), str(ROOT / "rmsnorm-h100_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402

from oracle import rmsnorm_oracle as oracle  # noqa: E402

import rmsnorm  # noqa: E402
from rmsnorm import _lib  # noqa: E402

DEV = torch.device("cuda", 0)
F16, BF16, F32 = torch.float16, torch.bfloat16, torch.float32


def poison():
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    free, _ = torch.cuda.mem_get_info()
    big = torch.empty(min(free // 4, 8 << 30), dtype=torch.uint8, device=DEV)
    big.fill_(0xFF)
    small = [torch.empty((1 << 20) - 512, dtype=torch.uint8, device=DEV).fill_(0xFF) for _ in range(8)]
    torch.cuda.synchronize()
    del big, small


def g(shape, dtype, seed, kind="normal"):
    return oracle.gen(shape, dtype, seed, kind).to(DEV)


def fwd_case(M, N, dtype, *, H=1, residual=None, bias=False, weight=True, seed=0):
    shape = (M // H, H, N) if H > 1 else (M, N)
    x = g(shape, dtype, seed)
    res = None if residual is None else g(shape, F32 if residual == "f32" else dtype, seed + 1)
    aff = (H, N) if H > 1 else (N,)
    w = g(aff, F32, seed + 2, "weight") if weight else None
    b = g(aff, F32, seed + 3, "bias") if bias else None
    out, ro, rstd = rmsnorm.rmsnorm_fwd(x, w, b, res, store_rstd=True)
    torch.cuda.synchronize()
    plan = _lib.last_plan()
    _, o_ro, o_rstd, y = oracle.fwd(x.cpu(), None if w is None else w.cpu(), None if b is None else b.cpu(),
                                    None if res is None else res.cpu())
    oracle.check_close(out, y, dtype, f"out {M}x{N} [{plan}]")
    if o_ro is not None:
        assert torch.equal(ro.cpu(), o_ro), f"residual_out [{plan}]"
    assert torch.allclose(rstd.cpu(), o_rstd, rtol=1e-5, atol=0), f"rstd [{plan}]"
    return plan


def bwd_case(M, N, dtype, *, H=1, has_bias=False, dro=False, weight=True, seed=100):
    shape = (M // H, H, N) if H > 1 else (M, N)
    x = g(shape, dtype, seed)
    dy = g(shape, dtype, seed + 1)
    aff = (H, N) if H > 1 else (N,)
    w = g(aff, F32, seed + 2, "weight") if weight else None
    _, _, rstd, _ = oracle.fwd(x.cpu(), None if w is None else w.cpu())
    rstd = rstd.to(DEV)
    d_ro = g(shape, dtype, seed + 3) if dro else None
    dx, dw, db, _ = rmsnorm.rmsnorm_bwd(x, w, dy, rstd, dresidual_out=d_ro, has_bias=has_bias, has_residual=dro)
    torch.cuda.synchronize()
    plan = _lib.last_plan()
    o_dx, o_dw, o_db, s_dw, s_db = oracle.bwd(x.cpu(), None if w is None else w.cpu(), dy.cpu(), rstd.cpu(),
                                              dresidual_out=d_ro.cpu() if dro else None, has_bias=has_bias)
    oracle.check_close(dx, o_dx, dtype, f"dx {M}x{N} [{plan}]")
    if weight:
        oracle.check_reduction(dw, o_dw, s_dw, f"dweight [{plan}]")
    if has_bias:
        oracle.check_reduction(db, o_db, s_db, f"dbias [{plan}]")
    return plan


def noalloc_case(M, N, dtype, seed=200):
    x = g((M, N), dtype, seed)
    dy = g((M, N), dtype, seed + 1)
    w = g((N,), F32, seed + 2, "weight")
    _, _, rstd, _ = oracle.fwd(x.cpu(), w.cpu())
    rstd = rstd.to(DEV)
    dx = torch.full_like(x, float("nan"))
    dw = torch.full((N,), float("nan"), device=DEV)
    db = torch.full((N,), float("nan"), device=DEV)
    a = _lib.bwd_args(x, dy, rstd, w, 1, None, dx, None, dw, db, 1, 1)
    st = _lib.bwd_noalloc(a, DEV)
    assert st == 0, st
    torch.cuda.synchronize()
    plan = _lib.last_plan()
    o_dx, o_dw, o_db, s_dw, s_db = oracle.bwd(x.cpu(), w.cpu(), dy.cpu(), rstd.cpu(), has_bias=True)
    oracle.check_close(dx, o_dx, dtype, f"noalloc dx [{plan}]")
    oracle.check_reduction(dw, o_dw, s_dw, f"noalloc dweight [{plan}]")
    oracle.check_reduction(db, o_db, s_db, f"noalloc dbias [{plan}]")
    return plan


def ln_case(M, N, dtype, *, bias=True, seed=300):
    x = g((M, N), dtype, seed)
    w = g((N,), F32, seed + 1, "weight")
    b = g((N,), F32, seed + 2, "bias") if bias else None
    out, rstd, mean = rmsnorm.layernorm_fwd(x, w, bias=b, return_rstd=True, return_mean=True)
    torch.cuda.synchronize()
    plan = _lib.last_plan()
    _, r_rstd, r_mean, r_y = oracle.layernorm_fwd(x.cpu(), w.cpu(), None if b is None else b.cpu(), 1e-6)
    oracle.check_close(out, r_y, dtype, f"ln out {M}x{N} [{plan}]")
    assert torch.allclose(rstd.cpu(), r_rstd, rtol=1e-4, atol=0), f"ln rstd [{plan}]"
    return plan


def cases():
    """(label, environment, callable) for the matrix."""
    out = []
    for N in (1, 7, 8, 24, 100, 256, 1001, 4096, 4100, 16384, 32768, 65536, 262144):
        for M, dt in ((1, BF16), (3, F16), (17, F32)):
            if N * M * 4 > (1 << 27):
                continue
            out.append((f"fwd {M}x{N} {dt}", {}, lambda M=M, N=N, dt=dt: fwd_case(M, N, dt)))
    for N, dt, res in ((4096, BF16, "f32"), (16384, BF16, "same"), (65536, F16, "same"), (131072, BF16, "f32")):
        out.append((f"fwd residual {N} {dt}", {}, lambda N=N, dt=dt, res=res: fwd_case(37, N, dt, residual=res, bias=True)))
    for M in (300, 1001, 2000):
        out.append((f"fwd rows {M}", {}, lambda M=M: fwd_case(M, 2048, BF16, bias=True)))
    for H, N, dt, tok in ((32, 128, F16, 37), (32, 128, BF16, 4099), (3, 256, F16, 29), (4, 16, BF16, 50),
                          (128, 128, F16, 5), (8, 64, F32, 45)):
        out.append((f"fwd per-head {H}x{N}", {}, lambda H=H, N=N, dt=dt, tok=tok: fwd_case(tok * H, N, dt, H=H, bias=True)))
    for xm in ("0", "1"):
        for M, N, dt in ((1, 262144, BF16), (37, 262144, BF16), (111, 65536, BF16), (222, 32768, F16),
                         (9, 262144, F32)):
            out.append((f"fwd split {M}x{N} xmode={xm}", {"RMSNORM_B200_XMODE": xm},
                        lambda M=M, N=N, dt=dt: fwd_case(M, N, dt, bias=True)))
    for k in ("2", "4"):
        out.append((f"fwd split K={k}", {"RMSNORM_B200_FORCE_K": k, "RMSNORM_B200_FORCE_CLUSTER": "4"},
                    lambda: fwd_case(9, 65536, BF16, residual="same", bias=True)))
    out.append(("fwd generic forced", {"RMSNORM_B200_FORCE_GENERIC": "1"}, lambda: fwd_case(33, 4096, BF16, residual="f32", bias=True)))
    for N in (7, 256, 4096, 16384, 65536, 262144):
        for M, dt in ((1, BF16), (3, F32), (300, F16)):
            if N * M * 4 > (1 << 27):
                continue
            out.append((f"bwd {M}x{N} {dt}", {}, lambda M=M, N=N, dt=dt: bwd_case(M, N, dt)))
    for N, dt in ((4096, BF16), (8192, F32), (16384, BF16), (32768, F16)):
        out.append((f"bwd dbias dres {N} {dt}", {}, lambda N=N, dt=dt: bwd_case(33, N, dt, has_bias=True, dro=True)))
    out.append(("bwd dbias TMEM off", {"RMSNORM_B200_TMEM_ACC": "0"}, lambda: bwd_case(300, 4096, BF16, has_bias=True)))
    for H, N, dt in ((32, 128, F16), (3, 256, F16), (8, 64, BF16), (8, 512, BF16)):
        out.append((f"bwd per-head {H}x{N}", {}, lambda H=H, N=N, dt=dt: bwd_case(41 * H, N, dt, H=H, has_bias=True)))
    for xm in ("0", "1"):
        out.append((f"bwd split xmode={xm}", {"RMSNORM_B200_XMODE": xm}, lambda: bwd_case(37, 131072, BF16, has_bias=True)))
    out.append(("bwd generic forced", {"RMSNORM_B200_FORCE_GENERIC": "1"}, lambda: bwd_case(33, 4096, BF16, has_bias=True, dro=True)))
    for M, N, dt in ((7, 8192, F32), (4096, 8192, BF16), (300, 4096, BF16)):
        out.append((f"bwd noalloc {M}x{N}", {}, lambda M=M, N=N, dt=dt: noalloc_case(M, N, dt)))
    for M, N, dt, bias in ((4096, 16384, BF16, True), (3001, 1536, BF16, True), (2000, 2560, F32, True),
                           (17, 4100, F16, False), (5, 262144, BF16, True)):
        out.append((f"ln {M}x{N}", {}, lambda M=M, N=N, dt=dt, bias=bias: ln_case(M, N, dt, bias=bias)))
    return out


def clip_selftest():
    """The checker's positive control (see the module docstring)."""
    M, N = 64, 4096
    x = g((M, N), BF16, 900)
    w = g((N,), F32, 901, "weight")
    out = torch.full((M, N), float("nan"), dtype=BF16, device=DEV)
    rstd = torch.full((M,), float("nan"), device=DEV)
    _lib.debug_report(DEV, clear=True)
    os.environ["RMSNORM_B200_DEBUG_CLIP_OUT"] = str(N * 2)
    try:
        _lib.fwd(x, None, w, 1, None, 1, out, None, rstd, 1, 1e-6)
    finally:
        del os.environ["RMSNORM_B200_DEBUG_CLIP_OUT"]
    rep = _lib.debug_report(DEV, clear=True)
    base = out.data_ptr()
    _, _, _, y = oracle.fwd(x[:-1].cpu(), w.cpu())
    rest_ok = True
    try:
        oracle.check_close(out[:-1], y, BF16, "clip: rows before the clipped one")
    except AssertionError:
        rest_ok = False
    return {
        "violations": rep["violations"],
        "site": rep["site"],
        "in_clipped_row": (M - 1) * N * 2 <= rep["address"] - base < M * N * 2,
        "last_row_untouched": bool(torch.isnan(out[-1].float()).all()),
        "rest_ok": rest_ok,
    }


def main() -> int:
    assert _lib.debug_bounds_build(), "RMSNORM_B200_LIBRARY does not name the bounds-checked build"
    _lib.debug_report(DEV, clear=True)
    failures = []
    n = 0
    for label, env, fn in cases():
        poison()
        for k, v in env.items():
            os.environ[k] = v
        try:
            plan = fn()
            rep = _lib.debug_report(DEV, clear=True)
            status = _lib.device_status(DEV, clear=True)
            if rep["violations"] or status[0]:
                failures.append({"case": label, "plan": plan, "report": rep, "device_status": list(status)})
        except Exception as exc:  # noqa: BLE001 -- every failure is reported in the summary
            failures.append({"case": label, "error": f"{type(exc).__name__}: {exc}"[:400],
                             "report": _lib.debug_report(DEV, clear=True),
                             "device_status": list(_lib.device_status(DEV, clear=True))})
        finally:
            for k in env:
                os.environ.pop(k, None)
        n += 1
    status = _lib.device_status(DEV)
    clip = clip_selftest()
    summary = {"cases": n, "failures": failures, "device_status": list(status), "clip": clip}
    print(json.dumps(summary))
    ok = (not failures and status[0] == 0 and clip["violations"] > 0 and clip["site"] == 2
          and clip["in_clipped_row"] and clip["last_row_untouched"] and clip["rest_ok"])
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())

# SPDX-License-Identifier: MIT
"""`torch.compile` keeps the native kernels: the torch.library custom ops
rmsnorm_b200::fwd / ::bwd pass torch.library.opcheck (schema, fake tensors, autograd
registration, AOT dispatch), and compiled modules that call `rmsnorm` (residual, prenorm,
bias, per-head parameters) launch the library's kernels and match the CPU oracle in the
forward and the backward. The reference instead fell back to PyTorch ops while compiling
(rmsnorm/rmsnorm.py:611-614)."""

from __future__ import annotations

import pytest
import torch

from oracle import rmsnorm_oracle as oracle

import rmsnorm
from rmsnorm import _compile  # noqa: F401  (registers the custom ops)
from rmsnorm import _lib

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device"),
]

DEV = "cuda"
F16, BF16, F32 = torch.float16, torch.bfloat16, torch.float32


def _g(shape, dtype, seed, kind="normal"):
    return oracle.gen(shape, dtype, seed, kind).to(DEV)


def test_opcheck_fwd_op():
    x = _g((6, 512), BF16, 1)
    res = _g((6, 512), BF16, 2)
    w = _g((512,), F32, 3, "weight")
    b = _g((512,), F32, 4, "bias")
    for args in [(x, w, b, res, BF16, F32, 1e-6, True),
                 (x, w, None, None, BF16, None, 1e-6, False),
                 (x, w, b, None, F32, None, 1e-6, True),
                 (_g((4, 3, 64), F16, 5), _g((3, 64), F32, 6, "weight"), _g((3, 64), F32, 7, "bias"), None, F16,
                  None, 1e-6, True)]:
        torch.library.opcheck(torch.ops.rmsnorm_b200.fwd.default, args)


def test_opcheck_bwd_op():
    x = _g((6, 512), F32, 11)
    dy = _g((6, 512), BF16, 12)
    w = _g((512,), F32, 13, "weight")
    b = _g((512,), F32, 14, "bias")
    _, _, rstd, _ = oracle.fwd(x.cpu(), w.cpu())
    rstd = rstd.to(DEV)
    dro = _g((6, 512), F32, 15)
    for args in [(x, w, dy, rstd, None, b, True, True, BF16, BF16),
                 (x, w, dy, rstd, dro, None, False, True, BF16, F32),
                 (x, None, dy, rstd, None, None, True, False, F32, None)]:
        torch.library.opcheck(torch.ops.rmsnorm_b200.bwd.default, args)


class _Block(torch.nn.Module):
    def __init__(self, shape, bias=True, prenorm=True):
        super().__init__()
        self.w = torch.nn.Parameter(_g(shape, F32, 21, "weight"))
        self.b = torch.nn.Parameter(_g(shape, F32, 22, "bias")) if bias else None
        self.prenorm = prenorm

    def forward(self, x, res=None):
        if res is None:
            return rmsnorm.rmsnorm(x, self.w, self.b)
        if self.prenorm:
            out, ro = rmsnorm.rmsnorm(x, self.w, self.b, residual=res, residual_dtype=torch.float32, prenorm=True)
            return out, ro
        return rmsnorm.rmsnorm(x, self.w, self.b, residual=res)


def _grads(m, *ts):
    return [t.grad for t in ts] + [m.w.grad] + ([m.b.grad] if m.b is not None else [])


@pytest.mark.parametrize("backend", ["aot_eager", "inductor"])
def test_compiled_prenorm_residual_block_matches_oracle(backend):
    torch._dynamo.reset()
    m = _Block((1024,))
    mc = torch.compile(m, backend=backend, fullgraph=True)
    x = _g((2, 9, 1024), BF16, 30).requires_grad_(True)
    res = _g((2, 9, 1024), BF16, 31).requires_grad_(True)
    dy = _g((2, 9, 1024), BF16, 32)
    dro = _g((2, 9, 1024), F32, 33)
    n0 = _lib.launch_count()
    out, ro = mc(x, res)
    ((out.float() * dy.float()).sum() + (ro * dro).sum()).backward()
    torch.cuda.synchronize()
    assert _lib.launch_count() - n0 >= 3, "the compiled graph did not run the native kernels"
    assert out.dtype == BF16 and ro.dtype == F32 and out.shape == x.shape and ro.shape == x.shape

    xc, rc, w, b = x.detach().cpu(), res.detach().cpu(), m.w.detach().cpu(), m.b.detach().cpu()
    _, o_ro, o_rstd, y = oracle.fwd(xc.reshape(-1, 1024), w, b, rc.reshape(-1, 1024), residual_dtype=F32)
    oracle.check_close(out.reshape(-1, 1024), y, BF16, "compiled out")
    assert torch.equal(ro.detach().cpu().reshape(-1, 1024), o_ro)
    o_dx, o_dw, o_db, s_dw, s_db = oracle.bwd(o_ro, w, dy.cpu().reshape(-1, 1024), o_rstd,
                                              dresidual_out=dro.cpu().reshape(-1, 1024), has_bias=True)
    oracle.check_close(x.grad.reshape(-1, 1024), o_dx, BF16, "compiled dx")
    oracle.check_close(res.grad.reshape(-1, 1024), o_dx, BF16, "compiled dresidual")
    oracle.check_reduction(m.w.grad, o_dw, s_dw, "compiled dweight")
    oracle.check_reduction(m.b.grad, o_db, s_db, "compiled dbias")


def test_compiled_matches_eager_per_head_and_plain():
    torch._dynamo.reset()
    for shape, xshape, dt in [((32, 128), (64, 32, 128), F16), ((2048,), (7, 2048), BF16)]:
        m = _Block(shape, bias=len(shape) == 2)
        mc = torch.compile(m, backend="aot_eager", fullgraph=True)
        x = _g(xshape, dt, 40).requires_grad_(True)
        dy = _g(xshape, dt, 41)
        n0 = _lib.launch_count()
        out = mc(x)
        out.backward(dy)
        torch.cuda.synchronize()
        assert _lib.launch_count() - n0 >= 2
        got = [out.detach()] + _grads(m, x)
        for t in [x] + list(m.parameters()):
            t.grad = None
        out_e = m(x)
        out_e.backward(dy)
        want = [out_e.detach()] + _grads(m, x)
        for a, e in zip(got, want):
            assert torch.equal(a, e), "compiled and eager results differ"
        # and the eager result against the oracle
        h = shape[0] if len(shape) == 2 else 1
        xr = x.detach().cpu()
        _, _, rstd, y = oracle.fwd(xr, m.w.detach().cpu(), m.b.detach().cpu() if m.b is not None else None)
        oracle.check_close(out_e, y, dt, f"eager out {xshape}")
        o_dx, o_dw, _, s_dw, _ = oracle.bwd(xr, m.w.detach().cpu(), dy.cpu(), rstd)
        oracle.check_close(x.grad, o_dx, dt, f"dx {xshape}")
        oracle.check_reduction(m.w.grad, o_dw, s_dw, f"dweight {xshape} (heads {h})")

# SPDX-License-Identifier: MIT
"""The backward entry point that allocates nothing (rmsnorm_b200_bwd_noalloc).

Some callers cannot allocate device memory when they call the backward: a plugin inside a
framework that has reserved all device memory for its own pool, or code that must not
allocate once running. They call this entry point, which keeps the dweight/dbias partial
sums in the library's built-in scratch buffer instead of a caller-provided workspace.

Checked through the C ABI: two calls in a row (the buffer keeps the previous call's
contents) must give the same results as the workspace entry point, within the tolerances
the other tests use; a problem needing more scratch than the buffer holds is refused with
RMSNORM_B200_ERR_SCRATCH_LIMIT before anything runs. The file is named so pytest collects
it last; it also passes alone in a fresh process."""

from __future__ import annotations

import pytest
import torch

from oracle import rmsnorm_oracle as oracle

from rmsnorm import _lib

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]
DEV = torch.device("cuda")


def _problem(rows, n, heads, dtype, seed):
    shape = (rows // heads, heads, n) if heads > 1 else (rows, n)
    aff = (heads, n) if heads > 1 else (n,)
    x = oracle.gen(shape, dtype, seed).to(DEV)
    dy = oracle.gen(shape, dtype, seed + 1).to(DEV)
    w = oracle.gen(aff, torch.float32, seed + 2, "weight").to(DEV)
    rstd = torch.rsqrt(x.float().square().mean(-1) + 1e-6).reshape(-1).contiguous()
    return x, dy, w, rstd


def _outputs(x, w):
    return (torch.full_like(x, float("nan")), torch.full(w.shape, float("nan"), device=DEV),
            torch.full(w.shape, float("nan"), device=DEV))


@pytest.mark.parametrize("rows,n,heads,dtype", [(4096, 8192, 1, torch.bfloat16), (2048, 128, 32, torch.float16),
                                                (64, 65536, 1, torch.bfloat16), (300, 100, 1, torch.float32)])
def test_noalloc_backward_matches_workspace_entry_point(rows, n, heads, dtype):
    x, dy, w, rstd = _problem(rows, n, heads, dtype, 7)
    h = heads
    dx_ref, dw_ref, db_ref = _outputs(x, w)
    a = _lib.bwd_args(x, dy, rstd, w, h, None, dx_ref, None, dw_ref, db_ref, h, h)
    _lib.bwd(a, DEV)  # workspace from the caching allocator
    for call in range(2):  # the scratch buffer keeps the previous call's contents
        dx, dw, db = _outputs(x, w)
        b = _lib.bwd_args(x, dy, rstd, w, h, None, dx, None, dw, db, h, h)
        st = _lib.bwd_noalloc(b, DEV)
        assert st == 0, _lib.load_library().rmsnorm_b200_strerror(st)
        torch.cuda.synchronize()
        oracle.check_close(dx, dx_ref.float(), dtype, f"no-alloc dx, call {call}")
        _, _, _, s_dw, s_db = oracle.bwd(x.cpu(), w.cpu(), dy.cpu(), rstd.cpu().reshape(x.shape[:-1]),
                                         has_bias=True, bias_shape=w.shape)
        oracle.check_reduction(dw, dw_ref, s_dw, f"no-alloc dweight, call {call}")
        oracle.check_reduction(db, db_ref, s_db, f"no-alloc dbias, call {call}")
    assert _lib.device_status(DEV) == (0, 0)


def test_noalloc_refuses_problems_beyond_its_scratch():
    # one very wide row on the generic path: its partial row needs more than the buffer
    n = (_lib_scratch_bytes() // 4) + 9  # odd width -> generic kernels, W * 4 B > buffer
    x = torch.ones(1, n, dtype=torch.bfloat16, device=DEV)
    dy = torch.ones_like(x)
    w = torch.ones(n, device=DEV)
    rstd = torch.ones(1, device=DEV)
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    a = _lib.bwd_args(x, dy, rstd, w, 1, None, dx, None, dw, None, 1, 1)
    assert _lib.bwd_noalloc(a, DEV) == _lib.ERR_SCRATCH_LIMIT
    assert b"scratch" in _lib.load_library().rmsnorm_b200_strerror(_lib.ERR_SCRATCH_LIMIT)


def _lib_scratch_bytes():
    import re
    from pathlib import Path

    hdr = (Path(__file__).resolve().parents[1] / "include" / "rmsnorm_b200.h").read_text()
    m = re.search(r"RMSNORM_B200_NOALLOC_SCRATCH_BYTES \((\d+)u << (\d+)\)", hdr)
    return int(m.group(1)) << int(m.group(2))

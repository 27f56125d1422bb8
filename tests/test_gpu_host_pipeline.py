# SPDX-License-Identifier: MIT
"""The host-buffer pipeline (rmsnorm.host_pipeline) gives the same results as the device
path: the same kernels run on row chunks, copies overlapped on three streams."""

from __future__ import annotations

import pytest
import torch

from oracle import rmsnorm_oracle as oracle

import rmsnorm
from rmsnorm.host_pipeline import HostPipeline

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]
DEV = torch.device("cuda")


@pytest.mark.parametrize("rows,n,chunk", [(1000, 2048, 128), (64, 16384, 64), (7, 512, 3)])
def test_host_pipeline_forward_matches_device_path(rows, n, chunk):
    x = oracle.gen((rows, n), torch.bfloat16, 1).pin_memory()
    res = oracle.gen((rows, n), torch.bfloat16, 2).pin_memory()
    w = oracle.gen((n,), torch.float32, 3, "weight").to(DEV)
    b = oracle.gen((n,), torch.float32, 4, "bias").to(DEV)
    rstd = torch.empty(rows, device=DEV)
    pipe = HostPipeline(DEV, chunk_rows=chunk)
    out, ro = pipe.fwd(x, w, b, res, residual_dtype=torch.float32, rstd=rstd)
    torch.cuda.synchronize()
    d_out, d_ro, d_rstd = rmsnorm.rmsnorm_fwd(x.to(DEV), w, b, res.to(DEV), residual_dtype=torch.float32,
                                              store_rstd=True)
    assert torch.equal(out, d_out.cpu()) and torch.equal(ro, d_ro.cpu())
    assert torch.equal(rstd, d_rstd)


def test_host_pipeline_per_head_forward():
    x = oracle.gen((64 * 32, 128), torch.float16, 5).pin_memory()
    w = oracle.gen((32, 128), torch.float32, 6, "weight").to(DEV)
    b = oracle.gen((32, 128), torch.float32, 7, "bias").to(DEV)
    out, _ = HostPipeline(DEV, chunk_rows=100).fwd(x, w, b)  # chunks round down to 96 = 3 tokens
    torch.cuda.synchronize()
    d_out, _, _ = rmsnorm.rmsnorm_fwd(x.to(DEV).view(64, 32, 128), w, b)
    assert torch.equal(out, d_out.reshape(-1, 128).cpu())


def test_host_pipeline_backward_matches_oracle():
    rows, n = 300, 4096
    x = oracle.gen((rows, n), torch.bfloat16, 8).pin_memory()
    dy = oracle.gen((rows, n), torch.bfloat16, 9).pin_memory()
    w = oracle.gen((n,), torch.float32, 10, "weight").to(DEV)
    _, _, rstd, _ = oracle.fwd(x, w.cpu())
    dx, dw, db = HostPipeline(DEV, chunk_rows=64).bwd(x, w, dy, rstd.to(DEV), has_bias=True)
    torch.cuda.synchronize()
    o_dx, o_dw, o_db, s_dw, s_db = oracle.bwd(x, w.cpu(), dy, rstd, has_bias=True)
    oracle.check_close(dx, o_dx, torch.bfloat16, "pipeline dx")
    oracle.check_reduction(dw, o_dw, s_dw, "pipeline dweight")
    oracle.check_reduction(db, o_db, s_db, "pipeline dbias")

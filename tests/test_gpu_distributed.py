# SPDX-License-Identifier: MIT
"""Row-sharded RMSNorm over 2 GPUs with NCCL (one process per GPU): every rank runs the
kernels on its own rows; the backward's dweight/dbias are combined by one all-reduce.
The result must equal the single-process computation. Skipped with fewer than 2 GPUs."""

from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    for p in (str(ROOT), str(ROOT / "rmsnorm-h100_b200")):
        sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch.distributed as dist

    from oracle import rmsnorm_oracle as oracle
    from rmsnorm import distributed as rd

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        rows, n = 1000, 8192
        x = oracle.gen((rows, n), torch.bfloat16, 1).to(dev)
        res = oracle.gen((rows, n), torch.bfloat16, 2).to(dev)
        dy = oracle.gen((rows, n), torch.bfloat16, 3).to(dev)
        w = oracle.gen((n,), torch.float32, 4, "weight").to(dev)
        b = oracle.gen((n,), torch.float32, 5, "bias").to(dev)
        xs, rs, ds = (rd.shard_rows(t, rank, world) for t in (x, res, dy))
        out, ro, rstd = rd.rmsnorm_fwd_sharded(xs, w, b, rs, residual_dtype=torch.float32, store_rstd=True)
        dx, dw, db, _ = rd.rmsnorm_bwd_sharded(ro, w, ds, rstd, has_bias=True, bias=b)
        torch.cuda.synchronize(dev)
        s, e = rd.row_range(rows, rank, world)
        # numpy arrays travel by value (a tensor's shared-memory handle dies with this process)
        q.put((rank, s, e) + tuple(t.cpu().float().numpy() for t in (out, dx, dw, db)))
    finally:
        dist.destroy_process_group()


def test_two_gpu_row_sharding_matches_single_process():
    import rmsnorm
    from oracle import rmsnorm_oracle as oracle

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted((q.get(timeout=300) for _ in range(world)), key=lambda r: r[0])
    results = [r[:3] + tuple(torch.from_numpy(a) for a in r[3:]) for r in results]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0

    dev = torch.device("cuda", 0)
    rows, n = 1000, 8192
    x = oracle.gen((rows, n), torch.bfloat16, 1).to(dev)
    res = oracle.gen((rows, n), torch.bfloat16, 2).to(dev)
    dy = oracle.gen((rows, n), torch.bfloat16, 3).to(dev)
    w = oracle.gen((n,), torch.float32, 4, "weight").to(dev)
    b = oracle.gen((n,), torch.float32, 5, "bias").to(dev)
    out, ro, rstd = rmsnorm.rmsnorm_fwd(x, w, b, res, residual_dtype=torch.float32, store_rstd=True)
    dx, dw, db, _ = rmsnorm.rmsnorm_bwd(ro, w, dy, rstd, has_bias=True, bias=b)
    _, _, o_db, s_dw, s_db = oracle.bwd(ro.cpu(), w.cpu(), dy.cpu(), rstd.cpu(), has_bias=True)
    for rank, s, e, o, g, gw, gb in results:
        assert torch.equal(o, out[s:e].cpu().float())   # the forward is row-local: bitwise equal
        assert torch.equal(g, dx[s:e].cpu().float())    # so is dx
        oracle.check_reduction(gw, dw.cpu(), s_dw, f"rank {rank} dweight")
        oracle.check_reduction(gb, db.cpu(), s_db, f"rank {rank} dbias")
    assert torch.equal(results[0][5], results[1][5]) and torch.equal(results[0][6], results[1][6])

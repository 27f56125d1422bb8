# SPDX-License-Identifier: MIT
"""Row-sharded RMSNorm over 2 GPUs with NCCL (one process per GPU): every rank runs the
kernels on its own rows; the backward's dweight/dbias are combined by one all-reduce.
Every rank's rows of out / residual_out / dx and the all-reduced dweight / dbias are
checked against the CPU oracle. Skipped with fewer than 2 GPUs."""

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


ROWS, N = 1000, 8192


def _inputs():
    from oracle import rmsnorm_oracle as oracle

    x = oracle.gen((ROWS, N), torch.bfloat16, 1)
    res = oracle.gen((ROWS, N), torch.bfloat16, 2)
    dy = oracle.gen((ROWS, N), torch.bfloat16, 3)
    w = oracle.gen((N,), torch.float32, 4, "weight")
    b = oracle.gen((N,), torch.float32, 5, "bias")
    return x, res, dy, w, b


def _worker(rank, world, port, q, mode="nccl"):
    for p in (str(ROOT), str(ROOT / "rmsnorm-h100_b200")):
        sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch.distributed as dist

    from rmsnorm import distributed as rd

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        x, res, dy, w, b = (t.to(dev) for t in _inputs())
        xs, rs, ds = (rd.shard_rows(t, rank, world) for t in (x, res, dy))
        out, ro, rstd = rd.rmsnorm_fwd_sharded(xs, w, b, rs, residual_dtype=torch.float32, store_rstd=True)
        buf = torch.full((rd.grad_buffer_numel(ro, w, b, True),), float("nan"), device=dev)
        pg = rd.PeerGroup(2 * N) if mode == "peer" else None
        try:
            for _ in range(2):  # two steps in a row (the second reuses the exchange buffers)
                dx, dw, db, _ = rd.rmsnorm_bwd_sharded(ro, w, ds, rstd, has_bias=True, bias=b, grad_buffer=buf,
                                                       peer_group=pg)
            torch.cuda.synchronize(dev)
            if pg is not None:
                from rmsnorm import _lib

                assert _lib.device_status(dev) == (0, 0)
        finally:
            if pg is not None:
                pg.close()
        s, e = rd.row_range(ROWS, rank, world)
        # numpy arrays travel by value (a tensor's shared-memory handle dies with this process)
        q.put((rank, s, e) + tuple(t.cpu().float().numpy() for t in (out, ro, rstd, dx, dw, db)))
    except Exception as exc:  # report to the parent instead of leaving it waiting
        q.put((rank, repr(exc)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["nccl", "peer"])
def test_two_gpu_row_sharding_matches_oracle(mode):
    """mode nccl: dweight / dbias summed by NCCL; mode peer: by the library's fused
    reduction + all-reduce kernel over NVLink peer memory (rmsnorm_b200_bwd_allreduce)."""
    from oracle import rmsnorm_oracle as oracle

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted((q.get(timeout=300) for _ in range(world)), key=lambda r: r[0])
    for r in results:
        assert len(r) > 2, f"rank {r[0]} failed: {r[1]}"
    results = [r[:3] + tuple(torch.from_numpy(a) for a in r[3:]) for r in results]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0

    x, res, dy, w, b = _inputs()
    _, o_ro, o_rstd, y = oracle.fwd(x, w, b, res, residual_dtype=torch.float32)
    o_dx, o_dw, o_db, s_dw, s_db = oracle.bwd(o_ro, w, dy, o_rstd, has_bias=True)
    covered = 0
    for rank, s, e, out, ro, rstd, dx, dw, db in results:
        oracle.check_close(out, y[s:e], torch.bfloat16, f"rank {rank} out")
        assert torch.equal(ro, o_ro[s:e]), f"rank {rank} residual_out"
        assert torch.allclose(rstd, o_rstd[s:e], rtol=1e-5, atol=0), f"rank {rank} rstd"
        oracle.check_close(dx, o_dx[s:e], torch.bfloat16, f"rank {rank} dx")
        oracle.check_reduction(dw, o_dw, s_dw, f"rank {rank} dweight (all-reduced)")
        oracle.check_reduction(db, o_db, s_db, f"rank {rank} dbias (all-reduced)")
        covered += e - s
    assert covered == ROWS
    # every rank holds the same bits of the all-reduced gradients
    assert torch.equal(results[0][7], results[1][7]) and torch.equal(results[0][8], results[1][8])

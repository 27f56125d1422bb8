# SPDX-License-Identifier: MIT
"""Multi-rank host logic on CPU (gloo, world_size 2): row sharding, the single all-reduce
of dweight/dbias in the backward, uneven row splits, and failure detection on the host
(a rank that leaves before the collective makes the other rank's collective end with an
error after a short process-group timeout, instead of waiting forever)."""

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


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank, world, port, timeout_s=30):
    for p in (str(ROOT), str(ROOT / "rmsnorm-h100_b200"), str(ROOT / "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))
    return dist


def _sharded_worker(rank, world, port, rows, n, heads, result_q):
    dist = _setup(rank, world, port)
    from oracle import rmsnorm_oracle as oracle

    from rmsnorm import distributed as rd

    try:
        aff = (heads, n) if heads > 1 else (n,)
        shape = (rows, heads, n) if heads > 1 else (rows, n)
        x = oracle.gen(shape, torch.float32, 1)
        dy = oracle.gen(shape, torch.float32, 2)
        w = oracle.gen(aff, torch.float32, 3, "weight")
        b = oracle.gen(aff, torch.float32, 4, "bias")
        xs = rd.shard_rows(x, rank, world)
        ys = rd.shard_rows(dy, rank, world)
        out, _, rstd = rd.rmsnorm_fwd_sharded(xs, w, b, store_rstd=True)
        dx, dw, db, _ = rd.rmsnorm_bwd_sharded(xs, w, ys, rstd, has_bias=True, bias=b)
        s, e = rd.row_range(rows, rank, world)
        # numpy arrays travel by value: a tensor would be handed over through a shared-memory
        # handle that disappears when this process exits before the parent unpickles it
        result_q.put((rank, s, e) + tuple(t.numpy() for t in (out, dx, dw, db)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("rows,n,heads", [(8, 64, 1), (7, 32, 1), (6, 16, 3)])
def test_row_sharded_fwd_bwd_equals_single_process(rows, n, heads):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, world, port, rows, n, heads, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    results = [r[:3] + tuple(torch.from_numpy(a) for a in r[3:]) for r in results]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0

    import rmsnorm
    from oracle import rmsnorm_oracle as oracle

    aff = (heads, n) if heads > 1 else (n,)
    shape = (rows, heads, n) if heads > 1 else (rows, n)
    x = oracle.gen(shape, torch.float32, 1)
    dy = oracle.gen(shape, torch.float32, 2)
    w = oracle.gen(aff, torch.float32, 3, "weight")
    b = oracle.gen(aff, torch.float32, 4, "bias")
    out, _, rstd = rmsnorm.rmsnorm_fwd(x, w, b, store_rstd=True)
    dx, dw, db, _ = rmsnorm.rmsnorm_bwd(x, w, dy, rstd, has_bias=True, bias=b)
    covered = 0
    for rank, s, e, o, g, gw, gb in sorted(results, key=lambda r: r[0]):
        assert torch.equal(o, out[s:e]) and torch.equal(g, dx[s:e])
        # every rank ends with the same all-reduced sums, equal to the single-process ones
        assert torch.allclose(gw, dw, rtol=1e-5, atol=1e-5)
        assert torch.allclose(gb, db, rtol=1e-5, atol=1e-5)
        covered += e - s
    assert covered == rows
    assert torch.equal(results[0][5], results[1][5])  # identical on both ranks


def test_row_range_is_an_even_partition():
    from rmsnorm.distributed import row_range

    for rows in (0, 1, 7, 8, 32768):
        for world in (1, 2, 4, 8):
            spans = [row_range(rows, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == rows
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1


def _failing_worker(rank, world, port, result_q):
    dist = _setup(rank, world, port, timeout_s=3)
    from rmsnorm.distributed import allreduce_sum_

    if rank == 1:
        os._exit(3)  # this rank dies before the collective
    t = torch.ones(4)
    try:
        allreduce_sum_([t])
        result_q.put(("no error", rank))
    except Exception as exc:  # the collective ends with an error after the timeout
        result_q.put(("error", type(exc).__name__))


def test_dead_rank_makes_collective_fail_not_hang():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    status, what = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert status == "error", what
    assert procs[1].exitcode == 3

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


_DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _inputs(rows, n, heads, xdt, wdt):
    from oracle import rmsnorm_oracle as oracle

    aff = (heads, n) if heads > 1 else (n,)
    shape = (rows, heads, n) if heads > 1 else (rows, n)
    x = oracle.gen(shape, _DT[xdt], 1)
    dy = oracle.gen(shape, _DT[xdt], 2)
    w = oracle.gen(aff, _DT[wdt], 3, "weight")
    b = oracle.gen(aff, _DT[wdt], 4, "bias")
    return x, dy, w, b


def _sharded_worker(rank, world, port, rows, n, heads, xdt, wdt, result_q):
    dist = _setup(rank, world, port)
    from rmsnorm import distributed as rd

    try:
        x, dy, w, b = _inputs(rows, n, heads, xdt, wdt)
        xs = rd.shard_rows(x, rank, world)
        ys = rd.shard_rows(dy, rank, world)
        out, _, rstd = rd.rmsnorm_fwd_sharded(xs, w, b, store_rstd=True)
        buf = torch.empty(rd.grad_buffer_numel(xs, w, b, True), dtype=torch.float32)
        dx, dw, db, _ = rd.rmsnorm_bwd_sharded(xs, w, ys, rstd, has_bias=True, bias=b, grad_buffer=buf)
        assert dw.dtype == w.dtype and db.dtype == b.dtype
        s, e = rd.row_range(rows, rank, world)
        # numpy arrays travel by value: a tensor would be handed over through a shared-memory
        # handle that disappears when this process exits before the parent unpickles it
        result_q.put((rank, s, e) + tuple(t.float().numpy() for t in (out, dx, dw, db)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("rows,n,heads,xdt,wdt", [(8, 64, 1, "f32", "f32"), (7, 32, 1, "f32", "f32"),
                                                  (6, 16, 3, "f32", "f32"), (9, 256, 1, "bf16", "bf16"),
                                                  (10, 128, 1, "f16", "f32")])
def test_row_sharded_fwd_bwd_matches_oracle(rows, n, heads, xdt, wdt):
    """Every rank's rows of out / dx match the oracle; every rank ends with the same
    dweight / dbias, equal to the oracle's fp32 sums over all rows within the task's
    tolerance (bf16 weights: summed in fp32 across ranks, rounded once)."""
    from oracle import rmsnorm_oracle as oracle

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, world, port, rows, n, heads, xdt, wdt, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    results = [r[:3] + tuple(torch.from_numpy(a) for a in r[3:]) for r in results]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0

    x, dy, w, b = _inputs(rows, n, heads, xdt, wdt)
    o_out, _, o_rstd, y = oracle.fwd(x, w, b)
    o_dx, o_dw, o_db, s_dw, s_db = oracle.bwd(x, w, dy, o_rstd, has_bias=True, bias_shape=b.shape)
    covered = 0
    for rank, s, e, o, g, gw, gb in sorted(results, key=lambda r: r[0]):
        oracle.check_close(o, y[s:e], _DT[xdt], f"rank {rank} out")
        oracle.check_close(g, o_dx[s:e], _DT[xdt], f"rank {rank} dx")
        oracle.check_reduction(gw.to(_DT[wdt]), o_dw, s_dw, f"rank {rank} dweight")
        oracle.check_reduction(gb.to(_DT[wdt]), o_db, s_db, f"rank {rank} dbias")
        covered += e - s
    assert covered == rows
    assert torch.equal(results[0][5], results[1][5]) and torch.equal(results[0][6], results[1][6])


def test_allreduce_sum_packs_mixed_dtypes():
    """allreduce_sum_ with one rank on CPU (world 1 group of gloo) leaves the values and
    dtypes of mixed-dtype tensors intact."""
    world = 1
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_pack_worker, args=(0, world, _free_port(), q))
    p.start()
    ok = q.get(timeout=120)
    p.join(timeout=60)
    assert ok == "ok", ok


def _pack_worker(rank, world, port, q):
    dist = _setup(rank, world, port)
    try:
        from rmsnorm.distributed import allreduce_sum_

        a = torch.arange(6, dtype=torch.float32).view(2, 3)
        b = torch.tensor([0.5, 1.5], dtype=torch.bfloat16)
        a0, b0 = a.clone(), b.clone()
        allreduce_sum_([a, None, b])
        q.put("ok" if torch.equal(a, a0) and torch.equal(b, b0) and b.dtype == torch.bfloat16 else "changed")
    except Exception as exc:  # report, do not hang the parent
        q.put(repr(exc))
    finally:
        dist.destroy_process_group()


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

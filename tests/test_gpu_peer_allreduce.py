# SPDX-License-Identifier: MIT
"""The backward's fused reduction + all-reduce over peer memory (rmsnorm_b200_bwd_allreduce)
on one GPU: a one-rank group gives the same dx as the plain backward and dweight / dbias
within the task's tolerance of the oracle, repeatably and across CUDA-graph replays; and
the failure-detection self test: a two-rank group whose second rank never runs makes the
waiting kernel give up after the peer timeout, record the timeout in the device status
word and return, leaving the context usable. (Two ranks that wait on each other never run
on one GPU: tests/test_gpu_distributed.py runs them on two.)"""

from __future__ import annotations

import pytest
import torch

from oracle import rmsnorm_oracle as oracle

from rmsnorm import _lib

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device"),
]

DEV = torch.device("cuda", 0)
BF16, F32 = torch.bfloat16, torch.float32


def _case(rows, n, dt, seed):
    x = oracle.gen((rows, n), dt, seed).to(DEV)
    dy = oracle.gen((rows, n), dt, seed + 1).to(DEV)
    w = oracle.gen((n,), F32, seed + 2, "weight").to(DEV)
    _, _, rstd, _ = oracle.fwd(x.cpu(), w.cpu())
    return x, dy, w, rstd.to(DEV)


@pytest.mark.parametrize("rows,n,dt", [(300, 16384, BF16), (7, 4096, F32), (2000, 1024, BF16), (0, 2048, BF16)])
def test_one_rank_group_matches_plain_backward_and_oracle(rows, n, dt):
    torch.cuda.set_device(DEV)
    handle, _ = _lib.peer_group_create(DEV, 0, 1, 2 * n)
    try:
        _lib.peer_group_connect_buffers(DEV, handle, [None])
        x, dy, w, rstd = _case(rows, n, dt, 10 + rows)
        outs = []
        for use_peer in (False, True, True):  # two calls in a row through the group
            dx = torch.empty_like(x)
            dw = torch.full((n,), float("nan"), device=DEV)
            db = torch.full((n,), float("nan"), device=DEV)
            a = _lib.bwd_args(x, dy, rstd, w, 1, None, dx, None, dw, db, 1, 1)
            _lib.bwd(a, DEV, peer_group=handle if use_peer else None)
            torch.cuda.synchronize()
            if use_peer:
                assert "allreduce=peer world=1" in _lib.last_plan(), _lib.last_plan()
            outs.append((dx, dw, db))
        assert torch.equal(outs[0][0], outs[1][0])
        assert torch.equal(outs[1][1], outs[2][1]) and torch.equal(outs[1][2], outs[2][2])
        o_dx, o_dw, o_db, s_dw, s_db = oracle.bwd(x.cpu(), w.cpu(), dy.cpu(), rstd.cpu(), has_bias=True)
        oracle.check_reduction(outs[1][1], o_dw, s_dw, "peer dweight")
        oracle.check_reduction(outs[1][2], o_db, s_db, "peer dbias")
        assert _lib.device_status(DEV) == (0, 0)
    finally:
        _lib.peer_group_destroy(DEV, handle)


def test_one_rank_group_in_a_cuda_graph():
    """The call counter lives on the device: graph replays draw new tags and parities."""
    torch.cuda.set_device(DEV)
    n = 8192
    handle, _ = _lib.peer_group_create(DEV, 0, 1, 2 * n)
    try:
        _lib.peer_group_connect_buffers(DEV, handle, [None])
        x, dy, w, rstd = _case(64, n, BF16, 50)
        dx = torch.empty_like(x)
        dw = torch.empty(n, device=DEV)
        db = torch.empty(n, device=DEV)
        a = _lib.bwd_args(x, dy, rstd, w, 1, None, dx, None, dw, db, 1, 1)
        ws = torch.empty(max(16, _lib.bwd_workspace_bytes(a, DEV)), dtype=torch.uint8, device=DEV)
        _lib.bwd(a, DEV, ws, peer_group=handle)
        torch.cuda.synchronize()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            _lib.bwd(a, DEV, ws, peer_group=handle)
        torch.cuda.current_stream().wait_stream(side)
        for rep in range(3):
            xs = oracle.gen((64, n), BF16, 60 + rep)
            x.copy_(xs.to(DEV))
            _, _, r, _ = oracle.fwd(xs, w.cpu())
            rstd.copy_(r.to(DEV))
            dw.fill_(float("nan"))
            db.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
            _, o_dw, o_db, s_dw, s_db = oracle.bwd(xs, w.cpu(), dy.cpu(), r, has_bias=True)
            oracle.check_reduction(dw, o_dw, s_dw, f"replay {rep} dweight")
            oracle.check_reduction(db, o_db, s_db, f"replay {rep} dbias")
        del g
        assert _lib.device_status(DEV) == (0, 0)
    finally:
        _lib.peer_group_destroy(DEV, handle)


def test_missing_peer_times_out_without_faulting():
    """Rank 0 of a two-rank group runs alone: its kernel waits for rank 1's values, which
    never come, gives up after the (shortened) peer timeout, records the timeout at the
    peer site and returns; the context keeps working."""
    torch.cuda.set_device(DEV)
    n = 1024
    assert _lib.device_status(DEV, clear=True) == (0, 0)
    h0, _ = _lib.peer_group_create(DEV, 0, 2, 2 * n)
    h1, _ = _lib.peer_group_create(DEV, 1, 2, 2 * n)  # rank 1's buffer only: rank 1 never runs
    try:
        _lib.peer_group_connect_buffers(DEV, h0, [None, _lib.peer_group_buffer(h1)])
        _lib.set_peer_timeout_ns(DEV, 20_000_000)  # 20 ms
        x, dy, w, rstd = _case(16, n, BF16, 70)
        dx = torch.empty_like(x)
        dw = torch.empty(n, device=DEV)
        a = _lib.bwd_args(x, dy, rstd, w, 1, None, dx, None, dw, None, 1, 1)
        _lib.bwd(a, DEV, peer_group=h0)
        torch.cuda.synchronize()
        st, where = _lib.device_status(DEV, clear=True)
        assert st == _lib.ERR_DEVICE_TIMEOUT and where == 9, (st, where)
        assert _lib.device_status(DEV) == (0, 0)
        # still usable: a plain backward afterwards is correct
        db = torch.empty(n, device=DEV)
        a = _lib.bwd_args(x, dy, rstd, w, 1, None, dx, None, dw, db, 1, 1)
        _lib.bwd(a, DEV)
        torch.cuda.synchronize()
        o_dx, o_dw, _, s_dw, _ = oracle.bwd(x.cpu(), w.cpu(), dy.cpu(), rstd.cpu())
        oracle.check_close(dx, o_dx, BF16, "dx after the timeout")
        oracle.check_reduction(dw, o_dw, s_dw, "dweight after the timeout")
    finally:
        _lib.set_peer_timeout_ns(DEV, 10_000_000_000)
        _lib.peer_group_destroy(DEV, h0)
        _lib.peer_group_destroy(DEV, h1)


def test_group_argument_checks():
    torch.cuda.set_device(DEV)
    lib = _lib.load_library()
    import ctypes

    h = ctypes.c_void_p()
    ipc = ctypes.create_string_buffer(64)
    assert lib.rmsnorm_b200_peer_group_create(2, 2, 16, ipc, ctypes.byref(h)) == 1   # rank >= world
    assert lib.rmsnorm_b200_peer_group_create(0, 9, 16, ipc, ctypes.byref(h)) == 1   # more than 8 ranks
    assert lib.rmsnorm_b200_peer_group_create(0, 2, 0, ipc, ctypes.byref(h)) == 1    # no room
    handle, _ = _lib.peer_group_create(DEV, 0, 1, 100)
    try:
        x, dy, w, rstd = _case(4, 512, BF16, 80)
        dx = torch.empty_like(x)
        dw = torch.empty(512, device=DEV)
        a = _lib.bwd_args(x, dy, rstd, w, 1, None, dx, None, dw, None, 1, 1)
        n0 = _lib.launch_count()
        with pytest.raises(_lib.LibraryError):  # not connected yet: refused before any launch
            _lib.bwd(a, DEV, peer_group=handle)
        _lib.peer_group_connect_buffers(DEV, handle, [None])
        with pytest.raises(_lib.LibraryError):  # 512 gradient values do not fit a 100-value group
            _lib.bwd(a, DEV, peer_group=handle)
        assert _lib.launch_count() == n0
    finally:
        _lib.peer_group_destroy(DEV, handle)

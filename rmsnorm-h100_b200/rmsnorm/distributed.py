# SPDX-License-Identifier: MIT
"""Row-sharded data parallelism for RMSNorm over the GPUs of one node.

Rows are independent in both directions, so every rank owns a contiguous block of rows
and runs the kernels on it with no communication. The only exchange is in the backward:
the per-rank dweight / dbias sums are combined with ONE all-reduce (sum, fp32) over
NVLink / NVSwitch -- either NCCL's, or, with a `PeerGroup`, the library's own kernel that
fuses the backward's final reduction with the all-reduce over peer memory (every rank
pushes its column sums to every rank and sums them in rank order: identical bits on every
rank). The reference is single-GPU and has no counterpart to this module.

The backward writes its fp32 dweight / dbias sums straight into one packed fp32 buffer
[dweight | dbias]; the all-reduce sums that buffer in place and each gradient is rounded
once, afterwards, to its parameter's dtype. (Reducing bf16 / fp16 gradients would round
every rank's partial sum before the cross-rank sum and again after it.)
"""

from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from .rmsnorm import _grad_layout, _rmsnorm_bwd_fp32_grads, rmsnorm_fwd


def row_range(rows: int, rank: int, world: int) -> tuple:
    """[start, stop) of the rows rank `rank` owns: an even split, the first `rows % world`
    ranks taking one extra row."""
    base, extra = divmod(rows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_rows(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's rows of t (split along dim 0), as a view."""
    s, e = row_range(t.shape[0], rank, world)
    return t[s:e]


def allreduce_sum_(tensors: Sequence[Optional[torch.Tensor]], group=None) -> None:
    """Sums the given tensors across ranks in place with a single all_reduce. Several
    tensors, or tensors that are not contiguous fp32, go through one packed fp32 buffer
    (one collective, one latency, one rounding back to each tensor's dtype)."""
    ts: List[torch.Tensor] = [t for t in tensors if t is not None]
    if not ts:
        return
    if len(ts) == 1 and ts[0].dtype == torch.float32 and ts[0].is_contiguous():
        dist.all_reduce(ts[0], op=dist.ReduceOp.SUM, group=group)
        return
    flat = torch.empty(sum(t.numel() for t in ts), dtype=torch.float32, device=ts[0].device)
    off = 0
    for t in ts:
        flat[off : off + t.numel()].view(t.shape).copy_(t)
        off += t.numel()
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    off = 0
    for t in ts:
        t.copy_(flat[off : off + t.numel()].view(t.shape))
        off += t.numel()


def grad_buffer_numel(x: torch.Tensor, weight: Optional[torch.Tensor], bias: Optional[torch.Tensor] = None,
                      has_bias: bool = False) -> int:
    """fp32 elements of the packed [dweight | dbias] buffer of a backward with these
    arguments (x: this rank's rows; only its shape matters)."""
    dw_shape, db_shape = _grad_layout(x, weight, bias, has_bias)
    n = 0
    for s in (dw_shape, db_shape):
        if s is not None:
            n += int(torch.Size(s).numel())
    return n


class PeerGroup:
    """The library's peer-memory all-reduce for the backward's dweight / dbias, set up over
    a process group whose ranks are the GPUs of one node (one process per GPU, the current
    CUDA device of each). Each rank allocates one exchange buffer at set-up (room for
    `max_grad_floats` gradient values: dweight + dbias elements); the CUDA IPC handles are
    exchanged once with an all-gather. Every rank must then make the same sequence of
    backward calls with the same gradient shapes. close() (or the owner's exit) frees it."""

    def __init__(self, max_grad_floats: int, group=None, device: Optional[torch.device] = None):
        from . import _lib

        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.max_grad_floats = int(max_grad_floats)
        self.handle, ipc = _lib.peer_group_create(self.device, self.rank, self.world, self.max_grad_floats)
        handles: List[Optional[bytes]] = [None] * self.world
        dist.all_gather_object(handles, ipc, group=group)
        _lib.peer_group_connect(self.device, self.handle, handles)
        # every rank has mapped its peers before any rank pushes into them
        dist.barrier(group=group)

    def close(self) -> None:
        from . import _lib

        if self.handle is not None:
            torch.cuda.synchronize(self.device)
            _lib.peer_group_destroy(self.device, self.handle)
            self.handle = None


def rmsnorm_fwd_sharded(x_shard, weight=None, bias=None, residual_shard=None, **kw):
    """Forward on this rank's rows: no communication."""
    return rmsnorm_fwd(x_shard, weight, bias, residual_shard, **kw)


def rmsnorm_bwd_sharded(
    x_shard: torch.Tensor,
    weight: Optional[torch.Tensor],
    dout_shard: torch.Tensor,
    rstd_shard: torch.Tensor,
    dresidual_out_shard: Optional[torch.Tensor] = None,
    has_bias: bool = False,
    has_residual: bool = False,
    bias: Optional[torch.Tensor] = None,
    group=None,
    grad_buffer: Optional[torch.Tensor] = None,
    peer_group: Optional[PeerGroup] = None,
) -> Tuple[torch.Tensor, Optional[torch.Tensor], Optional[torch.Tensor], Optional[torch.Tensor]]:
    """Backward on this rank's rows, then one all-reduce of dweight (+ dbias): NCCL's over
    `group`, or, with `peer_group` (CUDA tensors), the library's fused kernel.

    Returns (dx, dweight, dbias, dresidual) like rmsnorm_bwd: dx and dresidual stay
    sharded, dweight / dbias are the sums over every rank's rows in the affine dtypes (the
    same values on every rank). `grad_buffer`: a contiguous fp32 tensor of at least
    grad_buffer_numel(...) elements on x's device, reused across calls to avoid an
    allocation per step; an fp32 dweight / dbias is then returned as a view of it, valid
    until the buffer's next use. The all-reduce runs on the current stream."""
    dw_shape, db_shape = _grad_layout(x_shard, weight, bias, has_bias)
    nw = int(torch.Size(dw_shape).numel()) if dw_shape is not None else 0
    nb = int(torch.Size(db_shape).numel()) if db_shape is not None else 0
    if grad_buffer is None:
        grad_buffer = torch.empty(nw + nb, dtype=torch.float32, device=x_shard.device)
    elif grad_buffer.dtype != torch.float32 or not grad_buffer.is_contiguous() or grad_buffer.numel() < nw + nb:
        raise ValueError(f"grad_buffer must be a contiguous float32 tensor of at least {nw + nb} elements")
    buf = grad_buffer.reshape(-1)[: nw + nb]
    dw32 = buf[:nw].view(dw_shape) if dw_shape is not None else None
    db32 = buf[nw:].view(db_shape) if db_shape is not None else None
    use_peer = peer_group is not None and x_shard.is_cuda
    dx, dres = _rmsnorm_bwd_fp32_grads(x_shard, weight, dout_shard, rstd_shard, dresidual_out_shard, has_bias,
                                       has_residual, bias, dw32, db32,
                                       peer_group=peer_group.handle if use_peer else None)
    if (not use_peer and nw + nb and dist.is_available() and dist.is_initialized()
            and dist.get_world_size(group) > 1):
        dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
    dw = db = None
    if dw32 is not None:
        dw = dw32 if weight.dtype == torch.float32 else dw32.to(weight.dtype)
    if db32 is not None:
        db_dtype = bias.dtype if bias is not None else (weight.dtype if weight is not None else x_shard.dtype)
        db = db32 if db_dtype == torch.float32 else db32.to(db_dtype)
    return dx, dw, db, dres

# SPDX-License-Identifier: MIT
"""Row-sharded data parallelism for RMSNorm over the GPUs of one node.

Rows are independent in both directions, so every rank owns a contiguous block of rows
and runs the kernels on it with no communication. The only exchange is in the backward:
the per-rank dweight / dbias sums are combined with ONE all-reduce (sum, fp32) over NCCL
(NVLink / NVSwitch). The reference is single-GPU and has no counterpart to this module.
"""

from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from .rmsnorm import rmsnorm_bwd, rmsnorm_fwd


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
    """Sums the given tensors across ranks in place with a single all_reduce: several
    tensors are packed into one fp32 buffer first (one collective, one latency)."""
    ts: List[torch.Tensor] = [t for t in tensors if t is not None]
    if not ts:
        return
    if len(ts) == 1 and ts[0].dtype == torch.float32 and ts[0].is_contiguous():
        dist.all_reduce(ts[0], op=dist.ReduceOp.SUM, group=group)
        return
    flat = torch.cat([t.reshape(-1).float() for t in ts])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    off = 0
    for t in ts:
        n = t.numel()
        t.copy_(flat[off : off + n].view(t.shape))
        off += n


def rmsnorm_fwd_sharded(x_shard, weight=None, bias=None, residual_shard=None, **kw):
    """Forward on this rank's rows: no communication."""
    return rmsnorm_fwd(x_shard, weight, bias, residual_shard, **kw)


def rmsnorm_bwd_sharded(x_shard, weight, dout_shard, rstd_shard, dresidual_out_shard=None,
                        has_bias=False, has_residual=False, bias=None, group=None):
    """Backward on this rank's rows, then one all-reduce of dweight (+ dbias). dx and
    dresidual stay sharded. dweight / dbias must be fp32 for an exact sum order per rank
    (they are when the affine parameters are fp32)."""
    dx, dw, db, dres = rmsnorm_bwd(x_shard, weight, dout_shard, rstd_shard, dresidual_out_shard,
                                   has_bias, has_residual, bias)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        allreduce_sum_([dw, db], group=group)
    return dx, dw, db, dres

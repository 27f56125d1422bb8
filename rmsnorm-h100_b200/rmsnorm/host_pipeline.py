# SPDX-License-Identifier: MIT
"""RMSNorm on host-resident (pinned) tensors, streamed through the GPU.

Callers that keep activations in host memory (offloading, CPU-side data pipelines) would
otherwise pay copy-in, kernel and copy-out back to back. `HostPipeline` cuts the rows into
chunks and runs, for consecutive chunks, the host->device copy, the kernel and the
device->host copy concurrently on three CUDA streams: the two copy directions use separate
copy engines, so a step costs about max(bytes in, bytes out) / link bandwidth instead of
their sum. Device staging buffers are allocated once per pipeline (rotating `depth` sets);
the kernels are the same library calls as `rmsnorm_fwd` / `rmsnorm_bwd`.
"""

from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from . import _lib


class HostPipeline:
    def __init__(self, device: torch.device, chunk_rows: int = 1024, depth: int = 3):
        self.device = torch.device(device)
        self.chunk_rows = int(chunk_rows)
        self.depth = int(depth)
        self.h2d = torch.cuda.Stream(self.device)
        self.comp = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)
        self._bufs: Dict[Tuple, list] = {}
        self._ws: Optional[torch.Tensor] = None

    def _staging(self, key, specs):
        """`depth` sets of device buffers, one per spec (name -> (shape, dtype))."""
        if key not in self._bufs:
            self._bufs[key] = [
                {n: torch.empty(shape, dtype=dt, device=self.device) for n, (shape, dt) in specs.items()}
                for _ in range(self.depth)
            ]
        return self._bufs[key]

    def _run(self, rows, ins: Dict[str, torch.Tensor], outs: Dict[str, torch.Tensor], launch, multiple=1,
             scratch: Optional[Dict[str, Tuple[tuple, torch.dtype]]] = None):
        """Generic chunk loop: copy `ins` rows in, call launch(buffer_set, nrows) on the
        compute stream, copy `outs` rows back. Chunks hold a multiple of `multiple` rows.
        `scratch` (name -> (trailing shape, dtype)) adds device-only buffers of `chunk` rows
        to every buffer set (intermediates that never leave the device)."""
        cur = torch.cuda.current_stream(self.device)
        n = ins[next(iter(ins))].shape[-1]
        chunk = max(multiple, self.chunk_rows - self.chunk_rows % multiple)
        specs = {k: ((chunk, n), v.dtype) for k, v in {**ins, **outs}.items()}
        for k, (tail, dt) in (scratch or {}).items():
            specs[k] = ((chunk, *tail), dt)
        bufs = self._staging(("rows", n, tuple(sorted((k, str(v[1])) for k, v in specs.items()))), specs)
        h2d_done = [torch.cuda.Event() for _ in range(self.depth)]
        comp_done = [torch.cuda.Event() for _ in range(self.depth)]
        d2h_done = [torch.cuda.Event() for _ in range(self.depth)]
        self.h2d.wait_stream(cur)
        self.comp.wait_stream(cur)
        self.d2h.wait_stream(cur)
        for c, s in enumerate(range(0, rows, chunk)):
            e = min(rows, s + chunk)
            b = c % self.depth
            buf = bufs[b]
            if c >= self.depth:
                self.h2d.wait_event(d2h_done[b])  # this buffer set's last results are home
            with torch.cuda.stream(self.h2d):
                for k, v in ins.items():
                    buf[k][: e - s].copy_(v[s:e], non_blocking=True)
                h2d_done[b].record(self.h2d)
            self.comp.wait_event(h2d_done[b])
            with torch.cuda.stream(self.comp):
                launch(buf, e - s)
                comp_done[b].record(self.comp)
            self.d2h.wait_event(comp_done[b])
            with torch.cuda.stream(self.d2h):
                for k, v in outs.items():
                    v[s:e].copy_(buf[k][: e - s], non_blocking=True)
                d2h_done[b].record(self.d2h)
        cur.wait_stream(self.d2h)
        cur.wait_stream(self.comp)

    @staticmethod
    def _heads(weight, bias):
        for t in (weight, bias):
            if t is not None and t.dim() == 2:
                return int(t.shape[0])
        return 1

    def fwd(self, x: torch.Tensor, weight: Optional[torch.Tensor], bias: Optional[torch.Tensor] = None,
            residual: Optional[torch.Tensor] = None, residual_dtype: Optional[torch.dtype] = None,
            eps: float = 1e-6, out: Optional[torch.Tensor] = None,
            residual_out: Optional[torch.Tensor] = None, rstd: Optional[torch.Tensor] = None):
        """Forward of host tensors x / residual ([rows, N], pinned for overlap; rows are
        token*head rows for per-head (H, N) parameters) with device weight / bias. Returns
        (out, residual_out) on the host; residual_out is None when there is no residual.
        When `rstd` (a device fp32 tensor with one element per row) is given it is filled.
        Work is enqueued on the current stream's device timeline; synchronise before
        reading the results."""
        rows, n = x.shape
        h = self._heads(weight, bias)
        wh = h if (weight is not None and weight.dim() == 2) else 1
        bh = h if (bias is not None and bias.dim() == 2) else 1
        if out is None:
            out = torch.empty((rows, n), dtype=x.dtype, pin_memory=True)
        ins = {"x": x}
        outs = {"out": out}
        if residual is not None:
            ins["res"] = residual
            if residual_out is None:
                residual_out = torch.empty((rows, n), dtype=residual_dtype or residual.dtype, pin_memory=True)
            outs["ro"] = residual_out
        w = weight.contiguous() if weight is not None else None
        b = bias.contiguous() if bias is not None else None

        state = {"row": 0}

        def launch(buf, m):
            r0 = state["row"]
            _lib.fwd(buf["x"][:m], buf["res"][:m] if "res" in buf else None, w, wh, b, bh,
                     buf["out"][:m], buf["ro"][:m] if "ro" in buf else None,
                     rstd[r0:r0 + m] if rstd is not None else None, h, float(eps))
            state["row"] = r0 + m

        self._run(rows, ins, outs, launch, multiple=h)
        return out, residual_out

    def layernorm(self, x: torch.Tensor, weight: Optional[torch.Tensor], bias: Optional[torch.Tensor] = None,
                  eps: float = 1e-6, out: Optional[torch.Tensor] = None, mean: Optional[torch.Tensor] = None,
                  rstd: Optional[torch.Tensor] = None):
        """LayerNorm forward of a host tensor x ([rows, N], pinned for overlap) with device
        weight / bias (N,). Returns out on the host; `mean` / `rstd` (device fp32, one per
        row) are filled when given."""
        rows, n = x.shape
        if out is None:
            out = torch.empty((rows, n), dtype=x.dtype, pin_memory=True)
        w = weight.contiguous() if weight is not None else None
        b = bias.contiguous() if bias is not None else None
        state = {"row": 0}

        def launch(buf, m):
            r0 = state["row"]
            _lib.layernorm_fwd(buf["x"][:m], n, w, b, buf["out"][:m],
                               mean[r0:r0 + m] if mean is not None else None,
                               rstd[r0:r0 + m] if rstd is not None else None, float(eps))
            state["row"] = r0 + m

        self._run(rows, {"x": x}, {"out": out}, launch, multiple=1)
        return out

    def bwd(self, x: torch.Tensor, weight: Optional[torch.Tensor], dout: torch.Tensor, rstd: torch.Tensor,
            has_bias: bool = False, dx: Optional[torch.Tensor] = None):
        """Backward of host tensors x / dout ([rows, N], pinned) with device weight and
        device rstd. Returns (dx on the host, dweight and dbias on the device): the
        per-chunk partial sums are accumulated on the device in chunk order."""
        rows, n = x.shape
        h = self._heads(weight, None)
        if dx is None:
            dx = torch.empty((rows, n), dtype=x.dtype, pin_memory=True)
        dw = torch.zeros(weight.shape, dtype=torch.float32, device=self.device) if weight is not None else None
        db_shape = weight.shape if weight is not None else (n,)
        db = torch.zeros(db_shape, dtype=torch.float32, device=self.device) if has_bias else None
        dw_c = torch.empty_like(dw) if dw is not None else None
        db_c = torch.empty_like(db) if db is not None else None
        w = weight.contiguous() if weight is not None else None
        state = {"row": 0}

        def launch(buf, m):
            r0 = state["row"]
            a = _lib.bwd_args(buf["x"][:m], buf["dy"][:m], rstd[r0:r0 + m], w, h, None, buf["dx"][:m], None,
                              dw_c, db_c, h, h)
            nbytes = _lib.bwd_workspace_bytes(a, self.device)
            if self._ws is None or self._ws.numel() < nbytes:
                self._ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=self.device)
            _lib.bwd(a, self.device, self._ws)
            if dw is not None:
                dw.add_(dw_c)
            if db is not None:
                db.add_(db_c)
            state["row"] = r0 + m

        self._run(rows, {"x": x, "dy": dout}, {"dx": dx}, launch, multiple=h)
        return dx, dw, db

    def fwd_bwd(self, x: torch.Tensor, weight: Optional[torch.Tensor], bias: Optional[torch.Tensor],
                residual: Optional[torch.Tensor], dout: torch.Tensor,
                residual_dtype: Optional[torch.dtype] = None, eps: float = 1e-6,
                out: Optional[torch.Tensor] = None, dx: Optional[torch.Tensor] = None,
                grads: Optional[torch.Tensor] = None):
        """Forward and backward of one training step on host tensors x / residual / dout
        ([rows, N] with a shared (N,) weight / bias on the device; pinned for overlap).
        Per chunk: the inputs are copied in, the forward writes out, residual_out and rstd
        (residual_out and rstd stay in device buffers), the backward reads them with dout
        and writes dx, and out / dx are copied back; dresidual is dx, as in rmsnorm_bwd with
        has_residual. dweight / dbias are fp32 sums over all chunks on the device,
        accumulated in chunk order (into `grads` = [dweight | dbias] fp32 when given).
        Returns (out, dx, dweight, dbias)."""
        rows, n = x.shape
        if out is None:
            out = torch.empty((rows, n), dtype=x.dtype, pin_memory=True)
        if dx is None:
            dx = torch.empty((rows, n), dtype=x.dtype, pin_memory=True)
        nw = n if weight is not None else 0
        nb = n if bias is not None else 0
        if grads is None:
            grads = torch.empty(nw + nb, dtype=torch.float32, device=self.device)
        grads.zero_()
        acc_w = grads[:nw] if nw else None
        acc_b = grads[nw:nw + nb] if nb else None
        part = torch.empty(nw + nb, dtype=torch.float32, device=self.device)
        part_w = part[:nw] if nw else None
        part_b = part[nw:nw + nb] if nb else None
        w = weight.contiguous() if weight is not None else None
        b = bias.contiguous() if bias is not None else None
        ro_dt = residual_dtype or (residual.dtype if residual is not None else x.dtype)
        ins = {"x": x, "dy": dout}
        if residual is not None:
            ins["res"] = residual
        scratch = {"ro": ((n,), ro_dt), "rstd": ((), torch.float32)}

        def launch(buf, m):
            ro = buf["ro"][:m]
            rstd = buf["rstd"][:m]
            _lib.fwd(buf["x"][:m], buf["res"][:m] if "res" in buf else None, w, 1, b, 1, buf["out"][:m], ro,
                     rstd, 1, float(eps))
            a = _lib.bwd_args(ro, buf["dy"][:m], rstd, w, 1, None, buf["dx"][:m], None, part_w, part_b, 1, 1)
            nbytes = _lib.bwd_workspace_bytes(a, self.device)
            if self._ws is None or self._ws.numel() < nbytes:
                self._ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=self.device)
            _lib.bwd(a, self.device, self._ws)
            if nw or nb:
                grads.add_(part)

        self._run(rows, ins, {"out": out, "dx": dx}, launch, multiple=1, scratch=scratch)
        return out, dx, acc_w, acc_b

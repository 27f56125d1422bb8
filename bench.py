# SPDX-License-Identifier: MIT
"""Benchmark of the RMSNorm hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|refgpu]
                    [--workload NAME] [--scaling strong|weak]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1; one rank per GPU, NCCL)

Default workload `cfg2fb` (BASELINE config 2 as a training step, the configuration the
headline metric is quoted on): RMSNorm forward with residual fusion -- x and residual
(32768, 16384) bf16, fp32 weight and bias, fp32 residual_out, rstd saved, eps 1e-6 --
followed by its backward (the saved fp32 residual_out, dout bf16 -> dx bf16, which is also
dresidual, and fp32 dweight / dbias), then ONE NCCL all-reduce of [dweight | dbias] across
the ranks. The 32768 rows are sharded evenly across the N ranks (strong scaling: 4096 rows
per GPU at N = 8); `--scaling weak` gives every rank the full batch instead. The forward
never communicates; the all-reduce is the only collective.

value     : algorithmic bytes moved by all ranks per step (every tensor read or written
            once, the reference's byte model) / max-over-ranks device time per step (GB/s);
            inputs resident in HBM and larger than L2 (small configs rotate a pool of input
            sets larger than L2); CUDA events on the launching stream around K steps
            replayed from one CUDA graph.
directions: the forward, the backward (dx + the fixed-order dweight / dbias reduction) and
            the all-reduce, each timed alone the same way (K replays, max over ranks).
e2e       : the same metric through the public API on host (pinned) buffers
            (rmsnorm.host_pipeline.HostPipeline): every step copies its inputs host->device
            and its outputs (out, dx, dweight, dbias) device->host inside the timing.
roofline  : the dominant kernel's algorithmic bytes per launch / its event-timed duration,
            against the measured HBM copy bandwidth of this pool (MEASURED_PEAKS.json).
parity    : after the timing, every rank checks the final step's results against the CPU
            oracle (oracle/rmsnorm_oracle.py): a seeded sample of its rows (out,
            residual_out, rstd, dx) and a seeded sample of dweight / dbias columns, whose
            oracle sums over all ranks' rows are combined in fp64. "ok" or the process
            exits non-zero.
cpu_baseline / --impl reference : the reference's PyTorch CPU path (restated in
            oracle/rmsnorm_oracle.py; the reference checkout is not available on the GPU
            box) on a bounded row sample, all host threads.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "rmsnorm-h100_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "RMSNorm fwd/bwd achieved HBM GB/s (% of B200 peak) at 1/2/4/8 GPUs"
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 1024 * 1024
EPS = 1e-6

BF16, F16, F32 = torch.bfloat16, torch.float16, torch.float32
DTYPE_NAME = {BF16: "bf16", F16: "f16", F32: "f32"}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ----------------------------------------------------------------------------------------
# Workloads (rows = the global batch; per-rank rows depend on --scaling)
# ----------------------------------------------------------------------------------------
WORKLOADS = {
    "cfg2fb": dict(kind="train", rows=32768, n=16384, dtype=BF16, residual=True, bias=True, ro=F32, rstd=True,
                   desc="BASELINE cfg 2 training step: RMSNorm forward with residual fusion, x/residual "
                        "(32768,16384) bf16, fp32 weight+bias, fp32 residual_out, rstd saved, eps 1e-6; then its "
                        "backward (fp32 residual_out, dout bf16 -> dx bf16 = dresidual, fp32 dweight+dbias) and "
                        "one all-reduce of dweight|dbias across ranks"),
    "cfg2": dict(kind="fwd", rows=32768, n=16384, dtype=BF16, residual=True, bias=True, ro=F32, rstd=False,
                 desc="BASELINE cfg 2 forward only: RMSNorm forward with residual fusion, x/residual (32768,16384) "
                      "bf16, fp32 weight+bias, fp32 residual_out, eps 1e-6"),
    "cfg1": dict(kind="fwd", rows=8192, n=4096, dtype=BF16, residual=False, bias=False, ro=None, rstd=False,
                 desc="BASELINE cfg 1 shape on GPU: RMSNorm forward (8192,4096) bf16, fp32 weight"),
    "cfg3": dict(kind="bwd", rows=32768, n=65536, dtype=BF16, bias=False,
                 desc="BASELINE cfg 3: RMSNorm backward (32768,65536) bf16, fp32 weight -> dx bf16, dweight fp32"),
    "bwd16k": dict(kind="bwd", rows=32768, n=16384, dtype=BF16, bias=False,
                   desc="north-star target backward: RMSNorm backward (32768,16384) bf16, fp32 weight -> dx bf16, "
                        "dweight fp32"),
    "ln16k": dict(kind="ln", rows=32768, n=16384, dtype=BF16, bias=True,
                  desc="next-row LayerNorm forward (32768,16384) bf16, fp32 weight+bias, mean and rstd stored"),
    "cfg4f": dict(kind="fwd", rows=16384 * 32, n=128, heads=32, dtype=F16, residual=False, bias=True, ro=None,
                  rstd=True, desc="BASELINE cfg 4 forward: per-head (16384,32,128) fp16, (32,128) fp32 weight+bias, rstd"),
    "cfg4b": dict(kind="bwd", rows=16384 * 32, n=128, heads=32, dtype=F16, bias=True,
                  desc="BASELINE cfg 4 backward: per-head (16384,32,128) fp16 -> dx, dweight, dbias (32,128) fp32"),
    "cfg5f32f": dict(kind="fwd", rows=1024, n=262144, dtype=F32, residual=False, bias=False, ro=None, rstd=True,
                     outliers=0.01, desc="BASELINE cfg 5 fp32 forward (1024,262144), 1% x100 outliers, rstd"),
    "cfg5f32b": dict(kind="bwd", rows=1024, n=262144, dtype=F32, bias=False, outliers=0.01,
                     desc="BASELINE cfg 5 fp32 backward (1024,262144)"),
    "cfg5bf16f": dict(kind="fwd", rows=1024, n=262144, dtype=BF16, residual=False, bias=False, ro=None, rstd=True,
                      outliers=0.01, desc="BASELINE cfg 5 bf16 forward (1024,262144), 1% x100 outliers, rstd"),
    "cfg5bf16b": dict(kind="bwd", rows=1024, n=262144, dtype=BF16, bias=False, outliers=0.01,
                      desc="BASELINE cfg 5 bf16 backward (1024,262144)"),
}


def esize(dt):
    return torch.tensor([], dtype=dt).element_size()


def fwd_bytes(w, rows):
    """Forward: x (+ residual) read, out (+ residual_out) written, affine read, rstd written."""
    e = rows * w["n"]
    s = esize(w["dtype"])
    aff = w.get("heads", 1) * w["n"] * 4
    b = 2 * e * s + aff + (aff if w["bias"] else 0)
    if w.get("residual"):
        b += e * s
    if w.get("ro") is not None:
        b += e * esize(w["ro"])
    if w.get("rstd"):
        b += rows * 4
    return b


def bwd_bytes(w, rows, x_size=None):
    """Backward: x, dout and rstd read, dx written, weight read, dweight (+ dbias) written.
    x_size: element size of the saved x (the fp32 residual_out in a training step)."""
    e = rows * w["n"]
    s = esize(w["dtype"])
    aff = w.get("heads", 1) * w["n"] * 4
    b = e * ((x_size or s) + 2 * s) + rows * 4 + 2 * aff
    if w["bias"]:
        b += aff
    return b


def algo_bytes(w, rows=None):
    """Algorithmic bytes per step for `rows` rows: every tensor read or written once (the
    reference's byte model, rmsnorm/csrc/ptx_rmsnorm_kernels.cu:7107-7134)."""
    rows = w["rows"] if rows is None else rows
    if w["kind"] == "ln":
        e = rows * w["n"]
        return 2 * e * esize(w["dtype"]) + w["n"] * 4 * (2 if w["bias"] else 1) + rows * 8
    if w["kind"] == "fwd":
        return fwd_bytes(w, rows)
    if w["kind"] == "bwd":
        return bwd_bytes(w, rows)
    return fwd_bytes(w, rows) + bwd_bytes(w, rows, x_size=esize(w["ro"]))


def main_kernel(w, rows):
    """(name, bytes per launch) of the dominant kernel of a step: the streaming kernel, whose
    bytes exclude the dweight / dbias the separate reduction kernel writes; in a training
    step the forward (it moves the most bytes)."""
    aff = w.get("heads", 1) * w["n"] * 4
    if w["kind"] in ("fwd", "train"):
        return "fwd_stream_kernel", fwd_bytes(w, rows)
    if w["kind"] == "ln":
        return "fwd_stream_kernel (LayerNorm)", algo_bytes(w, rows)
    return "bwd_stream_kernel", bwd_bytes(w, rows) - aff * (2 if w["bias"] else 1)


def gen(shape, dtype, seed, dev, kind="normal", outliers=0.0):
    """Seeded synthetic tensors with the BASELINE distributions: N(0,1) activations,
    weight N(1, 0.1), bias N(0, 0.02), optional element outliers x100."""
    g = torch.Generator(device=dev).manual_seed(20260514 + seed)
    t = torch.randn(shape, generator=g, device=dev, dtype=torch.float32)
    if kind == "weight":
        t = 1.0 + 0.1 * t
    elif kind == "bias":
        t = 0.02 * t
    if outliers > 0:
        t = torch.where(torch.rand(shape, generator=g, device=dev) < outliers, t * 100.0, t)
    return t.to(dtype)


def make_inputs(w, rows, dev, seed):
    h = w.get("heads", 1)
    shape = (rows, w["n"])
    aff = (h, w["n"]) if h > 1 else (w["n"],)
    t = {}
    t["x"] = gen(shape, w["dtype"], seed, dev, outliers=w.get("outliers", 0.0))
    t["w"] = gen(aff, F32, 1, dev, "weight")  # the parameters are the same on every rank
    t["b"] = gen(aff, F32, 3, dev, "bias") if w["bias"] else None
    if w["kind"] in ("fwd", "ln", "train"):
        t["res"] = gen(shape, w["dtype"], seed + 2, dev) if w.get("residual") else None
    if w["kind"] in ("bwd", "train"):
        t["dy"] = gen(shape, w["dtype"], seed + 4, dev)
    if w["kind"] == "bwd":
        t["rstd"] = torch.cat([torch.rsqrt(t["x"][i:i + 1024].float().square().mean(-1) + EPS)
                               for i in range(0, rows, 1024)]) if rows else torch.empty(0, device=dev)
    return t


class Runner:
    """Preallocated outputs + the C-ABI launches of one step for one input set."""

    def __init__(self, w, t, dev, group):
        from rmsnorm import _lib

        self.w, self.t, self.dev, self.group, self.lib = w, t, dev, group, _lib
        self.peer = None  # native peer group handle (set when the fused all-reduce is used)
        self.h = h = w.get("heads", 1)
        x = t["x"]
        rows = x.shape[0]
        kind = w["kind"]
        self.grads = None
        if kind == "ln":
            self.out = torch.empty_like(x)
            self.mean = torch.empty(rows, dtype=F32, device=dev)
            self.rstd = torch.empty(rows, dtype=F32, device=dev)
        if kind in ("fwd", "train"):
            self.out = torch.empty_like(x)
            self.ro = torch.empty(x.shape, dtype=w["ro"], device=dev) if w["ro"] is not None else None
            self.rstd = torch.empty(rows, dtype=F32, device=dev) if w["rstd"] else None
        if kind in ("bwd", "train"):
            n_aff = t["w"].numel()
            # fp32 [dweight | dbias]: the backward writes its sums here and the all-reduce sums
            # the buffer in place
            self.grads = torch.empty(n_aff * (2 if w["bias"] else 1), dtype=F32, device=dev)
            self.dw = self.grads[:n_aff].view(t["w"].shape)
            self.db = self.grads[n_aff:].view(t["w"].shape) if w["bias"] else None
            self.dx = torch.empty_like(x)
            saved_x = self.ro if kind == "train" else x
            rstd = self.rstd if kind == "train" else t["rstd"]
            self.args = _lib.bwd_args(saved_x, t["dy"], rstd, t["w"], h, None, self.dx, None, self.dw, self.db, h, h)
            nbytes = _lib.bwd_workspace_bytes(self.args, dev)
            self.ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
            self.ar_scratch = torch.zeros_like(self.grads)  # all-reduce timed alone

    def fwd(self):
        w, t, h = self.w, self.t, self.h
        if w["kind"] == "ln":
            self.lib.layernorm_fwd(t["x"], w["n"], t["w"], t["b"], self.out, self.mean, self.rstd, EPS)
        else:
            self.lib.fwd(t["x"], t.get("res"), t["w"], h, t["b"], h, self.out, self.ro, self.rstd, h, EPS)

    def bwd(self, local=False):
        """The backward; with a peer group (and not `local`) its dweight / dbias are summed
        over the ranks by the library's fused reduction + all-reduce kernel."""
        self.lib.bwd(self.args, self.dev, self.ws, peer_group=None if local else self.peer)

    def allreduce(self, buf=None):
        import torch.distributed as dist

        dist.all_reduce(self.grads if buf is None else buf, op=dist.ReduceOp.SUM, group=self.group)

    def step(self):
        kind = self.w["kind"]
        if kind in ("fwd", "ln", "train"):
            self.fwd()
        if kind in ("bwd", "train"):
            self.bwd()
            if self.group is not None and self.peer is None:
                self.allreduce()


# ----------------------------------------------------------------------------------------
# Clock sampling (NVML, in a thread, during the timed region)
# ----------------------------------------------------------------------------------------
_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
            0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


class ClockSampler:
    def __init__(self, index, period=0.005):
        self.samples, self.reasons, self.ok = [], 0, False
        self.period = period
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as exc:  # no NVML: report it, do not fail the benchmark
            log(f"[bench] NVML unavailable: {exc}")
            self.max_mhz = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        names = [v for k, v in _REASONS.items() if self.reasons & k and v != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def traffic_for(workload):
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        d = json.loads(p.read_text())
        v = d.get(workload)
        if isinstance(v, dict):
            return v.get("bytes_per_launch")
    return None


# ----------------------------------------------------------------------------------------
# CPU baseline: the reference's PyTorch CPU path (oracle port) on a bounded row sample
# ----------------------------------------------------------------------------------------
def cpu_sample_rows(w):
    # up to 32M elements per step (16M for a training step): the whole of cfg 1 (8192 x
    # 4096), a row sample of the larger configs (2048 rows of cfg 2, 1024 of its training
    # step) -- long enough to time, short enough to repeat
    elems = (16 << 20) if w["kind"] == "train" else (32 << 20)  # a training step does both passes
    rows = max(1, min(w["rows"], elems // w["n"]))
    if w.get("heads", 1) > 1:
        rows -= rows % w["heads"]
    return rows


def cpu_step_fn(w, rows):
    from oracle import rmsnorm_oracle as oracle

    h = w.get("heads", 1)
    shape = (rows, w["n"])
    aff = (h, w["n"]) if h > 1 else (w["n"],)
    x = gen(shape, w["dtype"], 1, "cpu", outliers=w.get("outliers", 0.0))
    wt = gen(aff, F32, 2, "cpu", "weight")
    if h > 1:
        x = x.reshape(rows // h, h, w["n"])
    b = gen(aff, F32, 4, "cpu", "bias") if w["bias"] else None
    if w["kind"] == "ln":
        return lambda: oracle.layernorm_fwd(x, wt, b)
    res = gen(x.shape, w["dtype"], 3, "cpu") if w.get("residual") else None
    if w["kind"] == "fwd":
        return lambda: oracle.fwd(x, wt, b, res, residual_dtype=w["ro"])
    dy = gen(x.shape, w["dtype"], 5, "cpu")
    if w["kind"] == "train":
        def train():
            _, ro, rstd, _ = oracle.fwd(x, wt, b, res, residual_dtype=w["ro"])
            oracle.bwd(ro, wt, dy, rstd, has_bias=w["bias"])
        return train
    rstd = torch.rsqrt(x.float().square().mean(-1) + EPS)
    return lambda: oracle.bwd(x, wt, dy, rstd, has_bias=w["bias"])


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline(w, budget_s=10.0):
    torch.set_num_threads(os.cpu_count() or 1)
    rows = cpu_sample_rows(w)
    fn = cpu_step_fn(w, rows)
    fn()  # warm
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < 3 or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
        if len(times) >= 200:
            break
    per = statistics.median(times)
    gbs = algo_bytes(w, rows) / per / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
            "cpu_model": cpu_model(), "rows_per_s": round(rows / per, 1),
            "sample": f"{rows} of {w['rows']} rows per step, median of {len(times)} steps, "
                      f"oracle/rmsnorm_oracle.py restating rmsnorm/rmsnorm.py (reference PyTorch CPU path)"}


# ----------------------------------------------------------------------------------------
def run_reference_arm(args, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    rows = cpu_sample_rows(w)
    fn = cpu_step_fn(w, rows)
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    el = time.perf_counter() - t0
    per = el / args.steps
    gbs = algo_bytes(w, rows) / per / 1e9
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per * 1e3, 4), "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": DTYPE_NAME[w["dtype"]], "impl": "reference",
        "data": "synthetic: seeded N(0,1) inputs, weight N(1,0.1), bias N(0,0.02)",
        "config": {"workload": w["desc"], "sample_rows_per_step": rows, "rows": w["rows"], "hidden": w["n"]},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
                         "cpu_model": cpu_model(), "rows_per_s": round(rows / per, 1),
                         "sample": f"{rows} rows per step of the workload; reference PyTorch CPU path restated "
                                   f"in oracle/rmsnorm_oracle.py (reference checkout absent on the GPU box)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


def run_refgpu(args, w):
    """Times the reference's Hopper kernels (recompiled for sm_100a) on this workload, one
    GPU, device time of K steps (CUDA graph replay when capturable, else eager)."""
    from oracle import ref_gpu

    if w["kind"] in ("ln", "train"):
        print(json.dumps({"impl": "refgpu", "unavailable": f"no reference-kernel step for workload kind "
                          f"{w['kind']} (the reference's layernorm_fwd is PyTorch ops; time cfg2 and the "
                          f"backward separately)"}), flush=True)
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ext = ref_gpu.load()
    h = w.get("heads", 1)
    rows = w["rows"]
    one_set = algo_bytes(w)
    pool = 1 if one_set > 2 * L2_BYTES else max(2, -(-3 * L2_BYTES // one_set))
    sets = [make_inputs(w, rows, dev, 100 * i) for i in range(pool)]
    steps = [ref_gpu.make_step(ext, w["kind"], t, heads=h, ro_dtype=w.get("ro"), store_rstd=w.get("rstd", False),
                               has_bias=w.get("bias", False) if w["kind"] == "bwd" else False) for t in sets]
    try:
        for i in range(args.warmup):
            steps[i % pool]()
        torch.cuda.synchronize(dev)
    except RuntimeError as exc:  # e.g. the fp32 backward at N = 262144 has no working path there
        print(json.dumps({"impl": "refgpu", "unavailable": "the reference kernels refuse this workload: "
                          + str(exc).splitlines()[0]}), flush=True)
        return
    stream = torch.cuda.current_stream(dev)
    graph, how = None, "eager launches"
    try:
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            for i in range(args.steps):
                steps[i % pool]()
        stream.wait_stream(side)
        g.replay()
        torch.cuda.synchronize(dev)
        graph, how = g, "CUDA graph replay of the K steps"
    except Exception as exc:  # the reference's bindings allocate and cache per call
        log(f"[bench] reference steps not capturable ({exc}); timing eager launches")
        torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    if graph is not None:
        graph.replay()
    else:
        for i in range(args.steps):
            steps[i % pool]()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / args.steps
    print(json.dumps({"impl": "refgpu", "metric": METRIC, "value": round(algo_bytes(w) / (ms * 1e-3) / 1e9, 2),
                      "unit": "GB/s", "ms_per_step": round(ms, 5), "n_gpus": 1, "steps": args.steps,
                      "warmup": args.warmup, "config": {"workload": w["desc"], "timing": how,
                      "kernels": "reference rmsnorm/csrc recompiled for sm_100a (oracle/_ref)"}}), flush=True)


# ----------------------------------------------------------------------------------------
# Timing helpers
# ----------------------------------------------------------------------------------------
def barrier(group):
    if group is not None:
        import torch.distributed as dist

        dist.barrier(group=group)


def max_over_ranks(v, dev, group):
    if group is None:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


class Timed:
    """K calls of fn captured once into a CUDA graph (eager launches when capture is off or
    fails), replayed once untimed, then timed with CUDA events on the launching stream."""

    def __init__(self, fn, steps, dev, use_graph):
        from rmsnorm import _lib

        self.fn, self.steps, self.dev = fn, steps, dev
        self.stream = torch.cuda.current_stream(dev)
        self.graph = None
        self.launches = None
        if use_graph:
            try:
                side = torch.cuda.Stream(dev)
                side.wait_stream(self.stream)
                g = torch.cuda.CUDAGraph()
                c0 = _lib.launch_count()
                with torch.cuda.graph(g, stream=side):
                    for i in range(steps):
                        fn(i)
                self.launches = _lib.launch_count() - c0
                self.stream.wait_stream(side)
                g.replay()
                torch.cuda.synchronize(dev)
                self.graph = g
            except Exception as exc:
                log(f"[bench] capture failed ({exc}); timing eager launches")
                torch.cuda.synchronize(dev)
        self.how = "CUDA graph replay of the K steps" if self.graph is not None else "eager launches"

    def run(self, group, clk=None):
        """Device time of the K calls in ms, max over ranks."""
        from rmsnorm import _lib

        barrier(group)
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        c0 = _lib.launch_count()
        torch.cuda.synchronize(self.dev)
        if clk is not None:
            clk.__enter__()
        t0.record(self.stream)
        if self.graph is not None:
            self.graph.replay()
        else:
            for i in range(self.steps):
                self.fn(i)
        t1.record(self.stream)
        torch.cuda.synchronize(self.dev)
        if clk is not None:
            clk.__exit__()
        if self.graph is None:
            self.launches = _lib.launch_count() - c0
        own = t0.elapsed_time(t1)
        return max_over_ranks(own, self.dev, group), own

    def release(self):
        self.graph = None


# ----------------------------------------------------------------------------------------
# Parity against the CPU oracle after the timing
# ----------------------------------------------------------------------------------------
def parity_check(w, runner, dev, group, rank):
    """Checks the final step's results of this rank against the oracle; returns (ok, why).
    Rows: a seeded sample of whole rows (tokens for per-head rows): out, residual_out, rstd,
    dx. Columns: a seeded sample of dweight / dbias columns, whose oracle sums over this
    rank's rows are combined across ranks in fp64 (the kernel's sums are fp32)."""
    from oracle import rmsnorm_oracle as oracle

    import torch.distributed as dist

    t = runner.t
    kind = w["kind"]
    h = w.get("heads", 1)
    x = t["x"]
    rows = x.shape[0]
    ntok = rows // h
    n = w["n"]
    g = torch.Generator().manual_seed(1234 + rank)
    why = []
    ok = True
    wt = t["w"].cpu()
    b = t["b"].cpu() if t.get("b") is not None else None
    if ntok > 0:
        toks = torch.unique(torch.cat([torch.tensor([0, ntok - 1]), torch.randint(0, ntok, (6,), generator=g)]))
        sel = (toks.view(-1, 1) * h + torch.arange(h).view(1, -1)).reshape(-1).to(dev)

        def rows_of(tt):
            v = tt[sel].cpu()
            return v.view(len(toks), h, *v.shape[1:]) if h > 1 else v

        try:
            xs = rows_of(x)
            if kind == "ln":
                _, o_rstd, o_mean, y = oracle.layernorm_fwd(xs, wt, b, EPS)
                oracle.check_close(rows_of(runner.out), y, w["dtype"], "ln out")
                assert torch.allclose(rows_of(runner.rstd), o_rstd, rtol=1e-4, atol=0), "ln rstd"
            if kind in ("fwd", "train"):
                res = rows_of(t["res"]) if t.get("res") is not None else None
                _, o_ro, o_rstd, y = oracle.fwd(xs, wt, b, res, EPS, residual_dtype=w["ro"])
                oracle.check_close(rows_of(runner.out), y, w["dtype"], "out")
                if runner.ro is not None:
                    assert torch.equal(rows_of(runner.ro), o_ro), "residual_out differs"
                if runner.rstd is not None:
                    assert torch.allclose(rows_of(runner.rstd), o_rstd, rtol=1e-5, atol=0), "rstd"
            if kind in ("bwd", "train"):
                saved = rows_of(runner.ro) if kind == "train" else xs
                rstd_in = rows_of(runner.rstd if kind == "train" else t["rstd"])
                o_dx, _, _, _, _ = oracle.bwd(saved, wt, rows_of(t["dy"]), rstd_in)
                oracle.check_close(rows_of(runner.dx), o_dx, w["dtype"], "dx")
        except AssertionError as exc:
            ok = False
            why.append(f"rank {rank} rows: {exc}")
    if kind in ("bwd", "train"):
        # dweight / dbias on a column sample: the oracle's per-column sums over this rank's
        # rows (oracle.bwd's dweight / dbias are column-separable; its dx output, which needs
        # whole rows, is not used here), summed across ranks in fp64
        cols = torch.unique(torch.randint(0, n, (64,), generator=torch.Generator().manual_seed(99)))
        cols_d = cols.to(dev)
        saved = runner.ro if kind == "train" else x
        rstd_in = runner.rstd if kind == "train" else t["rstd"]
        xs = saved[:, cols_d].cpu()
        dys = t["dy"][:, cols_d].cpu()
        if h > 1:
            xs, dys = xs.view(ntok, h, -1), dys.view(ntok, h, -1)
            wc = wt[:, cols]
            rs = rstd_in.cpu().view(ntok, h)
        else:
            wc = wt[cols]
            rs = rstd_in.cpu()
        _, o_dw, o_db, s_dw, s_db = oracle.bwd(xs, wc, dys, rs, has_bias=w["bias"], bias_shape=wc.shape)
        parts = [o_dw, s_dw] + ([o_db, s_db] if w["bias"] else [])
        ref = torch.cat([p.reshape(-1).double() for p in parts]).to(dev)
        if group is not None:
            dist.all_reduce(ref, op=dist.ReduceOp.SUM, group=group)
        ref = ref.cpu()
        m = o_dw.numel()
        got_dw = (runner.dw[:, cols_d] if h > 1 else runner.dw[cols_d]).cpu()
        try:
            oracle.check_reduction(got_dw, ref[0:m].view(o_dw.shape), ref[m:2 * m].view(o_dw.shape), "dweight")
            if w["bias"]:
                got_db = (runner.db[:, cols_d] if h > 1 else runner.db[cols_d]).cpu()
                oracle.check_reduction(got_db, ref[2 * m:3 * m].view(o_dw.shape), ref[3 * m:4 * m].view(o_dw.shape),
                                       "dbias")
        except AssertionError as exc:
            ok = False
            why.append(f"rank {rank} columns: {exc}")
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
    if group is not None:
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return bool(flag.item()), "; ".join(why)


# ----------------------------------------------------------------------------------------
# End to end on host buffers
# ----------------------------------------------------------------------------------------
def e2e_measure(w, t_dev, dev, steps, group):
    """Public API with pinned host buffers (rmsnorm.host_pipeline.HostPipeline): every step
    copies its inputs host->device, runs the kernels, and copies its results back, with
    the copies of consecutive row chunks overlapped on both copy engines."""
    import torch.distributed as dist

    from rmsnorm.host_pipeline import HostPipeline

    h = w.get("heads", 1)
    rows, n = t_dev["x"].shape
    pipe = HostPipeline(dev, chunk_rows=max(h, min(max(rows, 1), (32 << 20) // (n * 2))))
    host = {k: t_dev[k].cpu().pin_memory() for k in ("x", "res", "dy") if t_dev.get(k) is not None}
    wt, b = t_dev["w"], t_dev.get("b")
    stream = torch.cuda.current_stream(dev)
    kind = w["kind"]
    if kind == "ln":
        out_h = torch.empty((rows, n), dtype=w["dtype"], pin_memory=True)
        mean = torch.empty(rows, dtype=F32, device=dev)
        rstd = torch.empty(rows, dtype=F32, device=dev)
        stats_h = torch.empty(2, rows, dtype=F32, pin_memory=True)

        def one():
            pipe.layernorm(host["x"], wt, b, out=out_h, mean=mean, rstd=rstd)
            stats_h[0].copy_(mean, non_blocking=True)
            stats_h[1].copy_(rstd, non_blocking=True)

        d2h = out_h.numel() * out_h.element_size() + rows * 8
    elif kind == "fwd":
        out_h = torch.empty((rows, n), dtype=w["dtype"], pin_memory=True)
        ro_h = torch.empty((rows, n), dtype=w["ro"], pin_memory=True) if w["ro"] is not None else None
        rstd = torch.empty(rows, dtype=F32, device=dev) if w["rstd"] else None
        rstd_h = torch.empty(rows, dtype=F32, pin_memory=True) if w["rstd"] else None

        def one():
            pipe.fwd(host["x"], wt, b, host.get("res"), residual_dtype=w["ro"], out=out_h, residual_out=ro_h,
                     rstd=rstd)
            if rstd is not None:
                rstd_h.copy_(rstd, non_blocking=True)

        d2h = out_h.numel() * out_h.element_size() + (ro_h.numel() * ro_h.element_size() if ro_h is not None else 0)
        d2h += rows * 4 if rstd is not None else 0
    elif kind == "train":
        out_h = torch.empty((rows, n), dtype=w["dtype"], pin_memory=True)
        dx_h = torch.empty((rows, n), dtype=w["dtype"], pin_memory=True)
        grads = torch.empty(n * (2 if w["bias"] else 1), dtype=F32, device=dev)
        grads_h = torch.empty(grads.shape, dtype=F32, pin_memory=True)

        def one():
            pipe.fwd_bwd(host["x"], wt, b, host.get("res"), host["dy"], residual_dtype=w["ro"], out=out_h, dx=dx_h,
                         grads=grads)
            if group is not None:
                dist.all_reduce(grads, op=dist.ReduceOp.SUM, group=group)
            grads_h.copy_(grads, non_blocking=True)

        d2h = 2 * out_h.numel() * out_h.element_size() + grads.numel() * 4
    else:
        dx_h = torch.empty((rows, n), dtype=w["dtype"], pin_memory=True)
        dw_h = torch.empty(wt.shape, dtype=F32, pin_memory=True)
        db_h = torch.empty(wt.shape, dtype=F32, pin_memory=True) if w["bias"] else None

        def one():
            _, dw, db = pipe.bwd(host["x"], wt, host["dy"], t_dev["rstd"], has_bias=w["bias"], dx=dx_h)
            if group is not None:
                from rmsnorm.distributed import allreduce_sum_

                allreduce_sum_([dw, db], group=group)
            dw_h.copy_(dw, non_blocking=True)
            if db_h is not None:
                db_h.copy_(db, non_blocking=True)

        d2h = dx_h.numel() * dx_h.element_size() + dw_h.numel() * 4 * (2 if db_h is not None else 1)
    h2d = sum(v.numel() * v.element_size() for v in host.values())

    one()
    torch.cuda.synchronize(dev)
    barrier(group)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        one()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, dev, group)
    return ms, h2d, d2h


# ----------------------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference", "refgpu"], default="ours",
                    help="refgpu: the reference's own CUDA kernels recompiled for sm_100a (oracle/_ref), "
                         "timed on the same workload for comparison")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cfg2fb")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="strong: the workload's rows are split across the ranks; weak: every rank runs them all")
    ap.add_argument("--allreduce", choices=["auto", "peer", "nccl"], default="auto",
                    help="dweight/dbias across ranks: the library's fused kernel over peer memory (peer), NCCL, "
                         "or peer unless its set-up fails (auto)")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-directions", action="store_true", help="skip the per-direction timings")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--eager", action="store_true", help="time eager launches instead of a graph replay")
    ap.add_argument("--rows", type=int, default=0, help="override the workload's (global) rows (profiling runs)")
    ap.add_argument("--hidden", type=int, default=0, help="override the hidden size (profiling runs)")
    ap.add_argument("--no-e2e", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    w = dict(WORKLOADS[args.workload])
    if args.rows:
        w["rows"] = args.rows - args.rows % w.get("heads", 1)
        w["desc"] += f" [rows overridden: {w['rows']}]"
    if args.hidden:
        w["n"] = args.hidden
        w["desc"] += f" [hidden overridden: {w['n']}]"

    if args.impl == "reference":
        run_reference_arm(args, w)
        return
    if args.impl == "refgpu":
        run_refgpu(args, w)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    group = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
        group = dist.group.WORLD

    from rmsnorm import _lib
    from rmsnorm.distributed import row_range

    _lib.load_library()
    h = w.get("heads", 1)
    if args.scaling == "strong":
        t0_, t1_ = row_range(w["rows"] // h, rank, world)
        rows = (t1_ - t0_) * h
        all_rows = [(row_range(w["rows"] // h, r, world)[1] - row_range(w["rows"] // h, r, world)[0]) * h
                    for r in range(world)]
    else:
        rows = w["rows"]
        all_rows = [rows] * world
    job_bytes = sum(algo_bytes(w, r) for r in all_rows)
    kind = w["kind"]

    # rotating pool of input sets when one set is smaller than L2
    one_set = algo_bytes(w, rows)
    pool = 1 if one_set > 2 * L2_BYTES else max(2, -(-3 * L2_BYTES // max(one_set, 1)))
    sets = [make_inputs(w, rows, dev, 100 * i + 7 * rank) for i in range(pool)]
    runners = [Runner(w, t, dev, group) for t in sets]

    # dweight / dbias across ranks: the library's fused reduction + all-reduce over peer
    # memory, or NCCL (auto: the fused kernel unless its set-up fails on any rank)
    peer_group, ar_backend = None, "nccl" if group is not None else None
    if group is not None and kind in ("bwd", "train") and args.allreduce != "nccl":
        import torch.distributed as dist

        from rmsnorm.distributed import PeerGroup

        ok = 1
        try:
            peer_group = PeerGroup(runners[0].grads.numel(), group=group)
        except Exception as exc:  # e.g. no CUDA IPC between the ranks' GPUs
            log(f"[bench] peer group set-up failed on rank {rank}: {exc}")
            ok = 0
        flag = torch.tensor([ok], dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
        if flag.item() == 1:
            ar_backend = "peer"
            for r in runners:
                r.peer = peer_group.handle
        else:
            if peer_group is not None:
                peer_group.close()
            peer_group = None
            if args.allreduce == "peer":
                raise SystemExit("--allreduce peer: the peer group could not be set up")

    for i in range(args.warmup):
        runners[i % pool].step()
    torch.cuda.synchronize(dev)
    plan = _lib.last_plan()  # the launch plan of the (last kernel of the) timed steps
    plans = {}
    if kind in ("fwd", "train", "ln"):
        runners[0].fwd()
        plans["fwd"] = _lib.last_plan()
    if kind in ("bwd", "train"):
        runners[0].bwd()
        plans["bwd"] = _lib.last_plan()
    torch.cuda.synchronize(dev)
    use_graph = not args.eager

    # ---- the headline: K whole steps ----
    full = Timed(lambda i: runners[i % pool].step(), args.steps, dev, use_graph)
    clk = ClockSampler(local)  # samples only inside the timed region
    total_ms, own_total_ms = full.run(group, clk)
    ms_step = total_ms / args.steps
    launches = full.launches
    full.release()

    # ---- per direction ----
    directions = {}
    peak, peak_kind = peaks()
    kern_name, kern_bytes = main_kernel(w, rows)
    kern_ms = None
    if not args.no_directions and kind in ("train", "bwd"):
        if kind == "train":
            tf = Timed(lambda i: runners[i % pool].fwd(), args.steps, dev, use_graph)
            fwd_ms = tf.run(group)[0] / args.steps
            tf.release()
            fb = fwd_bytes(w, rows)
            directions["fwd"] = {"kernel": "fwd_stream_kernel", "ms": round(fwd_ms, 5),
                                 "bytes_per_rank": fb, "gbs_per_gpu": round(fb / (fwd_ms * 1e-3) / 1e9, 1),
                                 "frac": round(fb / (fwd_ms * 1e-3) / 1e9 / peak, 4), "plan": plans.get("fwd")}
            kern_ms = fwd_ms
        tb = Timed(lambda i: runners[i % pool].bwd(local=True), args.steps, dev, use_graph)
        bwd_ms = tb.run(group)[0] / args.steps
        tb.release()
        bb = bwd_bytes(w, rows, x_size=esize(w["ro"]) if kind == "train" else None)
        directions["bwd"] = {"kernels": "bwd_stream_kernel + reduce_partials_kernel", "ms": round(bwd_ms, 5),
                             "bytes_per_rank": bb, "gbs_per_gpu": round(bb / (bwd_ms * 1e-3) / 1e9, 1),
                             "frac": round(bb / (bwd_ms * 1e-3) / 1e9 / peak, 4), "plan": plans.get("bwd")}
        if group is not None:
            ar = {"bytes": runners[0].grads.numel() * 4, "backend": ar_backend}
            if peer_group is not None:
                # the fused kernel replaces reduce_partials_kernel: its cost is the backward
                # with it minus the backward with the local reduction
                tp = Timed(lambda i: runners[i % pool].bwd(), args.steps, dev, use_graph)
                bwd_peer_ms = tp.run(group)[0] / args.steps
                tp.release()
                ar["bwd_with_fused_allreduce_ms"] = round(bwd_peer_ms, 5)
                ar["us"] = round((bwd_peer_ms - bwd_ms) * 1e3, 2)
                ar["kernel"] = "reduce_allreduce_kernel (reduction of the partial rows + all-reduce over peer memory)"
            ta = Timed(lambda i: runners[i % pool].allreduce(runners[i % pool].ar_scratch), args.steps, dev,
                       use_graph)
            ar_ms = ta.run(group)[0] / args.steps
            ta.release()
            if peer_group is None:
                ar["us"] = round(ar_ms * 1e3, 2)
            else:
                ar["nccl_allreduce_alone_us"] = round(ar_ms * 1e3, 2)
            ar["timing"] = ta.how
            directions["allreduce"] = ar
        if kind == "bwd":
            kern_ms = None
    if kern_ms is None:
        # the whole step is the dominant kernel's launch (forward-only workloads), or the
        # backward step timed above (its reduction kernel included: a lower bound)
        kern_ms = directions["bwd"]["ms"] if "bwd" in directions and kind == "bwd" else ms_step
        if kind == "train":  # directions skipped: the whole step stands in for its kernels
            kern_name, kern_bytes = "whole step (forward + backward kernels)", algo_bytes(w, rows)
    value = job_bytes / (ms_step * 1e-3) / 1e9
    achieved = kern_bytes / (kern_ms * 1e-3) / 1e9

    # ---- parity of the final step's results ----
    parity = "skipped"
    if not args.no_parity:
        for r in runners:
            r.step()  # every runner's outputs from one full step (all-reduce included)
        torch.cuda.synchronize(dev)
        ok, why = parity_check(w, runners[0], dev, group, rank)
        parity = "ok" if ok else f"FAILED: {why or 'on another rank'}"
        if not ok:
            log(f"[bench] parity failed: {why}")

    if args.no_e2e:
        e2e_ms, h2d, d2h, e2e_value = float("nan"), 0, 0, None
    else:
        e2e_ms, h2d, d2h = e2e_measure(w, sets[0], dev, max(1, args.e2e_steps), group)
        e2e_value = job_bytes / (e2e_ms * 1e-3) / 1e9

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(w)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
            "scaling": args.scaling, "vs_baseline": None, "dtype": DTYPE_NAME[w["dtype"]],
            "data": "synthetic: seeded N(0,1) inputs, weight N(1,0.1), bias N(0,0.02)"
                    + (", 1% x100 outliers" if w.get("outliers") else ""),
            "config": {
                "workload": w["desc"], "workload_name": args.workload, "global_rows": sum(all_rows),
                "rows_per_rank": rows, "hidden": w["n"], "heads": h,
                "parallelism": f"dp{world} (row shards, one rank per GPU; {args.scaling} scaling)",
                "grad_allreduce": ar_backend,
                "bytes_per_step_all_ranks": job_bytes, "bytes_per_step_rank0": algo_bytes(w, rows),
                "l2": ("inputs larger than L2" if pool == 1 else f"rotating pool of {pool} input sets > L2"),
                "path": plans if plans else plan,
                "timing": full.how,
            },
            "directions": directions or None,
            "parity": parity,
            "roofline": {"bound": "hbm", "kernel": kern_name, "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": None if (args.rows or args.hidden) else traffic_for(args.workload),
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6.65 TB/s", "kernel_ms": round(kern_ms, 5),
                         "bytes_per_launch": kern_bytes},
            "cpu_baseline": cpu,
            "e2e": None if e2e_value is None else {
                "value": round(e2e_value, 3), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3)},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            # per-config figures of the reference's report: rows/s, per-GPU GB/s, and the
            # fraction of the nominal HBM roofline (N x 8 TB/s)
            "rows_per_s": round(sum(all_rows) / (ms_step * 1e-3), 1),
            "gbs_per_gpu": round(value / world, 2),
            "frac_of_nominal_8tbs": round(value / (8000.0 * world), 4),
        }
    if group is not None:
        import torch.distributed as dist

        torch.cuda.synchronize(dev)
        dist.barrier(group=group)
        if peer_group is not None:
            peer_group.close()
            dist.barrier(group=group)
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    if parity not in ("ok", "skipped"):
        sys.exit(1)


if __name__ == "__main__":
    main()

# SPDX-License-Identifier: MIT
"""Row-grid benchmark CLI with the command-line surface of the reference's
`rmsnorm-benchmark` (rmsnorm/benchmarks/benchmark_rmsnorm.py): the same M x N grid,
presets, gates, filters, pooled inputs, provider order, CSV rows, summary and thresholds.

    python -m rmsnorm.benchmarks.benchmark_rmsnorm [--dtype bfloat16] [--backward]
        [--residual [--residual-out-dtype float32]] [--m M] [--n N] [--pair M,N]
        [--preset NAME | --gate NAME|all] [--warmup W] [--rep R] [--summary]
        [--fail-ratio X] [--min-speedup S] [--output PATH] [--list-presets]

The reference times its kernels against QuACK's autotuned RMSNorm APIs, which are not
available here; the comparator column is instead PyTorch's own fused RMSNorm
(`torch.nn.functional.rms_norm`, and its autograd backward) by default, or -- with
`--reference-root PATH` -- the reference package imported from a checkout at PATH (its
rmsnorm_fwd / rmsnorm_bwd). Times are device times from CUDA events over `rep` calls after
`warmup` calls, inputs rotating through a pool so consecutive calls do not hit in L2.
CSV columns: M,N,pool_size,rmsnorm_ms,ref_ms,ratio,speedup,ref_config with
ratio = rmsnorm_ms / ref_ms and speedup = ref_ms / rmsnorm_ms - 1.
"""

from __future__ import annotations

import argparse
import gc
import math
import sys
from contextlib import redirect_stdout
from pathlib import Path
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch

# The reference's row grid and maintained presets / gates (benchmark_rmsnorm.py:24-64).
MN_PAIRS: List[Tuple[int, int]] = [
    (32768, 256), (32768, 512), (32768, 1024), (32768, 2048), (32768, 4096), (32768, 8192),
    (32768, 16384), (32768, 32768), (32768, 65536), (16384, 131072), (8192, 262144),
]
PRESETS: Dict[str, dict] = {
    "mid-backward": {
        "rows": [(32768, 16384)], "mode": "backward", "gate_dtypes": ("bfloat16", "float16"),
        "fail_ratio": 1.01, "description": "mid-sized backward row with maintained fp16 and bf16 1% ratio gates",
    },
    "large-backward": {
        "rows": [(32768, 65536), (16384, 131072), (8192, 262144)], "mode": "backward",
        "gate_dtypes": ("bfloat16", "float16"), "fail_ratio": 1.01,
        "description": "large backward rows with maintained fp16 and bf16 1% ratio gates",
    },
}
GATE_ALL = "all"
DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}
PROVIDER_ORDERS = ("rmsnorm-first", "ref-first", "balanced")
EPS = 1e-6

Result = Tuple[int, int, Optional[float]]  # (M, N, rmsnorm_ms / ref_ms or None)


def parse_pair(text: str) -> Tuple[int, int]:
    try:
        m, n = (int(v) for v in text.split(","))
    except ValueError as exc:
        raise argparse.ArgumentTypeError("--pair must be formatted as M,N") from exc
    return m, n


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="rmsnorm-benchmark")
    ap.add_argument("--dtype", choices=DTYPES, default=None)
    ap.add_argument("--backward", action="store_true")
    ap.add_argument("--residual", action="store_true")
    ap.add_argument("--residual-out-dtype", choices=("same", "float32"), default="same")
    ap.add_argument("--m", type=int, action="append", help="Only run rows with this M")
    ap.add_argument("--n", type=int, action="append", help="Only run rows with this N")
    ap.add_argument("--pair", type=parse_pair, action="append", help="Run an explicit M,N row (repeatable)")
    ap.add_argument("--preset", choices=sorted(PRESETS), help="Use a maintained row preset")
    ap.add_argument("--gate", choices=sorted(PRESETS) + [GATE_ALL],
                    help="Run a maintained gate over its dtypes and fail ratio ('all': every gate)")
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--rep", type=int, default=100)
    ap.add_argument("--input-pool-size", type=int, default=64,
                    help="Input sets to rotate through during timing (fewer for large rows)")
    ap.add_argument("--pool-memory-fraction", type=float, default=0.80,
                    help="Largest fraction of free device memory the input pool may use")
    ap.add_argument("--provider-order", choices=PROVIDER_ORDERS, default="balanced",
                    help="'balanced' times both orders on fresh pools and averages each provider")
    ap.add_argument("--reference-root", default=None,
                    help="Compare against the reference package imported from this checkout "
                         "(default comparator: torch.nn.functional.rms_norm)")
    ap.add_argument("--output", default=None, help="Write the CSV rows to this path")
    ap.add_argument("--fail-ratio", type=float, default=None,
                    help="Exit nonzero if any row has rmsnorm_ms / ref_ms above this value")
    ap.add_argument("--min-speedup", type=float, default=None,
                    help="Exit nonzero if any row has ref_ms / rmsnorm_ms - 1 below this value")
    ap.add_argument("--summary", action="store_true", help="Print min / geomean / max speedup rows")
    ap.add_argument("--list-presets", action="store_true", help="List the presets and exit")
    return ap


def validate_args(args: argparse.Namespace) -> None:
    if args.list_presets:
        return
    if args.input_pool_size < 1:
        raise ValueError("--input-pool-size must be positive")
    if not 0 < args.pool_memory_fraction <= 1:
        raise ValueError("--pool-memory-fraction must be in (0, 1]")
    if args.gate:
        clash = [flag for flag, used in (
            ("--preset", args.preset is not None), ("--pair", args.pair is not None), ("--m", args.m is not None),
            ("--n", args.n is not None), ("--backward", args.backward), ("--residual", args.residual),
            ("--residual-out-dtype", args.residual_out_dtype != "same"),
            ("--fail-ratio", args.fail_ratio is not None), ("--min-speedup", args.min_speedup is not None),
            ("--dtype", args.dtype is not None)) if used]
        if clash:
            raise ValueError(f"--gate cannot be combined with {', '.join(clash)}")
        return
    if args.backward and args.residual:
        raise ValueError("--residual is only supported for forward benchmarks")
    if args.residual_out_dtype != "same" and not args.residual:
        raise ValueError("--residual-out-dtype requires --residual")
    if args.fail_ratio is not None and args.fail_ratio <= 0:
        raise ValueError("--fail-ratio must be positive")
    if args.min_speedup is not None and args.min_speedup < 0:
        raise ValueError("--min-speedup must be nonnegative")
    if args.preset is not None and PRESETS[args.preset]["mode"] == "backward" and not args.backward:
        raise ValueError(f"--preset {args.preset} requires --backward")


def select_rows(m_values, n_values, pairs, preset) -> List[Tuple[int, int]]:
    if pairs is not None and preset is not None:
        raise ValueError("--pair cannot be combined with --preset")
    rows = pairs or (PRESETS[preset]["rows"] if preset else MN_PAIRS)
    ms, ns = set(m_values or ()), set(n_values or ())
    picked = [(m, n) for m, n in rows if (not ms or m in ms) and (not ns or n in ns)]
    if not picked:
        raise ValueError("no benchmark rows matched the requested filters")
    return picked


def format_presets() -> str:
    lines = ["preset,mode,gate_dtypes,fail_ratio,rows,description"]
    for name in sorted(PRESETS):
        p = PRESETS[name]
        rows = "|".join(f"{m}x{n}" for m, n in p["rows"])
        lines.append(f"{name},{p['mode']},{'|'.join(p['gate_dtypes'])},{p['fail_ratio']:.2f},{rows},"
                     f"{p['description']}")
    return "\n".join(lines)


# ---------------------------------------------------------------------------------------
# Speed-up arithmetic (ratio = ours / comparator)
# ---------------------------------------------------------------------------------------
def speedup(ratio: float) -> float:
    return 1.0 / ratio - 1.0


def summarize(results: Sequence[Result]) -> Optional[dict]:
    ratios = [r for _, _, r in results if r is not None]
    if not ratios:
        return None
    geo = math.exp(sum(math.log(r) for r in ratios) / len(ratios))
    sps = [speedup(r) for r in ratios]
    return {"count": len(ratios), "min": min(sps), "geomean": speedup(geo), "max": max(sps)}


def check_thresholds(results: Sequence[Result], fail_ratio=None, min_speedup=None) -> None:
    comparable = [(m, n, r) for m, n, r in results if r is not None]
    if (fail_ratio is not None or min_speedup is not None) and not comparable:
        raise ValueError("benchmark threshold requested but no comparable rows ran")
    if fail_ratio is not None:
        bad = [(m, n, r) for m, n, r in comparable if r > fail_ratio]
        if bad:
            raise ValueError("benchmark ratio threshold exceeded: " + ", ".join(f"{m}x{n}={r:.4f}" for m, n, r in bad))
    if min_speedup is not None:
        bad = [(m, n, r) for m, n, r in comparable if r > 1.0 / (1.0 + min_speedup)]
        if bad:
            raise ValueError("benchmark speedup threshold not met: "
                             + ", ".join(f"{m}x{n}={speedup(r):.2%}" for m, n, r in bad))


# ---------------------------------------------------------------------------------------
# Providers and timing
# ---------------------------------------------------------------------------------------
def _pool_size(m, n, dtype, backward, residual, requested, fraction) -> int:
    e = m * n * torch.empty((), dtype=dtype).element_size()
    entry = e * (2 if (backward or residual) else 1) + n * 4 + (m * 4 if backward else 0)
    outputs = e * (2 if residual else 1) + (n * 4 if backward else 0)
    free, _ = torch.cuda.mem_get_info()
    budget = int(free * fraction) - 2 * outputs  # both providers' outputs may be live
    return max(1, min(requested, budget // max(entry, 1)))


def _make_pool(m, n, dtype, backward, residual, size) -> List[dict]:
    g = torch.Generator(device="cuda").manual_seed(0)
    pool = []
    for _ in range(size):
        x = torch.randn(m, n, device="cuda", dtype=dtype, generator=g)
        e = {"x": x, "w": torch.randn(n, device="cuda", generator=g)}
        if backward:
            e["dout"] = torch.randn(m, n, device="cuda", dtype=dtype, generator=g)
            e["rstd"] = torch.rsqrt(x.float().square().mean(dim=-1) + EPS)
        elif residual:
            e["residual"] = torch.randn(m, n, device="cuda", dtype=dtype, generator=g)
        pool.append(e)
    return pool


def _ours(backward: bool, residual_dtype) -> Callable[[dict], object]:
    import rmsnorm

    if backward:
        return lambda e: rmsnorm.rmsnorm_bwd(e["x"], e["w"], e["dout"], e["rstd"])
    return lambda e: rmsnorm.rmsnorm_fwd(e["x"], e["w"], residual=e.get("residual"), residual_dtype=residual_dtype)


def _torch_ref(backward: bool, residual_dtype) -> Tuple[Callable[[dict], object], str]:
    """PyTorch's fused RMSNorm (fp32 math on the flattened rows, as the reference computes)."""
    import torch.nn.functional as F

    if backward:
        def step(e):
            x = e["x"].detach().requires_grad_(True)
            w = e["w"].detach().requires_grad_(True)
            y = F.rms_norm(x, (x.shape[-1],), w, EPS)
            y.backward(e["dout"])
            return x.grad, w.grad
        return step, "torch.nn.functional.rms_norm+autograd"

    def step(e):
        x = e["x"]
        if e.get("residual") is not None:
            h = x.float() + e["residual"].float() if residual_dtype == torch.float32 else x + e["residual"]
            y = F.rms_norm(h, (x.shape[-1],), e["w"], EPS).to(x.dtype)
            return y, h
        return F.rms_norm(x, (x.shape[-1],), e["w"], EPS)
    return step, "torch.nn.functional.rms_norm"


def _reference_pkg(root: str, backward: bool, residual_dtype) -> Tuple[Callable[[dict], object], str]:
    """The reference package's own entry points, imported from a checkout at `root`."""
    import importlib.util

    ref = sys.modules.get("_rmsnorm_reference")
    if ref is None:  # loaded under its own name, next to this package's `rmsnorm`
        pkg = Path(root).resolve() / "rmsnorm"
        spec = importlib.util.spec_from_file_location("_rmsnorm_reference", pkg / "__init__.py",
                                                      submodule_search_locations=[str(pkg)])
        ref = importlib.util.module_from_spec(spec)
        sys.modules["_rmsnorm_reference"] = ref
        spec.loader.exec_module(ref)
    if backward:
        return (lambda e: ref.rmsnorm_bwd(e["x"], e["w"], e["dout"], e["rstd"])), f"reference@{root}"
    return (lambda e: ref.rmsnorm_fwd(e["x"], e["w"], residual=e.get("residual"),
                                      residual_dtype=residual_dtype)), f"reference@{root}"


def _time(fn: Callable[[dict], object], pool: List[dict], warmup: int, rep: int) -> float:
    """Mean device time per call (ms) over `rep` calls after `warmup`, rotating the pool."""
    for i in range(warmup):
        fn(pool[i % len(pool)])
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(rep):
        fn(pool[i % len(pool)])
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / rep


def bench_pair(m, n, dtype, args, ref_factory) -> Tuple[float, Optional[float], Optional[str], int, str]:
    """(rmsnorm_ms, ref_ms or None, error or None, pool_size, ref_config) for one row."""
    residual_dtype = torch.float32 if (args.residual and args.residual_out_dtype == "float32") else None
    if args.provider_order == "balanced":
        runs = [bench_pair(m, n, dtype, argparse.Namespace(**{**vars(args), "provider_order": order}), ref_factory)
                for order in ("rmsnorm-first", "ref-first")]
        if any(r[2] is not None for r in runs):
            return runs[0]
        return (sum(r[0] for r in runs) / 2, sum(r[1] for r in runs) / 2, None, min(r[3] for r in runs), runs[0][4])
    gc.collect()
    torch.cuda.empty_cache()
    size = _pool_size(m, n, dtype, args.backward, args.residual, args.input_pool_size, args.pool_memory_fraction)
    pool = _make_pool(m, n, dtype, args.backward, args.residual, size)
    ours = _ours(args.backward, residual_dtype)
    ref, ref_config = ref_factory(args.backward, residual_dtype)
    error = None
    try:
        ref(pool[0])
        torch.cuda.synchronize()
    except (RuntimeError, NotImplementedError, TypeError) as exc:
        error = f"{exc.__class__.__name__}: {str(exc).splitlines()[0] if str(exc) else ''}"
    order = ["ref", "ours"] if args.provider_order == "ref-first" else ["ours", "ref"]
    times = {}
    for who in order:
        if who == "ref" and error is not None:
            continue
        times[who] = _time(ours if who == "ours" else ref, pool, args.warmup, args.rep)
    del pool
    return times["ours"], times.get("ref"), error, size, ref_config


def run_rows(rows, dtype, args, ref_factory, prefix: str = "") -> List[Result]:
    results: List[Result] = []
    for m, n in rows:
        ours, ref, error, size, config = bench_pair(m, n, dtype, args, ref_factory)
        if error is not None or ref is None:
            results.append((m, n, None))
            print(f"{prefix}{m},{n},{size},{ours:.6f},{error},nan,nan,", flush=True)
            continue
        ratio = ours / ref
        results.append((m, n, ratio))
        print(f"{prefix}{m},{n},{size},{ours:.6f},{ref:.6f},{ratio:.4f},{speedup(ratio):.4f},{config}", flush=True)
    return results


def _summary_line(s: Optional[dict], prefix: str = "") -> str:
    if s is None:
        return f"summary,{prefix}0,nan,nan,nan"
    return f"summary,{prefix}{s['count']},{s['min']:.4f},{s['geomean']:.4f},{s['max']:.4f}"


def run(args, parser) -> None:
    try:
        validate_args(args)
    except ValueError as exc:
        parser.error(str(exc))
    if not torch.cuda.is_available():
        parser.exit(2, "rmsnorm-benchmark needs a CUDA device\n")
    if args.reference_root:
        root = args.reference_root
        ref_factory = lambda backward, rd: _reference_pkg(root, backward, rd)  # noqa: E731
    else:
        ref_factory = _torch_ref
    if args.gate:
        print("preset,dtype,M,N,pool_size,rmsnorm_ms,ref_ms,ratio,speedup,ref_config")
        names = sorted(PRESETS) if args.gate == GATE_ALL else [args.gate]
        summaries, errors = [], []
        for name in names:
            p = PRESETS[name]
            for dname in p["gate_dtypes"]:
                gargs = argparse.Namespace(**{**vars(args), "backward": p["mode"] == "backward", "residual": False,
                                              "residual_out_dtype": "same"})
                res = run_rows(p["rows"], DTYPES[dname], gargs, ref_factory, prefix=f"{name},{dname},")
                summaries.append((name, dname, summarize(res)))
                try:
                    check_thresholds(res, fail_ratio=p["fail_ratio"])
                except ValueError as exc:
                    errors.append(f"{name}/{dname}: {exc}")
        if args.summary:
            print("summary,preset,dtype,count,min_speedup,geomean_speedup,max_speedup")
            for name, dname, s in summaries:
                print(_summary_line(s, prefix=f"{name},{dname},"))
        if errors:
            parser.exit(1, "; ".join(errors) + "\n")
        return
    dtype = DTYPES[args.dtype or "bfloat16"]
    try:
        rows = select_rows(args.m, args.n, args.pair, args.preset)
    except ValueError as exc:
        parser.error(str(exc))
    print("M,N,pool_size,rmsnorm_ms,ref_ms,ratio,speedup,ref_config")
    res = run_rows(rows, dtype, args, ref_factory)
    if args.summary:
        print("summary,count,min_speedup,geomean_speedup,max_speedup")
        print(_summary_line(summarize(res)))
    try:
        check_thresholds(res, args.fail_ratio, args.min_speedup)
    except ValueError as exc:
        parser.exit(1, f"{exc}\n")


def main(argv: Optional[Sequence[str]] = None) -> None:
    parser = build_parser()
    args = parser.parse_args(argv)
    if args.list_presets:
        print(format_presets())
        return
    if args.output is None:
        run(args, parser)
        return
    out = Path(args.output)
    out.parent.mkdir(parents=True, exist_ok=True)
    with out.open("w", encoding="utf-8", newline="") as fh, redirect_stdout(fh):
        run(args, parser)


if __name__ == "__main__":
    main()

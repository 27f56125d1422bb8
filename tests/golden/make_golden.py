# SPDX-License-Identifier: MIT
"""Generates tests/golden/*.npz from the REFERENCE package itself.

Run in a container where the reference repository (Int21-AI/RMSNorm-H100) is checked out:
    python tests/golden/make_golden.py path/to/reference
(or with the checkout's path in RMSNORM_REFERENCE_ROOT).
It imports the reference's `rmsnorm` package and runs its own CPU path (rmsnorm_ref,
rmsnorm_fwd / rmsnorm_bwd fallbacks, autograd through RMSNormFunction) on seeded inputs
with the BASELINE distributions, at sizes small enough to commit. The GPU box never runs
this script; tests only read the .npz files it wrote.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
BASE_SEED = 20260514

_CODES = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}


def gen(shape, dtype, seed, kind="normal", outliers=0.0):
    g = torch.Generator().manual_seed(BASE_SEED + seed)
    t = torch.randn(shape, generator=g, dtype=torch.float32)
    if kind == "weight":
        t = 1.0 + 0.1 * t
    elif kind == "bias":
        t = 0.02 * t
    if outliers > 0:
        mask = torch.rand(shape, generator=g) < outliers
        t = torch.where(mask, t * 100.0, t)
    return t.to(dtype)


def save(name: str, meta: dict, tensors: dict) -> None:
    arrays = {}
    dtypes = {}
    for k, t in tensors.items():
        if t is None:
            continue
        t = t.detach().contiguous()
        dtypes[k] = _CODES[t.dtype]
        arrays[k] = (t.view(torch.int16) if t.dtype in (torch.float16, torch.bfloat16) else t).numpy()
    arrays["__meta__"] = np.array(json.dumps({"dtypes": dtypes, **meta}))
    np.savez_compressed(HERE / f"{name}.npz", **arrays)


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import rmsnorm as ref  # the reference package, CPU path

    eps = 1e-6

    # cfg 1 shape family: forward, no residual, bf16 x, fp32 weight (also rstd)
    x = gen((32, 4096), torch.bfloat16, 1)
    w = gen((4096,), torch.float32, 2, "weight")
    out_ref = ref.rmsnorm_ref(x, w, eps=eps)
    out, ro, rstd = ref.rmsnorm_fwd(x, w, eps=eps, store_rstd=True)
    assert torch.equal(out, out_ref) and ro is x
    save("fwd_cfg1", {"eps": eps, "config": "cfg1 family (32x4096 of 8192x4096)"},
         {"x": x, "weight": w, "out": out, "rstd": rstd})

    # cfg 2 family: residual + bias, fp32 residual_out
    x = gen((4, 16384), torch.bfloat16, 3)
    res = gen((4, 16384), torch.bfloat16, 4)
    w = gen((16384,), torch.float32, 5, "weight")
    b = gen((16384,), torch.float32, 6, "bias")
    out, ro, rstd = ref.rmsnorm_fwd(x, w, b, res, residual_dtype=torch.float32, eps=eps, store_rstd=True)
    save("fwd_cfg2", {"eps": eps, "config": "cfg2 family (4x16384 of 32768x16384)"},
         {"x": x, "residual": res, "weight": w, "bias": b, "out": out, "residual_out": ro, "rstd": rstd})

    # cfg 3 family: backward bf16, fp32 weight; rstd from the reference forward
    x = gen((16, 8192), torch.bfloat16, 7)
    dy = gen((16, 8192), torch.bfloat16, 8)
    w = gen((8192,), torch.float32, 9, "weight")
    _, _, rstd = ref.rmsnorm_fwd(x, w, eps=eps, store_rstd=True)
    dx, dw, db, dres = ref.rmsnorm_bwd(x, w, dy, rstd)
    assert db is None and dres is None
    save("bwd_cfg3", {"eps": eps, "config": "cfg3 family (16x8192 of 32768x65536)"},
         {"x": x, "dout": dy, "weight": w, "rstd": rstd, "dx": dx, "dweight": dw})

    # cfg 4 family: per-head weight + bias (QK-norm), fp16, through autograd
    x = gen((8, 32, 128), torch.float16, 10).requires_grad_(True)
    w = gen((32, 128), torch.float32, 11, "weight").requires_grad_(True)
    b = gen((32, 128), torch.float32, 12, "bias").requires_grad_(True)
    dy = gen((8, 32, 128), torch.float16, 13)
    out = ref.rmsnorm(x, w, b, eps=eps)
    (out.float() * dy.float()).sum().backward()
    _, _, rstd = ref.rmsnorm_fwd(x.detach(), w.detach(), b.detach(), eps=eps, store_rstd=True)
    save("perhead_cfg4", {"eps": eps, "config": "cfg4 family (8x32x128 of 16384x32x128)"},
         {"x": x.detach(), "weight": w.detach(), "bias": b.detach(), "dout": dy, "out": out.detach(),
          "rstd": rstd, "dx": x.grad, "dweight": w.grad, "dbias": b.grad})

    # cfg 5 family: very long row with 1% outliers, fp32 and bf16, forward + backward
    for dt, tag in ((torch.float32, "f32"), (torch.bfloat16, "bf16")):
        x = gen((1, 32768), dt, 14, outliers=0.01)
        w = gen((32768,), torch.float32, 15, "weight")
        dy = gen((1, 32768), dt, 16)
        out, _, rstd = ref.rmsnorm_fwd(x, w, eps=eps, store_rstd=True)
        dx, dw, _, _ = ref.rmsnorm_bwd(x, w, dy, rstd)
        save(f"large_cfg5_{tag}", {"eps": eps, "config": "cfg5 family (1x32768 of 1024x262144), 1% outliers"},
             {"x": x, "weight": w, "dout": dy, "out": out, "rstd": rstd, "dx": dx, "dweight": dw})

    # prenorm: fp16 x / residual, fp32 residual_out, gradients of both outputs
    x = gen((4, 512), torch.float16, 17).requires_grad_(True)
    res = gen((4, 512), torch.float16, 18).requires_grad_(True)
    w = gen((512,), torch.float32, 19, "weight").requires_grad_(True)
    dy = gen((4, 512), torch.float16, 20)
    dro = gen((4, 512), torch.float32, 21)
    out, ro = ref.rmsnorm(x, w, residual=res, residual_dtype=torch.float32, prenorm=True, eps=eps)
    ((out.float() * dy.float()).sum() + (ro * dro).sum()).backward()
    save("prenorm_mixed", {"eps": eps, "config": "prenorm, fp32 residual_out, both gradients"},
         {"x": x.detach(), "residual": res.detach(), "weight": w.detach(), "dout": dy,
          "dresidual_out": dro, "out": out.detach(), "residual_out": ro.detach(), "dx": x.grad,
          "dresidual": res.grad, "dweight": w.grad})

    # semantics: out_dtype / residual_dtype honoured, bias without weight, shared 1-D affine on
    # rank-3 input with dbias, mixed-dtype per-head bias (tests/test_rmsnorm_correctness.py:49-366)
    x = gen((3, 16), torch.float32, 22)
    w = gen((16,), torch.float32, 23, "weight")
    out = ref.rmsnorm(x, w, out_dtype=torch.float16, eps=eps)
    save("sem_out_dtype", {"eps": eps}, {"x": x, "weight": w, "out": out})

    x = gen((2, 16), torch.float32, 24).requires_grad_(True)
    b = gen((16,), torch.float32, 25, "bias").requires_grad_(True)
    dy = gen((2, 16), torch.float32, 26)
    out = ref.rmsnorm(x, None, bias=b, eps=eps)
    (out * dy).sum().backward()
    save("sem_bias_only", {"eps": eps}, {"x": x.detach(), "bias": b.detach(), "dout": dy,
                                         "out": out.detach(), "dx": x.grad, "dbias": b.grad})

    x = gen((2, 3, 16), torch.float32, 27)
    w = gen((16,), torch.float32, 28, "weight")
    dy = gen((2, 3, 16), torch.float32, 29)
    rstd = torch.rsqrt(x.square().mean(dim=-1) + eps)
    dx, dw, db, dres = ref.rmsnorm_bwd(x, w, dy, rstd, has_bias=True)
    save("sem_rank3_shared", {"eps": eps}, {"x": x, "weight": w, "dout": dy, "rstd": rstd,
                                            "dx": dx, "dweight": dw, "dbias": db})

    x = gen((2, 3, 16), torch.float32, 30)
    w = gen((3, 16), torch.float32, 31, "weight")
    b = gen((3, 16), torch.float16, 32, "bias")
    dy = gen((2, 3, 16), torch.float32, 33)
    rstd = torch.rsqrt(x.square().mean(dim=-1) + eps)
    dx, dw, db, dres = ref.rmsnorm_bwd(x, w, dy, rstd, has_bias=True, bias=b)
    save("sem_perhead_mixed_bias", {"eps": eps}, {"x": x, "weight": w, "bias": b, "dout": dy, "rstd": rstd,
                                                  "dx": dx, "dweight": dw, "dbias": db})
    make_layernorm(ref, eps)
    print("golden vectors written to", HERE)


def make_layernorm(ref, eps: float) -> None:
    """LayerNorm forward (rmsnorm/rmsnorm.py:655-676) through the reference's layernorm_fwd."""
    x = gen((16, 1024), torch.bfloat16, 40)
    w = gen((1024,), torch.float32, 41, "weight")
    b = gen((1024,), torch.float32, 42, "bias")
    out, rstd, mean = ref.layernorm_fwd(x, w, bias=b, eps=eps, return_rstd=True, return_mean=True)
    save("ln_fwd_bf16", {"eps": eps}, {"x": x, "weight": w, "bias": b, "out": out, "rstd": rstd, "mean": mean})

    # 2-D weight: out normalised over the last two dims, rstd / mean over the last dim
    x = gen((8, 4, 64), torch.float16, 43)
    w = gen((4, 64), torch.float32, 44, "weight")
    out, rstd, mean = ref.layernorm_fwd(x, w, eps=eps, return_rstd=True, return_mean=True)
    save("ln_fwd_2d_weight", {"eps": eps}, {"x": x, "weight": w, "out": out, "rstd": rstd, "mean": mean})

    # fp32 rows of 100 (not a multiple of 8), 1% x100 outliers, rstd only
    x = gen((8, 100), torch.float32, 45, outliers=0.01)
    w = gen((100,), torch.float32, 46, "weight")
    out, rstd = ref.layernorm_fwd(x, w, eps=eps, return_rstd=True)
    save("ln_fwd_f32_n100", {"eps": eps}, {"x": x, "weight": w, "out": out, "rstd": rstd})


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("RMSNORM_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py path/to/reference (or set RMSNORM_REFERENCE_ROOT)")
    main(root)

# SPDX-License-Identifier: MIT
"""ORACLE build recipe -- test/benchmark infrastructure only; the product never loads it.

Compiles the REFERENCE's own CUDA extension (rmsnorm/csrc/torch_bindings.cpp and
rmsnorm/csrc/ptx_rmsnorm_kernels.cu of Int21-AI/RMSNorm-H100, read in place from the
reference checkout) for sm_100a into oracle/_ref/, with the reference's flags
(-O3 --use_fast_math -std=c++17, -lcuda; rmsnorm/_extension.py:37-45) plus an explicit
sm_100a target. The result is the "Hopper kernels recompiled for B200" comparator that
oracle/ref_gpu.py loads on the GPU box. Nothing is copied out of the reference tree; the
build products stay in oracle/_ref/ (git-ignored, travels to the GPU box).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
NAME = "rmsnorm_ref_ext"
# The reference checkout: RMSNORM_REFERENCE_ROOT, else a directory named `reference` next
# to this repository's root (the layout of the build container); absent elsewhere.
DEFAULT_REF = Path(os.environ.get("RMSNORM_REFERENCE_ROOT", str(HERE.parent.parent / "reference")))


def built_path() -> Path:
    import importlib.machinery

    for suf in importlib.machinery.EXTENSION_SUFFIXES:
        p = OUT / f"{NAME}{suf}"
        if p.exists():
            return p
    return OUT / f"{NAME}.so"


def build_if_present(ref_root: Path = DEFAULT_REF) -> Path | None:
    csrc = ref_root / "rmsnorm" / "csrc"
    srcs = [csrc / "torch_bindings.cpp", csrc / "ptx_rmsnorm_kernels.cu"]
    if not all(s.exists() for s in srcs):
        return None
    out = built_path()
    if out.exists() and all(out.stat().st_mtime >= s.stat().st_mtime for s in srcs):
        return out
    OUT.mkdir(parents=True, exist_ok=True)
    from torch.utils.cpp_extension import load

    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    try:
        load(
            name=NAME,
            sources=[str(s) for s in srcs],
            extra_cflags=["-O3", "-std=c++17"],
            extra_cuda_cflags=["-O3", "--use_fast_math", "-std=c++17",
                               "-gencode", "arch=compute_100a,code=sm_100a"],
            extra_ldflags=["-lcuda"],
            build_directory=str(OUT),
            with_cuda=True,
            verbose=False,
        )
    except ImportError:
        # load() imports the module after building; without a driver (no libcuda.so.1 in a
        # CPU-only container) only that import fails, the built .so is complete
        if not built_path().exists():
            raise
    for obj in OUT.glob("*.o"):  # intermediate objects are not needed on the GPU box
        obj.unlink()
    return built_path()


if __name__ == "__main__":
    print(build_if_present(Path(sys.argv[1]) if len(sys.argv) > 1 else DEFAULT_REF))

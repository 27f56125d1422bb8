# SPDX-License-Identifier: MIT
"""The C-ABI library without a GPU: it loads, exports every function include/rmsnorm_b200.h
declares, the ctypes structs match the C layout (compiled probe), and invalid arguments
come back as status codes (no exception crosses the boundary, nothing is launched)."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from rmsnorm import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "rmsnorm_b200.h"


def _declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(rmsnorm_b200_[a-z_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load_library()
    names = _declared_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), f"{name} not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert lib.rmsnorm_b200_abi_version() == _lib.ABI_VERSION


def test_release_and_bounds_checked_builds_identify_themselves():
    """Both builds export the same symbols; only the bounds-checked one says so and keeps
    a report (the release build answers UNSUPPORTED without touching a device)."""
    lib = _lib.load_library()
    assert lib.rmsnorm_b200_debug_bounds_build() == 0
    assert lib.rmsnorm_b200_debug_report(None, None, None, None, None, 0) == 2  # UNSUPPORTED
    debug_path = Path(_lib.__file__).resolve().parent / "lib" / "librmsnorm_b200_debug.so"
    if not debug_path.exists():
        pytest.skip("bounds-checked build not built (__graft_entry__.build() makes it)")
    dbg = ctypes.CDLL(str(debug_path))
    for name in _declared_functions():
        assert hasattr(dbg, name), f"{name} not exported by the bounds-checked build"
    assert dbg.rmsnorm_b200_debug_bounds_build() == 1


def _c_layout(struct_name, fields):
    src = ["#include <stddef.h>", "#include <stdio.h>", f'#include "{HEADER}"', "int main(void) {",
           f'  printf("%zu\\n", sizeof({struct_name}));']
    for f in fields:
        src.append(f'  printf("%zu\\n", offsetof({struct_name}, {f}));')
    src += ["  return 0;", "}"]
    return "\n".join(src)


@pytest.mark.parametrize("cls,cname", [(_lib.FwdArgs, "rmsnorm_b200_fwd_args"),
                                       (_lib.BwdArgs, "rmsnorm_b200_bwd_args"),
                                       (_lib.LnFwdArgs, "rmsnorm_b200_ln_fwd_args")])
def test_ctypes_struct_layout_matches_c(cls, cname, tmp_path):
    fields = [f[0] for f in cls._fields_]
    c = tmp_path / "probe.c"
    c.write_text(_c_layout(cname, fields))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-o", str(exe), str(c)], check=True)
    vals = [int(v) for v in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(cls)
    for name, off in zip(fields, vals[1:]):
        assert getattr(cls, name).offset == off, name


def test_invalid_arguments_return_status_codes():
    lib = _lib.load_library()
    assert lib.rmsnorm_b200_fwd(None, None) == 1
    a = _lib.FwdArgs(rows=-1, hidden=16, heads=1)
    assert lib.rmsnorm_b200_fwd(ctypes.byref(a), None) == 1
    a = _lib.FwdArgs(rows=6, hidden=16, heads=4, x=0x1000, out=0x2000)  # rows % heads != 0
    assert lib.rmsnorm_b200_fwd(ctypes.byref(a), None) == 1
    a = _lib.FwdArgs(rows=4, hidden=16, heads=2, x=0x1000, out=0x2000)  # heads without per-head affine
    assert lib.rmsnorm_b200_fwd(ctypes.byref(a), None) == 1
    a = _lib.FwdArgs(rows=4, hidden=16, heads=1, x=0x1000, out=0x2000, x_dtype=7)
    assert lib.rmsnorm_b200_fwd(ctypes.byref(a), None) == 1
    # zero rows: valid and a no-op (no device needed)
    a = _lib.FwdArgs(rows=0, hidden=16, heads=1, x=0x1000, out=0x2000)
    assert lib.rmsnorm_b200_fwd(ctypes.byref(a), None) == 0
    ln = _lib.LnFwdArgs(rows=4, hidden=16, x=0x1000, out=0x2000, x_dtype=9)
    assert lib.rmsnorm_b200_layernorm_fwd(ctypes.byref(ln), None) == 1
    ln = _lib.LnFwdArgs(rows=4, hidden=0, x=0x1000)
    assert lib.rmsnorm_b200_layernorm_fwd(ctypes.byref(ln), None) == 1
    ln = _lib.LnFwdArgs(rows=0, hidden=16, x=0x1000)
    assert lib.rmsnorm_b200_layernorm_fwd(ctypes.byref(ln), None) == 0
    assert lib.rmsnorm_b200_set_wait_timeout_ns(10) == 1  # below the 1 ms floor: refused on the host
    b = _lib.BwdArgs(rows=4, hidden=16, heads=1)  # null pointers
    assert lib.rmsnorm_b200_bwd(ctypes.byref(b), None, 0, None) == 1
    n = ctypes.c_size_t(123)
    assert lib.rmsnorm_b200_bwd_workspace_size(None, ctypes.byref(n)) == 1
    assert lib.rmsnorm_b200_bwd_workspace_size(ctypes.byref(b), None) == 1
    b = _lib.BwdArgs(rows=4, hidden=16, heads=1, x=0x1000, dout=0x2000, rstd=0x3000, dx=0x4000,
                     dweight=0x5000)  # dweight without weight
    assert lib.rmsnorm_b200_bwd(ctypes.byref(b), None, 0, None) == 1


def test_strerror_strings():
    lib = _lib.load_library()
    assert lib.rmsnorm_b200_strerror(0) == b"ok"
    assert lib.rmsnorm_b200_strerror(1) == b"invalid argument"
    assert b"timed out" in lib.rmsnorm_b200_strerror(5)
    assert lib.rmsnorm_b200_strerror(999) == b"unknown status"


def test_python_layer_raises_on_bad_status():
    with pytest.raises(_lib.LibraryError, match="invalid argument"):
        _lib._check(1, "probe")


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(_lib.LibraryError, match="not found"):
        _lib.load_library(tmp_path / "nope.so")

# SPDX-License-Identifier: MIT
"""ctypes binding of the C ABI in include/rmsnorm_b200.h (librmsnorm_b200.so).

Replaces the reference's JIT loader (rmsnorm/_extension.py:23-45), which compiled the
Hopper kernels with torch.utils.cpp_extension.load at first use. Here the library is
prebuilt for sm_100a by `__graft_entry__.build()` and loaded once; a missing library on a
CUDA call raises instead of falling back to anything else.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path
from typing import Optional

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "librmsnorm_b200.so"

F16, BF16, F32 = 0, 1, 2
_DTYPE_CODES = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32}

OK = 0
ERR_DEVICE_TIMEOUT = 5
ERR_SCRATCH_LIMIT = 7


class FwdArgs(ctypes.Structure):
    _fields_ = [
        ("rows", ctypes.c_int64),
        ("hidden", ctypes.c_int64),
        ("heads", ctypes.c_int32),
        ("x_dtype", ctypes.c_int32),
        ("x", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("residual_dtype", ctypes.c_int32),
        ("weight_dtype", ctypes.c_int32),
        ("weight", ctypes.c_void_p),
        ("weight_heads", ctypes.c_int32),
        ("bias_dtype", ctypes.c_int32),
        ("bias", ctypes.c_void_p),
        ("bias_heads", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("out", ctypes.c_void_p),
        ("residual_out", ctypes.c_void_p),
        ("residual_out_dtype", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("rstd", ctypes.c_void_p),
        ("eps", ctypes.c_float),
        ("reserved1", ctypes.c_int32),
    ]


class BwdArgs(ctypes.Structure):
    _fields_ = [
        ("rows", ctypes.c_int64),
        ("hidden", ctypes.c_int64),
        ("heads", ctypes.c_int32),
        ("x_dtype", ctypes.c_int32),
        ("x", ctypes.c_void_p),
        ("dout", ctypes.c_void_p),
        ("dout_dtype", ctypes.c_int32),
        ("weight_dtype", ctypes.c_int32),
        ("rstd", ctypes.c_void_p),
        ("weight", ctypes.c_void_p),
        ("weight_heads", ctypes.c_int32),
        ("dresidual_out_dtype", ctypes.c_int32),
        ("dresidual_out", ctypes.c_void_p),
        ("dx", ctypes.c_void_p),
        ("dx_dtype", ctypes.c_int32),
        ("dresidual_dtype", ctypes.c_int32),
        ("dresidual", ctypes.c_void_p),
        ("dweight", ctypes.c_void_p),
        ("dweight_dtype", ctypes.c_int32),
        ("dbias_dtype", ctypes.c_int32),
        ("dbias", ctypes.c_void_p),
        ("dbias_heads", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
    ]


# Every symbol include/rmsnorm_b200.h declares, with (restype, argtypes).
class LnFwdArgs(ctypes.Structure):
    _fields_ = [
        ("rows", ctypes.c_int64),
        ("hidden", ctypes.c_int64),
        ("x_dtype", ctypes.c_int32),
        ("weight_dtype", ctypes.c_int32),
        ("x", ctypes.c_void_p),
        ("weight", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("bias_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("out", ctypes.c_void_p),
        ("mean", ctypes.c_void_p),
        ("rstd", ctypes.c_void_p),
        ("eps", ctypes.c_float),
        ("reserved0", ctypes.c_int32),
    ]


SIGNATURES = {
    "rmsnorm_b200_fwd": (ctypes.c_int, [ctypes.POINTER(FwdArgs), ctypes.c_void_p]),
    "rmsnorm_b200_layernorm_fwd": (ctypes.c_int, [ctypes.POINTER(LnFwdArgs), ctypes.c_void_p]),
    "rmsnorm_b200_bwd_workspace_size": (
        ctypes.c_int,
        [ctypes.POINTER(BwdArgs), ctypes.POINTER(ctypes.c_size_t)],
    ),
    "rmsnorm_b200_bwd": (
        ctypes.c_int,
        [ctypes.POINTER(BwdArgs), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p],
    ),
    "rmsnorm_b200_bwd_noalloc": (ctypes.c_int, [ctypes.POINTER(BwdArgs), ctypes.c_void_p]),
    "rmsnorm_b200_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "rmsnorm_b200_device_status": (
        ctypes.c_int,
        [
            ctypes.c_void_p,
            ctypes.POINTER(ctypes.c_int32),
            ctypes.POINTER(ctypes.c_int32),
            ctypes.c_int32,
        ],
    ),
    "rmsnorm_b200_set_wait_timeout_ns": (ctypes.c_int, [ctypes.c_uint64]),
    "rmsnorm_b200_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_uint64, ctypes.c_void_p]),
    "rmsnorm_b200_abi_version": (ctypes.c_int, []),
    "rmsnorm_b200_max_active_clusters": (ctypes.c_int, [ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)]),
    "rmsnorm_b200_launch_count": (ctypes.c_uint64, []),
    "rmsnorm_b200_debug_bounds_build": (ctypes.c_int, []),
    "rmsnorm_b200_debug_report": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_int32),
         ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint32), ctypes.c_int32],
    ),
    "rmsnorm_b200_peer_buffer_size": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int64, ctypes.POINTER(ctypes.c_size_t)]),
    "rmsnorm_b200_peer_group_create": (
        ctypes.c_int,
        [ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)],
    ),
    "rmsnorm_b200_peer_group_connect": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "rmsnorm_b200_peer_group_connect_buffers": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "rmsnorm_b200_peer_group_buffer": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "rmsnorm_b200_peer_group_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "rmsnorm_b200_set_peer_timeout_ns": (ctypes.c_int, [ctypes.c_uint64]),
    "rmsnorm_b200_bwd_allreduce": (
        ctypes.c_int,
        [ctypes.POINTER(BwdArgs), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "rmsnorm_b200_last_plan": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t]),
}

ABI_VERSION = 1

_LIB: Optional[ctypes.CDLL] = None
_LOCK = threading.Lock()


class LibraryError(RuntimeError):
    """Raised when the native library is missing or a call reports a non-zero status."""


def load_library(path: Optional[os.PathLike] = None) -> ctypes.CDLL:
    """Loads librmsnorm_b200.so once and declares every exported signature. The library
    is the in-tree build unless `path` or the RMSNORM_B200_LIBRARY environment variable
    names another build of the same ABI."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    with _LOCK:
        if _LIB is not None and path is None:
            return _LIB
        env_path = os.environ.get("RMSNORM_B200_LIBRARY")
        lib_path = Path(path) if path is not None else (Path(env_path) if env_path else LIB_PATH)
        if not lib_path.exists():
            raise LibraryError(
                f"rmsnorm-b200 native library not found at {lib_path}; build it with "
                "`python -c 'import __graft_entry__ as g; g.build()'` from the repository root"
            )
        lib = ctypes.CDLL(str(lib_path))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if lib.rmsnorm_b200_abi_version() != ABI_VERSION:
            raise LibraryError("rmsnorm-b200 native library ABI version mismatch")
        if path is None:
            _LIB = lib
        return lib


def dtype_code(dtype: torch.dtype) -> int:
    return _DTYPE_CODES[dtype]


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _check(status: int, what: str) -> None:
    if status != OK:
        msg = load_library().rmsnorm_b200_strerror(status).decode()
        raise LibraryError(f"{what} failed with status {status}: {msg}")


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def fwd(
    x: torch.Tensor,
    residual: Optional[torch.Tensor],
    weight: Optional[torch.Tensor],
    weight_heads: int,
    bias: Optional[torch.Tensor],
    bias_heads: int,
    out: torch.Tensor,
    residual_out: Optional[torch.Tensor],
    rstd: Optional[torch.Tensor],
    heads: int,
    eps: float,
) -> None:
    """Enqueues the forward on the current stream of x's device. All tensors contiguous,
    x / residual / out / residual_out viewed as [rows, hidden]."""
    lib = load_library()
    a = FwdArgs()
    a.rows = x.numel() // x.shape[-1]
    a.hidden = x.shape[-1]
    a.heads = heads
    a.x_dtype = _DTYPE_CODES[x.dtype]
    a.x = x.data_ptr()
    if residual is not None:
        a.residual = residual.data_ptr()
        a.residual_dtype = _DTYPE_CODES[residual.dtype]
    if weight is not None:
        a.weight = weight.data_ptr()
        a.weight_dtype = _DTYPE_CODES[weight.dtype]
        a.weight_heads = weight_heads
    if bias is not None:
        a.bias = bias.data_ptr()
        a.bias_dtype = _DTYPE_CODES[bias.dtype]
        a.bias_heads = bias_heads
    a.out = out.data_ptr()
    a.out_dtype = _DTYPE_CODES[out.dtype]
    if residual_out is not None:
        a.residual_out = residual_out.data_ptr()
        a.residual_out_dtype = _DTYPE_CODES[residual_out.dtype]
    if rstd is not None:
        a.rstd = rstd.data_ptr()
    a.eps = eps
    with torch.cuda.device(x.device):
        _check(lib.rmsnorm_b200_fwd(ctypes.byref(a), _stream_handle(x.device)), "rmsnorm_b200_fwd")


def layernorm_fwd(
    x: torch.Tensor,
    hidden: int,
    weight: Optional[torch.Tensor],
    bias: Optional[torch.Tensor],
    out: Optional[torch.Tensor],
    mean: Optional[torch.Tensor],
    rstd: Optional[torch.Tensor],
    eps: float,
) -> None:
    """Enqueues the LayerNorm forward on the current stream of x's device over rows of
    `hidden` elements of the contiguous x (out null = statistics only)."""
    lib = load_library()
    a = LnFwdArgs()
    a.rows = x.numel() // hidden if hidden else 0
    a.hidden = hidden
    a.x_dtype = _DTYPE_CODES[x.dtype]
    a.x = x.data_ptr()
    if weight is not None:
        a.weight = weight.data_ptr()
        a.weight_dtype = _DTYPE_CODES[weight.dtype]
    if bias is not None:
        a.bias = bias.data_ptr()
        a.bias_dtype = _DTYPE_CODES[bias.dtype]
    if out is not None:
        a.out = out.data_ptr()
        a.out_dtype = _DTYPE_CODES[out.dtype]
    if mean is not None:
        a.mean = mean.data_ptr()
    if rstd is not None:
        a.rstd = rstd.data_ptr()
    a.eps = eps
    with torch.cuda.device(x.device):
        _check(lib.rmsnorm_b200_layernorm_fwd(ctypes.byref(a), _stream_handle(x.device)), "rmsnorm_b200_layernorm_fwd")


def bwd_args(
    x: torch.Tensor,
    dout: torch.Tensor,
    rstd: torch.Tensor,
    weight: Optional[torch.Tensor],
    weight_heads: int,
    dresidual_out: Optional[torch.Tensor],
    dx: torch.Tensor,
    dresidual: Optional[torch.Tensor],
    dweight: Optional[torch.Tensor],
    dbias: Optional[torch.Tensor],
    dbias_heads: int,
    heads: int,
) -> BwdArgs:
    a = BwdArgs()
    a.rows = x.numel() // x.shape[-1]
    a.hidden = x.shape[-1]
    a.heads = heads
    a.x = x.data_ptr()
    a.x_dtype = _DTYPE_CODES[x.dtype]
    a.dout = dout.data_ptr()
    a.dout_dtype = _DTYPE_CODES[dout.dtype]
    a.rstd = rstd.data_ptr()
    if weight is not None:
        a.weight = weight.data_ptr()
        a.weight_dtype = _DTYPE_CODES[weight.dtype]
        a.weight_heads = weight_heads
    if dresidual_out is not None:
        a.dresidual_out = dresidual_out.data_ptr()
        a.dresidual_out_dtype = _DTYPE_CODES[dresidual_out.dtype]
    a.dx = dx.data_ptr()
    a.dx_dtype = _DTYPE_CODES[dx.dtype]
    if dresidual is not None:
        a.dresidual = dresidual.data_ptr()
        a.dresidual_dtype = _DTYPE_CODES[dresidual.dtype]
    if dweight is not None:
        a.dweight = dweight.data_ptr()
        a.dweight_dtype = _DTYPE_CODES[dweight.dtype]
    if dbias is not None:
        a.dbias = dbias.data_ptr()
        a.dbias_dtype = _DTYPE_CODES[dbias.dtype]
        a.dbias_heads = dbias_heads
    return a


def bwd_workspace_bytes(a: BwdArgs, device: torch.device) -> int:
    lib = load_library()
    n = ctypes.c_size_t(0)
    with torch.cuda.device(device):
        _check(lib.rmsnorm_b200_bwd_workspace_size(ctypes.byref(a), ctypes.byref(n)),
               "rmsnorm_b200_bwd_workspace_size")
    return int(n.value)


def bwd(a: BwdArgs, device: torch.device, workspace: Optional[torch.Tensor] = None, peer_group=None) -> None:
    """Enqueues the backward; allocates the workspace from the caching allocator unless
    one is given. With `peer_group` (a handle from peer_group_create), dweight / dbias are
    summed over the group's ranks by rmsnorm_b200_bwd_allreduce."""
    lib = load_library()
    nbytes = bwd_workspace_bytes(a, device)
    if nbytes and (workspace is None or workspace.numel() < nbytes):
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=device)
    ws_ptr = workspace.data_ptr() if (workspace is not None and nbytes) else None
    with torch.cuda.device(device):
        if peer_group is None:
            _check(lib.rmsnorm_b200_bwd(ctypes.byref(a), ws_ptr, nbytes, _stream_handle(device)), "rmsnorm_b200_bwd")
        else:
            _check(lib.rmsnorm_b200_bwd_allreduce(ctypes.byref(a), ws_ptr, nbytes, peer_group,
                                                   _stream_handle(device)), "rmsnorm_b200_bwd_allreduce")


IPC_HANDLE_BYTES = 64


def peer_group_create(device: torch.device, rank: int, world: int, max_grad_floats: int):
    """(handle, ipc_handle bytes) of this rank's member of a peer group on `device`."""
    lib = load_library()
    h = ctypes.c_void_p()
    ipc = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    with torch.cuda.device(device):
        _check(lib.rmsnorm_b200_peer_group_create(rank, world, max_grad_floats, ipc, ctypes.byref(h)),
               "rmsnorm_b200_peer_group_create")
    return h.value, ipc.raw


def peer_group_connect(device: torch.device, handle, ipc_handles) -> None:
    """Maps the other ranks' buffers (ipc_handles: one bytes object per rank, rank order)."""
    buf = ctypes.create_string_buffer(b"".join(ipc_handles), IPC_HANDLE_BYTES * len(ipc_handles))
    with torch.cuda.device(device):
        _check(load_library().rmsnorm_b200_peer_group_connect(handle, buf), "rmsnorm_b200_peer_group_connect")


def peer_group_connect_buffers(device: torch.device, handle, buffers) -> None:
    """Connects with device pointers for each rank's buffer (rank order; own entry ignored)."""
    arr = (ctypes.c_void_p * len(buffers))(*[b or 0 for b in buffers])
    with torch.cuda.device(device):
        _check(load_library().rmsnorm_b200_peer_group_connect_buffers(handle, arr),
               "rmsnorm_b200_peer_group_connect_buffers")


def peer_group_buffer(handle) -> int:
    p = ctypes.c_void_p()
    _check(load_library().rmsnorm_b200_peer_group_buffer(handle, ctypes.byref(p)), "rmsnorm_b200_peer_group_buffer")
    return int(p.value)


def peer_group_destroy(device: torch.device, handle) -> None:
    with torch.cuda.device(device):
        _check(load_library().rmsnorm_b200_peer_group_destroy(handle), "rmsnorm_b200_peer_group_destroy")


def set_peer_timeout_ns(device: torch.device, ns: int) -> None:
    with torch.cuda.device(device):
        _check(load_library().rmsnorm_b200_set_peer_timeout_ns(ns), "rmsnorm_b200_set_peer_timeout_ns")


def bwd_noalloc(a: BwdArgs, device: torch.device) -> int:
    """Backward through the entry point that allocates nothing (the library's built-in
    scratch buffer replaces the workspace). Returns the status code."""
    with torch.cuda.device(device):
        return int(load_library().rmsnorm_b200_bwd_noalloc(ctypes.byref(a), _stream_handle(device)))


def device_status(device: torch.device, clear: bool = False) -> tuple:
    """(status, site) of the device status word, read in stream order."""
    lib = load_library()
    st = ctypes.c_int32(0)
    wh = ctypes.c_int32(0)
    with torch.cuda.device(device):
        _check(
            lib.rmsnorm_b200_device_status(
                _stream_handle(device), ctypes.byref(st), ctypes.byref(wh), int(clear)
            ),
            "rmsnorm_b200_device_status",
        )
    return int(st.value), int(wh.value)


def set_wait_timeout_ns(device: torch.device, ns: int) -> None:
    with torch.cuda.device(device):
        _check(load_library().rmsnorm_b200_set_wait_timeout_ns(ns), "rmsnorm_b200_set_wait_timeout_ns")


def selftest_wait_timeout(device: torch.device, ns: int) -> None:
    with torch.cuda.device(device):
        _check(
            load_library().rmsnorm_b200_selftest_wait_timeout(ns, _stream_handle(device)),
            "rmsnorm_b200_selftest_wait_timeout",
        )


def max_active_clusters(device: torch.device, cluster_size: int) -> int:
    n = ctypes.c_int32(0)
    with torch.cuda.device(device):
        _check(load_library().rmsnorm_b200_max_active_clusters(cluster_size, ctypes.byref(n)),
               "rmsnorm_b200_max_active_clusters")
    return int(n.value)


def launch_count() -> int:
    return int(load_library().rmsnorm_b200_launch_count())


def debug_bounds_build() -> bool:
    """True for the bounds-checked build (librmsnorm_b200_debug.so)."""
    return bool(load_library().rmsnorm_b200_debug_bounds_build())


def debug_report(device: torch.device, clear: bool = False) -> dict:
    """Failed bounds checks since the last clear (bounds-checked build only): count and the
    first one's site code, address and size. Synchronises the current stream."""
    lib = load_library()
    n = ctypes.c_uint64(0)
    site = ctypes.c_int32(0)
    addr = ctypes.c_uint64(0)
    nbytes = ctypes.c_uint32(0)
    with torch.cuda.device(device):
        _check(
            lib.rmsnorm_b200_debug_report(_stream_handle(device), ctypes.byref(n), ctypes.byref(site),
                                          ctypes.byref(addr), ctypes.byref(nbytes), int(clear)),
            "rmsnorm_b200_debug_report",
        )
    return {"violations": int(n.value), "site": int(site.value), "address": int(addr.value), "bytes": int(nbytes.value)}


def last_plan() -> str:
    buf = ctypes.create_string_buffer(512)
    load_library().rmsnorm_b200_last_plan(buf, len(buf))
    return buf.value.decode()

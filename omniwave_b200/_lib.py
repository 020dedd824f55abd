"""ctypes binding of ``libomniwave_b200.so`` (the C ABI in include/omniwave_b200.h).

This module is the Python side of the drop-in boundary: it mirrors the C
structs field for field and calls the library with raw device pointers taken
from torch tensors.  It never computes anything itself; if the library is
missing it raises instead of falling back.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libomniwave_b200.so")
ABI_VERSION = 5

DTYPE_CODE = {
    torch.float32: 0,
    torch.float64: 1,
    torch.bfloat16: 2,
    torch.float16: 3,
}

OW_OK = 0
_ERR_NAMES = {1: "invalid argument", 2: "unsupported", 3: "CUDA error", 4: "workspace too small"}

_c_i32 = ctypes.c_int32
_vp = ctypes.c_void_p


class Route(ctypes.Structure):
    _fields_ = [
        ("batch", _c_i32), ("height", _c_i32), ("width", _c_i32), ("channels", _c_i32),
        ("q_s", _c_i32), ("q_c", _c_i32), ("g", _c_i32), ("d", _c_i32), ("rd", _c_i32),
        ("tok_idx", _vp), ("ch_idx", _vp), ("ch_stride", _c_i32),
    ]


class Args(ctypes.Structure):
    _fields_ = [
        ("route", Route),
        ("x", _vp), ("x_dtype", _c_i32), ("compute_dtype", _c_i32),
        ("rstd", _vp), ("norm_w", _vp),
        ("a_u", _vp), ("a_v", _vp), ("a_o", _vp),
        ("b_u", _vp), ("b_v", _vp), ("b_o", _vp),
        ("gamma", _vp), ("w_dtype", _c_i32),
        ("sample_scale", _vp), ("residual", _c_i32),
        ("out", _vp), ("out_dtype", _c_i32),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
    ]


class Grads(ctypes.Structure):
    _fields_ = [
        ("dout", _vp), ("dx", _vp),
        ("da_u", _vp), ("da_v", _vp), ("da_o", _vp),
        ("db_u", _vp), ("db_v", _vp), ("db_o", _vp),
        ("dgamma", _vp), ("dnorm_w", _vp),
    ]


class S2dLinear(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("x_dtype", _c_i32), ("layout", _c_i32),
        ("batch", _c_i32), ("height", _c_i32), ("width", _c_i32), ("channels", _c_i32),
        ("factor", _c_i32),
        ("weight", _vp), ("w_dtype", _c_i32), ("out_features", _c_i32),
        ("out", _vp), ("out_dtype", _c_i32),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
    ]


class D2sLinear(ctypes.Structure):
    _fields_ = [
        ("y", _vp), ("y_dtype", _c_i32),
        ("batch", _c_i32), ("height", _c_i32), ("width", _c_i32), ("channels", _c_i32),
        ("factor", _c_i32), ("in_features", _c_i32),
        ("weight", _vp), ("w_dtype", _c_i32),
        ("out", _vp), ("out_dtype", _c_i32),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
    ]


class PoolHead(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("x_dtype", _c_i32),
        ("batch", _c_i32), ("tokens", _c_i32), ("channels", _c_i32),
        ("weight", _vp), ("w_dtype", _c_i32),
        ("bias", _vp), ("bias_dtype", _c_i32),
        ("classes", _c_i32), ("compute_dtype", _c_i32),
        ("out", _vp), ("pooled", _vp),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
    ]


LAYOUT_NHWC = 0
LAYOUT_NCHW = 1

EXPORTS = (
    "ow_abi_version", "ow_last_error", "ow_device_supported", "ow_device_fault",
    "ow_launch_count", "ow_bigemm_workspace_size",
    "ow_rmsnorm_rstd", "ow_bigemm_fwd", "ow_bigemm_bwd", "ow_bigemm_fwd_noalloc",
    "ow_noalloc_scratch_limit", "ow_profile_events", "ow_debug_wait_probe",
    "ow_s2d_linear_workspace_size", "ow_s2d_linear_fwd",
    "ow_pool_head_workspace_size", "ow_pool_head_fwd",
    "ow_d2s_linear_workspace_size", "ow_d2s_linear_fwd",
)

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class NativeLibraryError(RuntimeError):
    """The CUDA library is missing or failed a call."""


def load() -> ctypes.CDLL:
    """Load the library once (thread-safe) and declare the prototypes."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise NativeLibraryError(
                f"{LIB_PATH} is missing; build it with `python -m omniwave_b200.build`"
            )
        lib = ctypes.CDLL(LIB_PATH)
        lib.ow_abi_version.restype = ctypes.c_int
        lib.ow_last_error.restype = ctypes.c_char_p
        lib.ow_device_supported.argtypes = [ctypes.c_int]
        lib.ow_device_supported.restype = ctypes.c_int
        lib.ow_device_fault.argtypes = [ctypes.c_int, ctypes.c_int]
        lib.ow_device_fault.restype = ctypes.c_int
        lib.ow_launch_count.restype = ctypes.c_uint64
        lib.ow_debug_wait_probe.argtypes = [ctypes.c_uint32]
        lib.ow_debug_wait_probe.restype = ctypes.c_int
        lib.ow_profile_events.argtypes = [ctypes.c_int, _vp, _vp]
        lib.ow_profile_events.restype = ctypes.c_int
        lib.ow_bigemm_workspace_size.argtypes = [ctypes.POINTER(Args), ctypes.c_int]
        lib.ow_bigemm_workspace_size.restype = ctypes.c_size_t
        lib.ow_rmsnorm_rstd.argtypes = [_vp, _c_i32, _c_i32, ctypes.c_int64, _c_i32,
                                        ctypes.c_double, _vp, _vp]
        lib.ow_rmsnorm_rstd.restype = ctypes.c_int
        lib.ow_bigemm_fwd.argtypes = [ctypes.POINTER(Args), _vp]
        lib.ow_bigemm_fwd.restype = ctypes.c_int
        lib.ow_bigemm_fwd_noalloc.argtypes = [ctypes.POINTER(Args), _vp]
        lib.ow_bigemm_fwd_noalloc.restype = ctypes.c_int
        lib.ow_noalloc_scratch_limit.restype = ctypes.c_size_t
        lib.ow_bigemm_bwd.argtypes = [ctypes.POINTER(Args), ctypes.POINTER(Grads), _vp]
        lib.ow_bigemm_bwd.restype = ctypes.c_int
        lib.ow_s2d_linear_workspace_size.argtypes = [ctypes.POINTER(S2dLinear)]
        lib.ow_s2d_linear_workspace_size.restype = ctypes.c_size_t
        lib.ow_s2d_linear_fwd.argtypes = [ctypes.POINTER(S2dLinear), _vp]
        lib.ow_s2d_linear_fwd.restype = ctypes.c_int
        lib.ow_pool_head_workspace_size.argtypes = [ctypes.POINTER(PoolHead)]
        lib.ow_pool_head_workspace_size.restype = ctypes.c_size_t
        lib.ow_pool_head_fwd.argtypes = [ctypes.POINTER(PoolHead), _vp]
        lib.ow_pool_head_fwd.restype = ctypes.c_int
        lib.ow_d2s_linear_workspace_size.argtypes = [ctypes.POINTER(D2sLinear)]
        lib.ow_d2s_linear_workspace_size.restype = ctypes.c_size_t
        lib.ow_d2s_linear_fwd.argtypes = [ctypes.POINTER(D2sLinear), _vp]
        lib.ow_d2s_linear_fwd.restype = ctypes.c_int
        v = lib.ow_abi_version()
        if v != ABI_VERSION:
            raise NativeLibraryError(f"ABI version mismatch: library {v}, binding {ABI_VERSION}")
        _lib = lib
        return lib


def check(status: int, what: str) -> None:
    if status != OW_OK:
        msg = load().ow_last_error().decode(errors="replace")
        raise NativeLibraryError(f"{what} failed ({_ERR_NAMES.get(status, status)}): {msg}")


class DeviceFaultError(RuntimeError):
    """A kernel of the library gave up on a bounded wait (its outputs are undefined)."""


def device_fault(device: int, reset: bool = False) -> int:
    """The device fault word (0: no kernel gave up on a wait).  Synchronises the device."""
    return int(load().ow_device_fault(int(device), 1 if reset else 0))


def check_device_fault(device: int, reset: bool = True) -> None:
    """Raise ``DeviceFaultError`` if a kernel on ``device`` gave up on a bounded wait."""
    v = device_fault(device, reset)
    if v != 0:
        raise DeviceFaultError(f"omniwave_b200 kernel on device {device} reported fault code {v} "
                               f"(a bounded wait ran out; outputs of that call are undefined)")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream

"""The C-ABI library: loads, exports every function include/omniwave_b200.h
declares, and its host-side argument checking (no GPU needed: every case
here fails validation before any CUDA call)."""

from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

from omniwave_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "omniwave_b200.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"OW_API\s+[\w\s\*]+?\b(ow_\w+)\s*\(", src)))


def test_header_declares_the_bound_functions():
    assert set(_declared()) == set(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True)
    exported = set(re.findall(r" T (ow_\w+)", out.stdout))
    assert set(_declared()) <= exported
    assert all(s.startswith("ow_") for s in exported)


def test_abi_version_and_counters():
    lib = _lib.load()
    assert lib.ow_abi_version() == _lib.ABI_VERSION
    lib.ow_launch_count.restype = ctypes.c_uint64
    assert lib.ow_launch_count() >= 0


def test_profile_events_checks_kernel_id():
    lib = _lib.load()
    assert lib.ow_profile_events(7, None, None) == 1  # OW_ERR_INVALID
    assert "unknown kernel" in lib.ow_last_error().decode()
    for k in (0, 1, 2, 3):  # NULL events: recording off, nothing touches CUDA
        assert lib.ow_profile_events(k, None, None) == 0


def _args(**over):
    r = _lib.Route(2, 14, 14, 512, 13, 4, 16, 128, 256, 1, 1)
    a = _lib.Args(r, 1, 2, 2, None, None, 1, 1, 1, 1, 1, 1, 1, 0, None, 0, 1, 2, None, 0)
    for k, v in over.items():
        if hasattr(a.route, k) and k not in ("x",):
            setattr(a.route, k, v)
        else:
            setattr(a, k, v)
    return a


@pytest.mark.parametrize("field,value,msg", [
    ("g", 8, "spatial tile g must be 16"),
    ("q_s", 12, "does not match ceil"),
    ("q_c", 3, "does not match ceil"),
    ("x_dtype", 9, "invalid dtype"),
    ("batch", 0, "must be positive"),
])
def test_invalid_arguments_rejected_without_gpu(field, value, msg):
    lib = _lib.load()
    a = _args(**{field: value})
    st = lib.ow_bigemm_fwd(ctypes.byref(a), None)
    assert st == 1
    assert msg in lib.ow_last_error().decode()
    assert lib.ow_bigemm_workspace_size(ctypes.byref(a), 0) == 0


def test_workspace_is_required():
    lib = _lib.load()
    a = _args()
    assert lib.ow_bigemm_workspace_size(ctypes.byref(a), 1) > 0
    st = lib.ow_bigemm_fwd(ctypes.byref(a), None)
    assert st == 4 and "workspace" in lib.ow_last_error().decode()


def test_null_pointers_rejected():
    lib = _lib.load()
    a = _args(a_u=None)
    assert lib.ow_bigemm_fwd(ctypes.byref(a), None) == 1
    g = _lib.Grads()
    assert lib.ow_bigemm_bwd(ctypes.byref(_args()), ctypes.byref(g), None) == 1
    assert "gradient pointer" in lib.ow_last_error().decode()


def test_device_query_without_gpu_is_safe():
    import torch

    lib = _lib.load()
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert lib.ow_device_supported(0) == 0

"""The allocation-free forward entry point, ow_bigemm_fwd_noalloc.

Callers that cannot allocate device memory when they run the operator (a
plugin host that hands over only input and output buffers, code that must not
enter the process's allocator) use this entry point: its scratch is a fixed
array inside the library, not a caller workspace.  These tests call it through
the C ABI and check, on two calls in a row, that it gives the same result as
ow_bigemm_fwd with a workspace: within the tolerance the other parity tests
use (2e-2 relative for bf16 compute, 1e-4 for fp32), and in fact bitwise,
since both run the same kernels on the same inputs.  Between the two checked
calls a call on a different problem leaves other data in the shared scratch,
so nothing relies on the scratch starting out zeroed or unchanged.  The file is named so that
pytest collects it last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _case(dev, h, w, c, d, b, dtype, route="shifted", level=0, seed=0):
    from omniwave_b200 import build_route_plan
    from omniwave_b200.ops import _make_args, _weights_common, route_tables

    g = torch.Generator().manual_seed(seed)
    qc = c // d
    x = torch.randn(b, h, w, c, generator=g).to(dev, dtype)
    ws = [torch.randn(16, 16, generator=g) / 4 for _ in range(3)]
    ws += [torch.randn(qc, d, 2 * d, generator=g) / d ** 0.5 for _ in range(2)]
    ws += [torch.randn(qc, 2 * d, d, generator=g) / (2 * d) ** 0.5, torch.randn(c, generator=g)]
    weights, wdt = _weights_common([t.to(dev, dtype) for t in ws])
    plan = build_route_plan(h, w, c, 16, d, route, level)
    tok, ch = route_tables(plan, dev)

    def make_args(out):
        return _make_args(x, plan, tok, ch, weights, wdt, dtype, None, None, None, False, out, out.dtype)

    keep = (x, weights, tok, ch)
    return make_args, keep


def _workspace_forward(lib, make_args, out, stream):
    from omniwave_b200 import _lib

    a = make_args(out)
    n = lib.ow_bigemm_workspace_size(ctypes.byref(a), 0)
    wsb = torch.empty(n, dtype=torch.uint8, device=out.device)
    a.workspace, a.workspace_bytes = wsb.data_ptr(), n
    _lib.check(lib.ow_bigemm_fwd(ctypes.byref(a), stream), "ow_bigemm_fwd")
    return wsb


def _noalloc_forward(lib, make_args, out, stream):
    from omniwave_b200 import _lib

    a = make_args(out)
    _lib.check(lib.ow_bigemm_fwd_noalloc(ctypes.byref(a), stream), "ow_bigemm_fwd_noalloc")


def _run_pair(dev, dtype, shape, tol):
    from omniwave_b200 import _lib

    lib = _lib.load()
    h, w, c, d, b = shape
    make_args, keep = _case(dev, h, w, c, d, b, dtype)
    # A different problem (batch, route, weights) whose call leaves other data
    # in the shared scratch between the two checked calls.
    other_args, other_keep = _case(dev, h, w, c, d, max(1, b // 2), dtype, route="radix", level=1, seed=7)
    stream = _lib.stream_handle(dev)
    ref = torch.empty(b, h, w, c, device=dev, dtype=dtype)
    wsb = _workspace_forward(lib, make_args, ref, stream)
    outs = []
    for i in range(2):  # two checked calls in a row share the static scratch
        o = torch.full((b, h, w, c), float("nan"), device=dev, dtype=dtype)
        _noalloc_forward(lib, make_args, o, stream)
        outs.append(o)
        if i == 0:
            junk = torch.full((max(1, b // 2), h, w, c), float("nan"), device=dev, dtype=dtype)
            _noalloc_forward(lib, other_args, junk, stream)
    torch.cuda.synchronize(dev)
    r = ref.double().cpu().numpy()
    for o in outs:
        on = o.double().cpu().numpy()
        assert np.isfinite(on).all()
        assert rel_err(on, r) <= tol
        # Same kernels on the same inputs: the results are bitwise equal.
        assert torch.equal(o, ref)
    assert lib.ow_device_fault(dev.index or 0, 0) == 0
    del keep, other_keep, wsb


def test_noalloc_matches_workspace_forward_bf16(cuda_device):
    _run_pair(cuda_device, torch.bfloat16, (14, 14, 512, 128, 4), 2e-2)


def test_noalloc_matches_workspace_forward_fp32(cuda_device):
    _run_pair(cuda_device, torch.float32, (28, 28, 256, 64, 2), 1e-4)


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda_device):
    from omniwave_b200 import _lib

    lib = _lib.load()
    limit = lib.ow_noalloc_scratch_limit()
    assert limit == 4 << 20
    # float64 compute keeps f64 weight copies in scratch: 2048 channels need ~12.6 MB.
    make_args, keep = _case(cuda_device, 8, 8, 2048, 128, 1, torch.float64)
    out = torch.empty(1, 8, 8, 2048, device=cuda_device, dtype=torch.float64)
    a = make_args(out)
    assert lib.ow_bigemm_workspace_size(ctypes.byref(a), 0) > limit
    st = lib.ow_bigemm_fwd_noalloc(ctypes.byref(a), _lib.stream_handle(cuda_device))
    assert st == 4
    assert "limit" in lib.ow_last_error().decode()
    del keep

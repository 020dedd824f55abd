"""Global average pool + classifier head (host side, no GPU).

The fused head (``omniwave_b200.head``) must differentiate as autograd
differentiates the reference's ``head(stage4.mean(dim=(1, 2)))``
(backbone.py:193-197), its C entry point must validate its arguments without
touching CUDA, and the installed ``forward`` keeps the reference path for
host tensors.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import rel_err

from omniwave_b200 import _lib, head

F32, BF16, F16 = 0, 2, 3


def test_backward_matches_autograd_of_the_reference_ops():
    """float64 on the host: the algebra alone, no rounding in the way."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(3, 4, 5, 16, generator=g, dtype=torch.float64, requires_grad=True)
    w = torch.randn(7, 16, generator=g, dtype=torch.float64, requires_grad=True)
    b = torch.randn(7, generator=g, dtype=torch.float64, requires_grad=True)
    y = torch.nn.functional.linear(x.mean(dim=(1, 2)), w, b)
    dy = torch.randn(y.shape, generator=g, dtype=torch.float64)
    want = torch.autograd.grad(y, [x, w, b], dy)
    pooled = x.detach().mean(dim=(1, 2))
    got = head.pool_head_backward(dy, pooled, w.detach(), tuple(x.shape), torch.float64, torch.float64,
                                  torch.float64)
    for name, a, e in zip(("dx", "dW", "db"), got, want):
        assert a.shape == e.shape, name
        assert rel_err(a.numpy(), e.numpy()) <= 1e-12, name
    none = head.pool_head_backward(dy, None, w.detach(), tuple(x.shape), torch.float64, None, torch.float64,
                                   (True, False, True))
    assert none[1] is None and none[2] is None  # no weight gradient asked, no bias


def _args(**over):
    a = _lib.PoolHead(None, F32, 256, 49, 1024, None, F32, None, F32, 1000, BF16, None, None, None, 0)
    for k, v in over.items():
        setattr(a, k, v)
    return a


def test_workspace_query_and_validation_without_gpu():
    lib = _lib.load()
    assert lib.ow_pool_head_workspace_size(ctypes.byref(_args())) == 1000 * 1024 * 2 + 256
    assert lib.ow_pool_head_workspace_size(ctypes.byref(_args(w_dtype=BF16, x_dtype=BF16))) == 256
    for over, msg in (({"channels": 768}, "multiple of 512"),
                      ({"channels": 2560}, "multiple of 512"),
                      ({"classes": 1025}, "at most 1024"),
                      ({"compute_dtype": F32}, "compute dtype"),
                      ({"x_dtype": F16}, "x dtype"),
                      ({"batch": 0}, "must be positive")):
        a = _args(**over)
        assert lib.ow_pool_head_workspace_size(ctypes.byref(a)) == 0, over
        assert lib.ow_pool_head_fwd(ctypes.byref(a), None) == 2  # OW_ERR_UNSUPPORTED
        assert msg in lib.ow_last_error().decode(), over
    # supported arguments with a NULL tensor: rejected before any CUDA call
    assert lib.ow_pool_head_fwd(ctypes.byref(_args()), None) == 1  # OW_ERR_INVALID
    assert "NULL" in lib.ow_last_error().decode()


def test_pool_head_refuses_host_tensors():
    x, w = torch.zeros(1, 7, 7, 512), torch.zeros(10, 512)
    assert head.pool_head_supported(x, w) == (False, "CUDA is unavailable")
    with pytest.raises(RuntimeError, match="CUDA is unavailable"):
        head.pool_head(x, w)


def test_installed_forward_is_patched_and_keeps_the_host_path(omniweave):
    from omniweave.models.backbone import OmniWeaveBackbone
    from omniweave.models.registry import create_model

    assert OmniWeaveBackbone.forward.__qualname__.endswith("install.<locals>.forward")
    torch.manual_seed(3)
    model = create_model("omniweave_t", input_size=64, layer_scale_init=0.5).eval()
    x = torch.randn(2, 3, 64, 64)
    with torch.no_grad():
        feats = model.forward_features(x)
        want = model.head(feats["stage4"].mean(dim=(1, 2)))
        assert torch.equal(model(x), want)

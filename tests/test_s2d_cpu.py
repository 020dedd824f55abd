"""Stem / downsample projections (host side, no GPU).

The fused space-to-depth GEMM (``omniwave_b200.s2d``) must rearrange exactly
as the reference's ``space_to_depth_nhwc`` (backbone.py:14-27), and its
backward -- the folded-anchor algebra ``dW_d = W_a^T dW``, ``dW_a = dW W_d^T``
with ``dW = dy^T s2d(x)`` -- must give the gradients autograd takes through
the reference's two ``nn.Linear`` layers.  The installed
``forward_features`` keeps the reference path for host tensors.
"""

from __future__ import annotations

import pytest
import torch

from conftest import load_golden, rel_err

from omniwave_b200 import s2d


def test_space_to_depth_matches_reference_and_inverts(omniweave):
    from omniweave.models.backbone import space_to_depth_nhwc as ref

    g = torch.Generator().manual_seed(0)
    for shape, f in (((2, 8, 12, 5), 2), ((1, 16, 8, 3), 4), ((3, 4, 4, 64), 2)):
        x = torch.randn(*shape, generator=g)
        y = s2d.space_to_depth_nhwc(x, f)
        assert torch.equal(y, ref(x, f))
        assert torch.equal(s2d.depth_to_space_nhwc(y, f), x)
    with pytest.raises(ValueError, match="divisible"):
        s2d.space_to_depth_nhwc(torch.zeros(1, 6, 8, 2), 4)


@pytest.mark.parametrize("nchw,anchor", [(True, False), (True, True), (False, False), (False, True)],
                         ids=["stem", "stem+anchor", "downsample", "downsample+anchor"])
def test_folded_backward_matches_autograd_of_the_reference_layers(omniweave, nchw, anchor):
    """float64 on the host: the algebra alone, no rounding in the way."""
    from omniweave.models.backbone import space_to_depth_nhwc as ref_s2d

    g = torch.Generator().manual_seed(1)
    f, c, n = (4, 3, 16) if nchw else (2, 8, 24)
    shape = (2, c, 8, 12) if nchw else (2, 8, 12, c)
    x = torch.randn(*shape, generator=g, dtype=torch.float64, requires_grad=True)
    wd = torch.randn(n, f * f * c, generator=g, dtype=torch.float64, requires_grad=True)
    wa = torch.randn(n, n, generator=g, dtype=torch.float64, requires_grad=True) if anchor else None
    xn = x.permute(0, 2, 3, 1) if nchw else x
    y = torch.nn.functional.linear(ref_s2d(xn, f), wd)
    if wa is not None:
        y = torch.nn.functional.linear(y, wa)
    dy = torch.randn(y.shape, generator=g, dtype=torch.float64)
    params = [x, wd] + ([wa] if wa is not None else [])
    want = torch.autograd.grad(y, params, dy)
    w_eff = (wa @ wd if wa is not None else wd).detach()
    got = s2d.s2d_linear_backward(dy, x.detach(), wd.detach(), None if wa is None else wa.detach(),
                                  w_eff, f, nchw, torch.float64)
    # the folded forward is the same map
    y_fold = torch.nn.functional.linear(ref_s2d(xn, f), w_eff)
    assert rel_err(y_fold.detach().numpy(), y.detach().numpy()) <= 1e-12
    for name, a, b in zip(("dx", "dW_d", "dW_a"), got, want):
        assert a.shape == b.shape, name
        assert rel_err(a.numpy(), b.numpy()) <= 1e-12, name


def test_installed_forward_features_keeps_the_reference_path_on_the_host(omniweave):
    from omniweave.models.backbone import OmniWeaveBackbone
    from omniweave.models.registry import create_model

    assert OmniWeaveBackbone.forward_features.__qualname__.endswith("install.<locals>.forward_features")
    torch.manual_seed(5)
    model = create_model("omniweave_t", input_size=64, layer_scale_init=0.5).eval()
    z = load_golden("model_f32")
    x = torch.from_numpy(z["inp"])
    assert s2d.features_supported(model, x) == (False, "stem: CUDA is unavailable")
    with torch.no_grad():
        logits = model(x)
    assert rel_err(logits.numpy(), z["logits"]) <= 1e-5


def test_s2d_linear_refuses_host_tensors():
    with pytest.raises(RuntimeError, match="CUDA is unavailable"):
        s2d.s2d_linear(torch.zeros(1, 4, 4, 64), torch.zeros(256, 256), 2)


def test_d2s_linear_validation_without_gpu():
    """The depth-to-space entry point sizes and refuses without touching CUDA."""
    import ctypes

    from omniwave_b200 import _lib

    lib = _lib.load()
    F32, BF16, F16 = 0, 2, 3

    def args(**over):
        a = _lib.D2sLinear(None, BF16, 2, 56, 56, 128, 2, 256, None, BF16, None, F32, None, 0)
        for k, v in over.items():
            setattr(a, k, v)
        return a

    assert lib.ow_d2s_linear_workspace_size(ctypes.byref(args())) == 512 * 256 * 2 + 256
    for over, msg in (({"y_dtype": F32}, "y dtype"), ({"channels": 96}, "multiple of 64"),
                      ({"in_features": 200}, "multiple of 64"), ({"out_dtype": F16}, "out dtype"),
                      ({"width": 57}, "divisible"), ({"factor": 1}, "multiple of 256"),
                      ({"width": 512, "channels": 64}, "at most 128")):
        a = args(**over)
        assert lib.ow_d2s_linear_workspace_size(ctypes.byref(a)) == 0, over
        assert lib.ow_d2s_linear_fwd(ctypes.byref(a), None) == 2  # OW_ERR_UNSUPPORTED
        assert msg in lib.ow_last_error().decode(), over
    assert lib.ow_d2s_linear_fwd(ctypes.byref(args()), None) == 1  # NULL pointers: OW_ERR_INVALID
    with pytest.raises(RuntimeError, match="CUDA is unavailable"):
        s2d.d2s_linear(torch.zeros(1, 4, 4, 256, dtype=torch.bfloat16), torch.zeros(256, 256), 2)

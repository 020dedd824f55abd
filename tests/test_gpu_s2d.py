"""Fused space-to-depth projections on the GPU (stem and downsamples).

``ow_s2d_linear_fwd`` against ``Linear(space_to_depth(x))`` computed by the
reference's own rearrangement in float64 from the same 16-bit-rounded
operands: the kernel's only differences are its f32 accumulation order and
the final rounding to bf16/f16, so each output must lie within 1.5 ulp of
the output dtype (plus an absolute floor for near-zero sums).  Shapes cover
the OmniWeave-T stem (224 -> 56x56x128) and all three downsamples, partial
last tiles, the widest supported rows (W/f = 128) and f16.  The model-level
tests compare the reference backbone with the installed cuda path against
the reference backend under bf16 autocast (outputs and every gradient within
the north star's 2e-2 of max|ref|).
"""

from __future__ import annotations

import copy

import pytest
import torch

from conftest import rel_err

from omniwave_b200 import _lib, s2d

pytestmark = pytest.mark.gpu


def _exact(x, w, f, nchw, dtype):
    """float64 Linear(s2d(x)) from the operands rounded to ``dtype``."""
    xn = x.permute(0, 2, 3, 1) if nchw else x
    a = s2d.space_to_depth_nhwc(xn.to(dtype).double(), f)
    return a @ w.to(dtype).double().t()


def _check_ulp(out, exact, dtype):
    eps = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11
    err = (out.double() - exact).abs()
    bound = 1.5 * eps * exact.abs() + 1e-6 * exact.abs().max()
    bad = (err > bound).sum().item()
    assert bad == 0, f"{bad} outputs beyond 1.5 ulp; worst {(err - bound).max().item():.3e}"


@pytest.mark.parametrize("b,hw,n,xdt,dtype", [
    (2, 224, 128, torch.float32, torch.bfloat16),   # the stem of OmniWeave-T
    (3, 64, 256, torch.float32, torch.bfloat16),    # two feature tiles, partial last row tile
    (1, 32, 512, torch.bfloat16, torch.bfloat16),   # bf16 images, four resident weight tiles
    (2, 48, 128, torch.float32, torch.float16),
], ids=["stem224", "n256-partial", "bf16-n512", "f16"])
def test_stem_matches_exact(cuda_device, b, hw, n, xdt, dtype):
    g = torch.Generator(device=cuda_device).manual_seed(0)
    x = torch.randn(b, 3, hw, hw, device=cuda_device, generator=g).to(xdt)
    w = torch.randn(n, 48, device=cuda_device, generator=g) * 0.2
    with torch.autocast("cuda", dtype=dtype):
        out = s2d.s2d_linear(x, w, 4, nchw=True)
    assert out.dtype == dtype and out.shape == (b, hw // 4, hw // 4, n)
    _check_ulp(out, _exact(x, w, 4, True, dtype), dtype)


@pytest.mark.parametrize("b,h,c,n,dtype", [
    (2, 56, 128, 256, torch.bfloat16),    # downsample 1 of OmniWeave-T
    (3, 28, 256, 512, torch.bfloat16),    # downsample 2, 9 rows of 14 per tile, partial last tile
    (5, 14, 512, 1024, torch.bfloat16),   # downsample 3, 18 rows of 7 per tile
    (1, 256, 64, 256, torch.bfloat16),    # W / f = 128: one output row per tile
    (2, 200, 64, 256, torch.bfloat16),    # W / f = 100: 100-row tiles
    (3, 28, 128, 256, torch.float16),
], ids=["ds1", "ds2-partial", "ds3", "wo128", "wo100", "f16"])
def test_downsample_matches_exact(cuda_device, b, h, c, n, dtype):
    g = torch.Generator(device=cuda_device).manual_seed(1)
    x = torch.randn(b, h, h, c, device=cuda_device, generator=g).to(dtype)
    w = torch.randn(n, 4 * c, device=cuda_device, generator=g) * (4 * c) ** -0.5
    out = s2d.s2d_linear(x, w, 2)
    assert out.dtype == dtype and out.shape == (b, h // 2, h // 2, n)
    _check_ulp(out, _exact(x, w, 2, False, dtype), dtype)


@pytest.mark.parametrize("b,h", [(3, 28), (2, 14), (1, 200)])
def test_downsample_with_identity_weight_is_the_rearrangement(cuda_device, b, h):
    """weight = I: the output is space_to_depth(x) bit for bit (every row, every k, once)."""
    c = 64 if h == 200 else 128
    x = torch.randn(b, h, h, c, device=cuda_device).bfloat16()
    out = s2d.s2d_linear(x, torch.eye(4 * c, device=cuda_device), 2)
    assert torch.equal(out, s2d.space_to_depth_nhwc(x, 2))


def test_stem_with_identity_weight_is_the_rearrangement(cuda_device):
    x = torch.randn(3, 3, 40, 56, device=cuda_device)
    w = torch.zeros(128, 48, device=cuda_device)
    w[:48] = torch.eye(48, device=cuda_device)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = s2d.s2d_linear(x, w, 4, nchw=True)
    want = s2d.space_to_depth_nhwc(x.permute(0, 2, 3, 1), 4).bfloat16()
    assert torch.equal(out[..., :48], want)
    assert not out[..., 48:].any()


@pytest.mark.parametrize("b,h,c,n,dtype,odt", [
    (2, 56, 128, 256, torch.bfloat16, torch.float32),    # downsample 1's input gradient, f32 stream
    (3, 28, 256, 512, torch.bfloat16, torch.float32),    # downsample 2, partial last tile
    (5, 14, 512, 1024, torch.bfloat16, torch.bfloat16),  # downsample 3, 16-bit out
    (1, 256, 64, 256, torch.bfloat16, torch.float32),    # W / f = 128: one row per tile
    (3, 28, 128, 256, torch.float16, torch.float16),
], ids=["ds1-f32", "ds2-partial", "ds3-bf16", "wo128", "f16"])
def test_depth_to_space_linear_matches_exact(cuda_device, b, h, c, n, dtype, odt):
    """depth_to_space(y W) against float64 from the same rounded operands:
    within 1.5 ulp of the compute dtype (f32 out holds the compute-type
    rounding, as the reference's autocast backward does)."""
    g = torch.Generator(device=cuda_device).manual_seed(4)
    y = torch.randn(b, h // 2, h // 2, n, device=cuda_device, generator=g).to(dtype)
    w = torch.randn(n, 4 * c, device=cuda_device, generator=g) * n ** -0.5
    out = s2d.d2s_linear(y, w, 2, out_dtype=odt)
    assert out.dtype == odt and out.shape == (b, h, h, c)
    exact = s2d.depth_to_space_nhwc(y.double() @ w.to(dtype).double(), 2)
    _check_ulp(out, exact, dtype)
    if odt == torch.float32:  # exactly the compute-type values
        assert torch.equal(out, out.to(dtype).float())
    # the downsample backward takes it and agrees with the PyTorch path
    x = torch.randn(b, h, h, c, device=cuda_device, generator=g)
    dx, _, _ = s2d.s2d_linear_backward(y, x, w, None, w, 2, False, dtype, (True, False, False), odt)
    assert torch.equal(dx, out.to(odt))


def test_anchor_fold_matches_two_linears(cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(2)
    x = torch.randn(4, 28, 28, 256, device=cuda_device, generator=g).bfloat16()
    wd = torch.randn(512, 1024, device=cuda_device, generator=g) * 1024 ** -0.5
    wa = torch.randn(512, 512, device=cuda_device, generator=g) * 512 ** -0.5
    out = s2d.s2d_linear(x, wd, 2, anchor=wa)
    a = s2d.space_to_depth_nhwc(x.double(), 2)
    exact = a @ (wa.double() @ wd.double()).t()
    assert rel_err(out.double().cpu().numpy(), exact.cpu().numpy()) <= 1e-2


def test_unsupported_shapes_are_refused(cuda_device):
    x = torch.zeros(1, 8, 8, 96, dtype=torch.bfloat16, device=cuda_device)
    ok, why = s2d.s2d_linear_supported(x, torch.zeros(256, 384, device=cuda_device), 2)
    assert not ok
    with pytest.raises(RuntimeError, match="not supported"):
        s2d.s2d_linear(x, torch.zeros(256, 384, device=cuda_device), 2)
    x32 = torch.zeros(1, 8, 8, 128, device=cuda_device)
    assert s2d.s2d_linear_supported(x32, torch.zeros(256, 512, device=cuda_device), 2)[0] is False


def _model(backend, dev, seed=5, size=64):
    from omniweave.models.registry import create_model

    torch.manual_seed(seed)
    return create_model("omniweave_t", input_size=size, layer_scale_init=0.5, backend=backend).to(dev)


@pytest.mark.parametrize("size", [64, 224])
def test_backbone_features_and_grads_match_reference_backend(omniweave, cuda_device, size):
    """Features and logits within 2e-2 of the reference backend under the same
    bf16 autocast.  Whole-model weight gradients go through every layer's
    rounding, so they are held to the reference's own bf16 error: against the
    reference in float32, the cuda model's error is at most
    max(2e-2, 1.5 x the reference bf16 run's error)."""
    ref = _model("reference", cuda_device, size=size)
    cud = _model("cuda", cuda_device, size=size)
    g = torch.Generator(device=cuda_device).manual_seed(3)
    x = torch.randn(2, 3, size, size, device=cuda_device, generator=g)
    assert s2d.features_supported(cud, x) == (False, "stem: compute dtype torch.float32 is not 16-bit")
    y = torch.randint(0, 1000, (2,), device=cuda_device, generator=g)
    res = []
    for m, amp in ((ref, False), (ref, True), (cud, True)):
        n0 = _lib.load().ow_launch_count()
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=amp):
            if m is cud:
                assert s2d.features_supported(m, x) == (True, None)
            feats = m.forward_features(x)
            logits = m.head(feats["stage4"].mean(dim=(1, 2)))
            loss = torch.nn.functional.cross_entropy(logits, y)
        grads = torch.autograd.grad(loss, list(m.parameters()))
        res.append((feats, logits.detach(), grads, _lib.load().ow_launch_count() - n0))
    (_, _, g32, _), (fr, lr_, gr, _), (fc, lc, gc, launched) = res
    assert launched > 0
    for k in fr:
        assert fc[k].dtype == fr[k].dtype, k
        assert rel_err(fc[k].float().detach().cpu().numpy(), fr[k].float().detach().cpu().numpy()) <= 2e-2, k
    assert rel_err(lc.float().cpu().numpy(), lr_.float().cpu().numpy()) <= 2e-2
    names = [n for n, _ in ref.named_parameters()]
    for n, a, b, t in zip(names, gc, gr, g32):
        assert a.dtype == b.dtype, n
        own = rel_err(b.cpu().numpy(), t.cpu().numpy())
        assert rel_err(a.cpu().numpy(), t.cpu().numpy()) <= max(2e-2, 1.5 * own), n


def test_bf16_model_runs_fused_projections(omniweave, cuda_device):
    """A bf16 model (no autocast) takes bf16 images straight into the stem kernel."""
    ref = _model("reference", cuda_device).bfloat16().eval()
    cud = copy.deepcopy(ref)
    for m in cud.modules():
        if type(m).__name__ == "OmniWeaveBlock":
            m.backend = "cuda"
    x = torch.randn(2, 3, 64, 64, device=cuda_device).bfloat16()
    assert s2d.features_supported(cud, x) == (True, None)
    with torch.no_grad():
        a, b = cud(x), ref(x)
    assert rel_err(a.float().cpu().numpy(), b.float().cpu().numpy()) <= 2e-2

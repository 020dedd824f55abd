"""Fused global average pool + classifier head on the GPU.

``ow_pool_head_fwd`` against float64 arithmetic on the same rounded
operands: the pooled means it writes must be the float64 means rounded to the
compute dtype (within one ulp: its f32 token sum may round the other way
near a tie), and each logit must match the float64 product of those pooled
values with the rounded weight plus the rounded bias within 1.5 ulp of the
output dtype (plus a floor for sums that cancel, relative to sum |p w|).
Shapes cover the OmniWeave-T tail at inference (bf16, 256 images, 32-slot
clusters) and training (f32 features and weight under autocast, 128 images,
16-slot clusters), partial clusters, one token, 196 tokens, the widest
channels and every class-tile count.  The model-level test runs the
reference backbone's whole forward (fused stem, blocks, downsamples, pool
and head) against the reference backend under bf16 autocast.
"""

from __future__ import annotations

import pytest
import torch

from conftest import rel_err

from omniwave_b200 import _lib, head

pytestmark = pytest.mark.gpu

BF, HF, F32 = torch.bfloat16, torch.float16, torch.float32


def _eps(dtype):
    return 2.0 ** -8 if dtype == BF else 2.0 ** -11


@pytest.mark.parametrize("b,h,c,n,xdt,wdt,bias,compute", [
    (256, 7, 1024, 1000, BF, BF, True, BF),     # OmniWeave-T inference tail
    (128, 7, 1024, 1000, F32, F32, True, BF),   # training tail under autocast
    (5, 7, 512, 37, HF, HF, True, HF),          # one partial cluster, one class tile
    (21, 1, 2048, 1024, BF, F32, False, BF),    # one token, widest rows, eight class tiles, no bias
    (3, 14, 1536, 129, F32, BF, True, BF),      # 196 tokens, three chunks per CTA, ragged last tile
    (1000, 2, 512, 300, BF, BF, True, BF),      # more images than one wave holds at 32 per cluster
], ids=["t-infer", "t-train", "f16-small", "wide", "tokens196", "waves"])
def test_pool_head_matches_float64(cuda_device, b, h, c, n, xdt, wdt, bias, compute):
    g = torch.Generator(device=cuda_device).manual_seed(0)
    x = torch.randn(b, h, h, c, device=cuda_device, generator=g).to(xdt)
    w = (torch.randn(n, c, device=cuda_device, generator=g) * c ** -0.5).to(wdt)
    bv = torch.randn(n, device=cuda_device, generator=g) * 0.1 if bias else None
    with torch.autocast("cuda", dtype=compute):
        assert head.pool_head_supported(x, w, bv) == (True, None)
        n0 = _lib.load().ow_launch_count()
        out, pooled = head._fwd(x, w, bv, compute, want_pooled=True)
        assert _lib.load().ow_launch_count() > n0
        out2, none = head._fwd(x, w, bv, compute, want_pooled=False)
        logits = head.pool_head(x, w, bv)
    _lib.check_device_fault(cuda_device.index or 0)
    assert out.dtype == compute and out.shape == (b, n) and pooled.shape == (b, c) and none is None
    # bitwise reproducible, with or without the pooled output, and through the autograd entry
    assert torch.equal(out, out2) and torch.equal(out, logits)
    eps = _eps(compute)
    mean = x.double().mean(dim=(1, 2))
    perr = (pooled.double() - mean).abs()
    assert (perr <= 2 * eps * mean.abs() + 1e-5 * mean.abs().max()).all(), perr.max().item()
    wd = w.to(compute).double()
    exact = pooled.double() @ wd.t()
    mag = pooled.double().abs() @ wd.abs().t()
    if bias:
        exact = exact + bv.to(compute).double()
    err = (out.double() - exact).abs()
    bound = 1.5 * eps * exact.abs() + 2e-5 * mag
    assert (err <= bound).all(), f"{(err > bound).sum().item()} logits off; worst {(err - bound).max().item():.3e}"


def test_pool_head_gradients_follow_autograd_of_the_reference_ops(cuda_device):
    """dx, dW, db of the fused head against autograd through the reference's
    mean + nn.Linear under the same autocast (same roundings, within 1e-2)."""
    g = torch.Generator(device=cuda_device).manual_seed(1)
    x = torch.randn(12, 7, 7, 1024, device=cuda_device, generator=g, requires_grad=True)
    lin = torch.nn.Linear(1024, 1000).to(cuda_device)
    dy = torch.randn(12, 1000, device=cuda_device, generator=g)
    res = []
    for fused in (False, True):
        with torch.autocast("cuda", dtype=BF):
            y = head.pool_head(x, lin.weight, lin.bias) if fused else lin(x.mean(dim=(1, 2)))
        res.append((y, torch.autograd.grad(y, [x, lin.weight, lin.bias], dy.to(y.dtype))))
    (yr, gr), (yf, gf) = res
    assert yf.dtype == yr.dtype
    assert rel_err(yf.float().detach().cpu().numpy(), yr.float().detach().cpu().numpy()) <= 1e-2
    for name, a, e in zip(("dx", "dW", "db"), gf, gr):
        assert a.dtype == e.dtype and a.shape == e.shape, name
        assert rel_err(a.float().cpu().numpy(), e.float().cpu().numpy()) <= 1e-2, name


def _model(backend, dev, seed=5, size=64):
    from omniweave.models.registry import create_model

    torch.manual_seed(seed)
    return create_model("omniweave_t", input_size=size, layer_scale_init=0.5, backend=backend).to(dev)


def test_model_forward_and_grads_match_reference_backend(omniweave, cuda_device):
    """The installed ``OmniWeaveBackbone.forward`` (fused projections, blocks,
    pool and head) against the reference backend, both under bf16 autocast:
    logits within 2e-2, every gradient within max(2e-2, 1.5 x the reference
    bf16 run's own error against float32)."""
    ref = _model("reference", cuda_device)
    cud = _model("cuda", cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(3)
    x = torch.randn(10, 3, 64, 64, device=cuda_device, generator=g)
    y = torch.randint(0, 1000, (10,), device=cuda_device, generator=g)
    res = []
    for m, amp in ((ref, False), (ref, True), (cud, True)):
        with torch.autocast("cuda", dtype=BF, enabled=amp):
            logits = m(x)
            loss = torch.nn.functional.cross_entropy(logits, y)
        res.append((logits.detach(), torch.autograd.grad(loss, list(m.parameters()))))
    (_, g32), (lr_, gr), (lc, gc) = res
    assert lc.dtype == lr_.dtype
    assert rel_err(lc.float().cpu().numpy(), lr_.float().cpu().numpy()) <= 2e-2
    for (n, _), a, b, t in zip(ref.named_parameters(), gc, gr, g32):
        assert a.dtype == b.dtype, n
        own = rel_err(b.cpu().numpy(), t.cpu().numpy())
        assert rel_err(a.cpu().numpy(), t.cpu().numpy()) <= max(2e-2, 1.5 * own), n

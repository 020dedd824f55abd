"""The reference's own modules on the cuda backend (GPU).

After ``omniwave_b200.integration.install()`` the reference package's
``OmniWeaveBlock``, ``OmniWeaveBackbone`` (``create_model``) and training
engine (``train_one_epoch``) run unchanged with ``backend="cuda"``.  These
tests compare them against the same modules with ``backend="reference"``
(the reference's einsum implementation, TF32 off) on identical seeded
inputs: fp32 within 1e-4 and bf16 autocast within 2e-2 of max|ref|, the
north star's tolerances, for outputs and every gradient; and they check that
checkpoints interchange between the two backends.
"""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

from conftest import load_golden, rel_err

pytestmark = pytest.mark.gpu

PARAMS = ("norm_weight", "a_u", "a_v", "a_o", "b_u", "b_v", "b_o", "gamma")


def _pair(omniweave, dev, shape, route, seed=0, scale=0.5):
    from omniweave.models.block import OmniWeaveBlock

    h, w, c, d = shape
    torch.manual_seed(seed)
    ref = OmniWeaveBlock(h, w, c, d, route[0], route[1], layer_scale_init=scale).to(dev)
    cud = copy.deepcopy(ref)
    cud.backend = "cuda"
    return ref, cud


def _fwd_bwd(blk, x, dy, amp):
    x = x.clone().requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=amp):
        out = blk(x)
    grads = torch.autograd.grad(out, [x] + [getattr(blk, k) for k in PARAMS], dy.to(out.dtype))
    return out.detach(), grads


@pytest.mark.parametrize("shape,route", [((14, 14, 512, 128), ("radix", 1)),
                                         ((28, 28, 256, 64), ("shifted", 0)),
                                         ((7, 7, 1024, 128), ("radix", 2))],
                         ids=["14x14x512-radix1", "28x28x256-shifted", "7x7x1024-radix2"])
@pytest.mark.parametrize("amp", [False, True], ids=["fp32", "bf16-autocast"])
def test_reference_block_on_cuda_matches_reference_backend(omniweave, cuda_device, shape, route, amp):
    ref, cud = _pair(omniweave, cuda_device, shape, route)
    g = torch.Generator(device=cuda_device).manual_seed(1)
    x = torch.randn(3, *shape[:3], device=cuda_device, generator=g)
    dy = torch.randn(3, *shape[:3], device=cuda_device, generator=g)
    o_r, g_r = _fwd_bwd(ref, x, dy, amp)
    o_c, g_c = _fwd_bwd(cud, x, dy, amp)
    tol = 2e-2 if amp else 1e-4
    assert o_c.dtype == o_r.dtype
    assert rel_err(o_c.cpu().numpy(), o_r.cpu().numpy()) <= tol
    if amp:
        # The delta alone (x dominates the block output).  Only meaningful
        # where the check's own cancellation error, ulp(x) / max|delta|, is
        # far below the tolerance: under autocast, not at 1e-4 in fp32.
        assert rel_err((o_c - x).cpu().numpy(), (o_r - x).cpu().numpy()) <= tol
    for name, a, b in zip(("x",) + PARAMS, g_c, g_r):
        assert a.dtype == b.dtype, name
        assert rel_err(a.cpu().numpy(), b.cpu().numpy()) <= tol, name


def _model(backend, dev, seed=5, **kw):
    from omniweave.models.registry import create_model

    torch.manual_seed(seed)
    return create_model("omniweave_t", input_size=64, layer_scale_init=0.5, backend=backend, **kw).to(dev)


def test_reference_model_on_cuda_matches_golden_logits(omniweave, cuda_device):
    z = load_golden("model_f32")
    model = _model("cuda", cuda_device).eval()
    with torch.no_grad():
        logits = model(torch.from_numpy(z["inp"]).to(cuda_device))
    assert rel_err(logits.cpu().numpy(), z["logits"]) <= 1e-4


def test_reference_model_gradients_cuda_vs_reference(omniweave, cuda_device):
    ref = _model("reference", cuda_device)
    cud = _model("cuda", cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(3)
    x = torch.randn(2, 3, 64, 64, device=cuda_device, generator=g)
    y = torch.randint(0, 1000, (2,), device=cuda_device, generator=g)
    res = []
    for m in (ref, cud):
        loss = torch.nn.functional.cross_entropy(m(x), y)
        grads = torch.autograd.grad(loss, list(m.parameters()))
        res.append((loss.detach(), grads))
    assert rel_err(res[1][0].cpu().numpy(), res[0][0].cpu().numpy()) <= 1e-4
    names = [n for n, _ in ref.named_parameters()]
    worst = max((rel_err(a.cpu().numpy(), b.cpu().numpy()), n)
                for n, a, b in zip(names, res[1][1], res[0][1]))
    assert worst[0] <= 1e-3, worst


def test_checkpoints_interchange_on_gpu(omniweave, cuda_device):
    """Weights trained on one backend load into the other and give the same logits."""
    src = _model("cuda", cuda_device)
    opt = torch.optim.AdamW(src.parameters(), lr=1e-3)
    g = torch.Generator(device=cuda_device).manual_seed(4)
    x = torch.randn(2, 3, 64, 64, device=cuda_device, generator=g)
    y = torch.randint(0, 1000, (2,), device=cuda_device, generator=g)
    loss = torch.nn.functional.cross_entropy(src(x), y)
    loss.backward()
    opt.step()
    dst = _model("reference", cuda_device, seed=99)
    dst.load_state_dict(src.state_dict(), strict=True)
    src.eval()
    dst.eval()
    with torch.no_grad():
        assert rel_err(src(x).cpu().numpy(), dst(x).cpu().numpy()) <= 1e-4
    back = _model("cuda", cuda_device, seed=98).eval()
    back.load_state_dict(dst.state_dict(), strict=True)
    with torch.no_grad():
        assert torch.equal(back(x), src(x))


def test_reference_training_engine_runs_the_cuda_model(omniweave, cuda_device):
    """engine.train_one_epoch (unchanged) with EMA, clipping and bf16 autocast."""
    from omniweave.training.engine import EMAModel, train_one_epoch

    g = torch.Generator().manual_seed(6)
    loader = [(torch.randn(4, 3, 64, 64, generator=g), torch.randint(0, 1000, (4,), generator=g))
              for _ in range(2)]
    out = {}
    for backend in ("reference", "cuda"):
        m = _model(backend, cuda_device)
        opt = torch.optim.AdamW(m.parameters(), lr=1e-3, weight_decay=0.05)
        ema = EMAModel(m, decay=0.9)
        metrics = train_one_epoch(m, loader, opt, cuda_device, epoch=0, ema=ema, amp_enabled=True)
        out[backend] = (metrics, m)
    mr, mc = out["reference"][0], out["cuda"][0]
    assert mc["steps"] == 2 and mc["non_finite_events"] == 0
    assert np.isfinite(mc["train_loss"])
    assert abs(mc["train_loss"] - mr["train_loss"]) <= 2e-2 * abs(mr["train_loss"])


def test_trainstep_cuda_graph_matches_eager(omniweave, cuda_device):
    """The whole train step as one CUDA graph gives the eager step's results."""
    from omniwave_b200.train import TrainStep

    g = torch.Generator(device=cuda_device).manual_seed(8)
    batches = [(torch.randn(4, 3, 64, 64, device=cuda_device, generator=g),
                torch.randint(0, 1000, (4,), device=cuda_device, generator=g)) for _ in range(6)]
    runs = []
    for graph in (False, True):
        m = _model("cuda", cuda_device, seed=11)
        ts = TrainStep(m, ema_decay=0.99, clip_norm=1.0, cuda_graph=graph, graph_warmup=2)
        losses = [ts.step(x, y).clone() for x, y in batches]
        ts.check_finite()
        runs.append((torch.stack(losses), [p.detach().clone() for p in m.parameters()], ts.ema.state_dict()))
    (le, pe, ee), (lg, pg, eg) = runs
    assert rel_err(lg.cpu().numpy(), le.cpu().numpy()) <= 1e-5
    for a, b in zip(pg, pe):
        assert rel_err(a.cpu().numpy(), b.cpu().numpy()) <= 1e-4
    for k in ee:
        assert rel_err(eg[k].float().cpu().numpy(), ee[k].float().cpu().numpy()) <= 1e-4, k


def test_trainstep_skips_nonfinite_step_on_gpu(omniweave, cuda_device):
    from omniwave_b200.train import TrainStep

    m = _model("cuda", cuda_device)
    ts = TrainStep(m, ema_decay=0.9)
    before = [p.detach().clone() for p in m.parameters()]
    x = torch.full((2, 3, 64, 64), float("nan"), device=cuda_device)
    ts.step(x, torch.zeros(2, dtype=torch.long, device=cuda_device))
    assert all(torch.equal(p.detach(), b) for p, b in zip(m.parameters(), before))
    with pytest.raises(FloatingPointError):
        ts.check_finite()


def test_full_size_bf16_inference_and_train_step(omniweave, cuda_device):
    from omniweave.models.registry import create_model

    torch.manual_seed(0)
    model = create_model("omniweave_t", backend="cuda").to(cuda_device)
    x = torch.randn(4, 3, 224, 224, device=cuda_device)
    with torch.no_grad():
        m16 = copy.deepcopy(model).to(torch.bfloat16).eval()
        out = m16(x.to(torch.bfloat16))
    assert out.shape == (4, 1000) and torch.isfinite(out).all()
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3, weight_decay=0.05)
    labels = torch.randint(0, 1000, (4,), device=cuda_device)
    losses = []
    for _ in range(3):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = torch.nn.functional.cross_entropy(model(x), labels)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        losses.append(float(loss))
    assert all(np.isfinite(losses))
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in model.parameters())

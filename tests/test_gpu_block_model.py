"""Fused block on the GPU against golden vectors and the oracle.

Forward and all gradients of ``OmniWeaveBlock`` (RMSNorm prologue, residual
epilogue fused) against the reference's autograd (fp64 case; tolerance 1e-6
because the reference takes the RMS variance in float32), bf16 autocast and
drop-path scales.  The reference's own modules on the cuda backend are in
test_gpu_integration.py.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden, rel_err
from oracle import bigemm as O

pytestmark = pytest.mark.gpu

PARAMS = ("norm_weight", "a_u", "a_v", "a_o", "b_u", "b_v", "b_o", "gamma")


def _golden_block(dev, dtype):
    from omniwave_b200 import OmniWeaveBlock

    z = load_golden("block_f64")
    blk = OmniWeaveBlock(8, 8, 128, 64, "shifted", 0, layer_scale_init=0.5)
    with torch.no_grad():
        for k in PARAMS:
            getattr(blk, k).copy_(torch.from_numpy(z[f"param_{k}"]))
    return z, blk.to(device=dev, dtype=dtype)


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-6), (torch.float32, 1e-4)])
def test_block_matches_reference(cuda_device, dtype, tol):
    z, blk = _golden_block(cuda_device, dtype)
    x = torch.tensor(z["in_x"], dtype=dtype, device=cuda_device, requires_grad=True)
    out = blk(x)
    assert out.dtype == dtype
    assert rel_err(out.detach().cpu().numpy(), z["out"]) <= tol
    grads = torch.autograd.grad(out, [x] + [getattr(blk, k) for k in PARAMS],
                                torch.tensor(z["dout"], dtype=dtype, device=cuda_device))
    assert rel_err(grads[0].cpu().numpy(), z["grad_x"]) <= tol
    for k, g in zip(PARAMS, grads[1:]):
        assert rel_err(g.cpu().numpy(), z[f"grad_{k}"]) <= tol, k


def test_block_autocast_bf16(cuda_device):
    """fp32 residual stream under bf16 autocast (the training configuration)."""
    z, blk = _golden_block(cuda_device, torch.float32)
    x = torch.tensor(z["in_x"], dtype=torch.float32, device=cuda_device, requires_grad=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = blk(x)
    assert out.dtype == torch.float32
    assert rel_err(out.detach().cpu().numpy(), z["out"]) <= 2e-2
    grads = torch.autograd.grad(out, [x] + [getattr(blk, k) for k in PARAMS],
                                torch.tensor(z["dout"], dtype=torch.float32, device=cuda_device))
    assert rel_err(grads[0].cpu().numpy(), z["grad_x"]) <= 2e-2
    for k, g in zip(PARAMS, grads[1:]):
        assert rel_err(g.cpu().numpy(), z[f"grad_{k}"]) <= 2e-2, k


def test_block_drop_path_scale(cuda_device):
    """Per-sample drop-path scale is applied to the delta only."""
    from omniwave_b200.ops import block_forward

    z, blk = _golden_block(cuda_device, torch.float64)
    x = torch.tensor(z["in_x"], dtype=torch.float64, device=cuda_device)
    scale = torch.tensor([0.0, 2.0], device=cuda_device)
    out = block_forward(x, blk.plan, blk.norm_weight, blk.a_u, blk.a_v, blk.a_o, blk.b_u,
                        blk.b_v, blk.b_o, blk.gamma, scale)
    ref = O.block_forward(z["in_x"], O.Plan(z["tok"], z["ch"], z["tmask"], z["cmask"], 8, 8, 128),
                          *[z[f"param_{k}"] for k in PARAMS], scale=np.array([0.0, 2.0]))
    assert rel_err(out.detach().cpu().numpy(), ref) <= 1e-6
    assert torch.equal(out[0], x[0])


def test_block_autocast_bf16_drop_path(cuda_device):
    """Tensor-core block forward (bf16 compute, f32 residual stream) with a
    per-sample drop-path scale: the epilogue's scale, gamma and residual add
    against the fp64 oracle; a zero scale returns x exactly."""
    from omniwave_b200.ops import block_forward

    z, blk = _golden_block(cuda_device, torch.float32)
    x = torch.tensor(z["in_x"], dtype=torch.float32, device=cuda_device)
    scale = torch.tensor([0.0, 1.5], device=cuda_device)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = block_forward(x, blk.plan, blk.norm_weight, blk.a_u, blk.a_v, blk.a_o, blk.b_u,
                            blk.b_v, blk.b_o, blk.gamma, scale)
    ref = O.block_forward(z["in_x"], O.Plan(z["tok"], z["ch"], z["tmask"], z["cmask"], 8, 8, 128),
                          *[z[f"param_{k}"] for k in PARAMS], scale=np.array([0.0, 1.5]))
    assert out.dtype == torch.float32
    assert rel_err(out.detach().cpu().numpy(), ref) <= 2e-2
    assert torch.equal(out[0], x[0])


@pytest.mark.parametrize("shape", [(14, 14, 256, 128), (10, 10, 128, 64)], ids=["14x14x256-d128", "10x10x128-d64"])
@pytest.mark.parametrize("route", [("shifted", 0), ("radix", 1)])
def test_block_bf16_scale_vs_oracle(cuda_device, route, shape):
    """bf16 residual stream (pad tokens, RMSNorm on the gathered tile --
    contiguous groups in the TMA-gather forward, strided ones in the pre-pass --
    scale and residual in the epilogue) against the oracle on the
    bf16-rounded operands."""
    from omniwave_b200 import build_route_plan
    from omniwave_b200.ops import block_forward

    (h, w, c, d), b = shape, 3
    rng = np.random.default_rng(11)
    qc = c // d

    def r16(a):
        return torch.tensor(a).to(torch.bfloat16)

    p = {"norm_weight": r16(1 + 0.1 * rng.standard_normal(c)),
         "a_u": r16(rng.standard_normal((16, 16)) / 4), "a_v": r16(rng.standard_normal((16, 16)) / 4),
         "a_o": r16(rng.standard_normal((16, 16)) / 4),
         "b_u": r16(rng.standard_normal((qc, d, 2 * d)) / np.sqrt(d)),
         "b_v": r16(rng.standard_normal((qc, d, 2 * d)) / np.sqrt(d)),
         "b_o": r16(rng.standard_normal((qc, 2 * d, d)) / np.sqrt(2 * d)),
         "gamma": r16(rng.standard_normal(c))}
    x = r16(rng.standard_normal((b, h, w, c)))
    scale = np.array([0.5, 2.0, 0.0])
    plan = build_route_plan(h, w, c, 16, d, route[0], route[1])
    dev = {k: v.to(cuda_device) for k, v in p.items()}
    out = block_forward(x.to(cuda_device), plan, dev["norm_weight"], dev["a_u"], dev["a_v"], dev["a_o"],
                        dev["b_u"], dev["b_v"], dev["b_o"], dev["gamma"],
                        torch.tensor(scale, dtype=torch.float32, device=cuda_device))
    assert out.dtype == torch.bfloat16
    op = O.Plan(plan.token_indices.numpy(), plan.channel_indices.numpy(), plan.token_mask.numpy(),
                plan.channel_mask.numpy(), h, w, c)
    ref = O.block_forward(x.double().numpy(), op, *[p[k].double().numpy() for k in PARAMS], scale=scale)
    got = out.double().cpu().numpy()
    x64 = x.double().numpy()
    assert rel_err(got[:2], ref[:2]) <= 2e-2
    # The delta alone (the residual dominates max|ref|).
    assert rel_err(got[:2] - x64[:2], ref[:2] - x64[:2]) <= 2e-2
    assert torch.equal(out[2].cpu(), x[2])

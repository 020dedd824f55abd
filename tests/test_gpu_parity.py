"""CUDA operator parity against the golden vectors and the numpy oracle.

Tolerances (max |cuda - ref| / max |ref|, per tensor):
  float64 compute: 1e-10;  float32 compute: 1e-4 (TF32 off);
  bf16 / f16 compute: 2e-2 -- the thresholds the BiGEMM north star states.
Every call goes through ``omniwave_b200.bigemm(backend="cuda")`` and so
through the C ABI of libomniwave_b200.so.
"""

from __future__ import annotations

import json
import os
import zlib

import numpy as np
import pytest
import torch

from conftest import load_golden, rel_err
from oracle import bigemm as O

pytestmark = pytest.mark.gpu

NAMES = ("x", "a_u", "a_v", "a_o", "b_u", "b_v", "b_o", "gamma")
TOL = {torch.float64: 1e-10, torch.float32: 1e-4, torch.bfloat16: 2e-2, torch.float16: 2e-2}


def _plan_from(z):
    from omniwave_b200.routing import RoutePlan

    h, w, c = (int(v) for v in z["hwc"])
    return RoutePlan(torch.from_numpy(z["tok"]), torch.from_numpy(z["ch"]),
                     torch.from_numpy(z["tmask"]), torch.from_numpy(z["cmask"]), h, w, c,
                     "golden", 0)


def run_cuda(plan, arrays: dict, dout: np.ndarray | None, dtype, dev, wdtype=None):
    """Forward (+ backward when ``dout`` is given) through the cuda backend."""
    from omniwave_b200 import bigemm

    wdtype = wdtype or dtype
    ts = {}
    for k in NAMES:
        dt = dtype if k == "x" else wdtype
        ts[k] = torch.tensor(arrays[k], dtype=dt, device=dev).requires_grad_(dout is not None)
    out = bigemm(plan=plan, backend="cuda", **ts)
    res = {"out": out.detach().double().cpu().numpy()}
    if dout is not None:
        go = torch.tensor(dout, dtype=out.dtype, device=dev)
        grads = torch.autograd.grad(out, [ts[k] for k in NAMES], go)
        for k, g in zip(NAMES, grads):
            res[k] = g.double().cpu().numpy()
    return res


@pytest.mark.parametrize("name", ["single_tile_f64", "gradcheck_f64", "radix1_pad_f64", "shifted_f64"])
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_golden_ops(cuda_device, name, dtype):
    z = load_golden(name)
    plan = _plan_from(z)
    arrays = {k: z[f"in_{k}"] for k in NAMES}
    res = run_cuda(plan, arrays, z["dout"], dtype, cuda_device)
    tol = TOL[dtype]
    assert rel_err(res["out"], z["out"]) <= tol
    for k in NAMES:
        assert rel_err(res[k], z[f"grad_{k}"]) <= tol, k


def test_golden_radix2_f32(cuda_device):
    z = load_golden("radix2_f32")
    plan = _plan_from(z)
    arrays = {k: z[f"in_{k}"] for k in NAMES}
    res = run_cuda(plan, arrays, z["dout"], torch.float32, cuda_device)
    assert rel_err(res["out"], z["out"]) <= 1e-4
    for k in NAMES:
        assert rel_err(res[k], z[f"grad_{k}"]) <= 1e-4, k


def test_config1_fp32(cuda_device):
    """X [8,14,14,512] seed 0, block init under seed 0, local route."""
    from omniwave_b200 import OmniWeaveBlock, bigemm

    z = load_golden("config1_f32")
    x = torch.randn(8, 14, 14, 512, generator=torch.Generator().manual_seed(0))
    torch.manual_seed(0)
    blk = OmniWeaveBlock(14, 14, 512, 128, "local", 0).to(cuda_device)
    with torch.no_grad():
        out = bigemm(x=x.to(cuda_device), plan=blk.plan, a_u=blk.a_u, a_v=blk.a_v, a_o=blk.a_o,
                     b_u=blk.b_u, b_v=blk.b_v, b_o=blk.b_o, gamma=blk.gamma, backend="cuda")
    assert rel_err(out.cpu().numpy(), z["out"]) <= 1e-4


def _rand_case(h, w, c, d, b, seed, gamma_scale=1.0):
    rng = np.random.default_rng(seed)
    qc = -(-c // d)
    rd = 2 * d
    return dict(
        x=rng.standard_normal((b, h, w, c)),
        a_u=rng.standard_normal((16, 16)) / 4, a_v=rng.standard_normal((16, 16)) / 4,
        a_o=rng.standard_normal((16, 16)) / 4,
        b_u=rng.standard_normal((qc, d, rd)) / np.sqrt(d),
        b_v=rng.standard_normal((qc, d, rd)) / np.sqrt(d),
        b_o=rng.standard_normal((qc, rd, d)) / np.sqrt(rd),
        gamma=rng.standard_normal(c) * gamma_scale,
    ), rng.standard_normal((b, h, w, c))


def _round(a, dtype):
    return torch.tensor(a).to(dtype).double().numpy()


STAGES = [(56, 56, 128, 64), (28, 28, 256, 64), (14, 14, 512, 128), (7, 7, 1024, 128)]
ROUTES = [("local", 0), ("shifted", 0), ("radix", 0), ("radix", 1), ("radix", 2)]


@pytest.mark.parametrize("shape", STAGES, ids=lambda s: f"{s[0]}x{s[1]}x{s[2]}")
@pytest.mark.parametrize("route", ROUTES, ids=lambda r: f"{r[0]}{r[1]}")
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_stage_shapes_vs_oracle(cuda_device, shape, route, dtype):
    """Every BASELINE stage shape and route (B=2) against the fp64 oracle."""
    from omniwave_b200 import build_route_plan

    h, w, c, d = shape
    arrays, dout = _rand_case(h, w, c, d, 2, seed=zlib.crc32(repr((shape, route)).encode()))
    # The oracle sees exactly the operands the kernel sees (rounded to dtype).
    arrays = {k: _round(v, dtype) for k, v in arrays.items()}
    dout_r = _round(dout, dtype)
    plan = build_route_plan(h, w, c, 16, d, route[0], route[1])
    p = O.Plan(plan.token_indices.numpy(), plan.channel_indices.numpy(),
               plan.token_mask.numpy(), plan.channel_mask.numpy(), h, w, c)
    wargs = [arrays[k] for k in NAMES[1:]]
    ref_out = O.forward(arrays["x"], p, *wargs)
    ref_g = O.backward(dout_r, arrays["x"], p, *wargs)
    res = run_cuda(plan, arrays, dout_r, dtype, cuda_device)
    tol = TOL[dtype]
    assert rel_err(res["out"], ref_out) <= tol
    for k in NAMES:
        assert rel_err(res[k], ref_g[k]) <= tol, k


def test_autocast_bf16_matches_oracle(cuda_device):
    """fp32 inputs and params under bf16 autocast: compute in bf16, fp32 delta."""
    from omniwave_b200 import bigemm, build_route_plan

    arrays, dout = _rand_case(14, 14, 512, 128, 2, seed=3)
    plan = build_route_plan(14, 14, 512, 16, 128, "shifted", 0)
    ts = {k: torch.tensor(v, dtype=torch.float32, device=cuda_device).requires_grad_(True)
          for k, v in arrays.items()}
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = bigemm(plan=plan, backend="cuda", **ts)
    assert out.dtype == torch.float32
    grads = torch.autograd.grad(out, list(ts.values()), torch.tensor(dout, dtype=torch.float32, device=cuda_device))
    p = O.Plan(plan.token_indices.numpy(), plan.channel_indices.numpy(),
               plan.token_mask.numpy(), plan.channel_mask.numpy(), 14, 14, 512)
    wargs = [arrays[k] for k in NAMES[1:]]
    assert rel_err(out.detach().cpu().numpy(), O.forward(arrays["x"], p, *wargs)) <= 2e-2
    ref_g = O.backward(dout, arrays["x"], p, *wargs)
    for k, g in zip(NAMES, grads):
        assert g.dtype == torch.float32
        assert rel_err(g.cpu().numpy(), ref_g[k]) <= 2e-2, k


def config2_case(h, w, c, d, route, level, batch=128):
    """BASELINE config 2's inputs: ``torch.manual_seed(1)``, an fp32
    ``OmniWeaveBlock`` with default init (orthogonal A_u/A_v, identity A_o,
    xavier B, gamma 1e-5), then ``x`` and ``dY`` ~ N(0,1), all cast to bf16
    (the order of scripts/benchmark.py:56-110)."""
    from omniwave_b200 import OmniWeaveBlock

    torch.manual_seed(1)
    blk = OmniWeaveBlock(h, w, c, d, route, level)
    x = torch.randn(batch, h, w, c)
    dy = torch.randn(batch, h, w, c)
    t = {"x": x}
    t.update({k: getattr(blk, k).detach() for k in NAMES[1:]})
    return blk.plan, {k: v.to(torch.bfloat16) for k, v in t.items()}, dy.to(torch.bfloat16)


FULL_SIZE_ERRORS: dict[str, dict[str, float]] = {}


@pytest.mark.parametrize("shape", STAGES, ids=lambda s: f"{s[0]}x{s[1]}x{s[2]}")
@pytest.mark.parametrize("route", ROUTES, ids=lambda r: f"{r[0]}{r[1]}")
def test_full_size_config2_bf16(cuda_device, shape, route, record_property):
    """Every benchmarked case at full size (B=128, bf16, fwd + bwd) on BASELINE
    config 2's inputs against the oracle on the bf16-rounded operands.  The
    oracle runs in float32 here (its own error, ~1e-6 of max|ref|, is far
    below the 2e-2 bf16 tolerance) to keep the host time and memory of the
    largest case to seconds and a few GB."""
    h, w, c, d = shape
    plan, t16, dy16 = config2_case(h, w, c, d, *route)
    arrays = {k: v.float().numpy() for k, v in t16.items()}
    dout = dy16.float().numpy()
    res = run_cuda(plan, arrays, dout, torch.bfloat16, cuda_device)
    p = O.Plan(plan.token_indices.numpy(), plan.channel_indices.numpy(),
               plan.token_mask.numpy(), plan.channel_mask.numpy(), h, w, c)
    wargs = [arrays[k] for k in NAMES[1:]]
    errs = {"out": rel_err(res["out"], O.forward(arrays["x"], p, *wargs))}
    ref_g = O.backward(dout, arrays["x"], p, *wargs)
    errs.update({f"d{k}": rel_err(res[k], ref_g[k]) for k in NAMES})
    case = f"{h}x{w}x{c}/{route[0]}{route[1]}"
    FULL_SIZE_ERRORS[case] = errs
    record_property("max_rel_err", errs)
    print(case, " ".join(f"{k}={v:.2e}" for k, v in errs.items()))
    report = os.environ.get("OW_PARITY_REPORT")
    if report:
        with open(report, "w") as f:
            json.dump(FULL_SIZE_ERRORS, f, indent=1)
    for k, v in errs.items():
        assert v <= 2e-2, (k, v)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_backward_is_deterministic(cuda_device, dtype):
    from omniwave_b200 import build_route_plan

    arrays, dout = _rand_case(28, 28, 256, 64, 8, seed=4)
    plan = build_route_plan(28, 28, 256, 16, 64, "radix", 1)
    r1 = run_cuda(plan, arrays, dout, dtype, cuda_device)
    r2 = run_cuda(plan, arrays, dout, dtype, cuda_device)
    for k in ("out",) + NAMES:
        assert np.array_equal(r1[k], r2[k]), k


def test_linear_in_gamma_full_size(cuda_device):
    """Size-independent property: delta is linear in gamma (x2 is exact)."""
    from omniwave_b200 import bigemm, build_route_plan

    torch.manual_seed(1)
    dev = cuda_device
    plan = build_route_plan(56, 56, 128, 16, 64, "shifted", 0)
    x = torch.randn(128, 56, 56, 128, device=dev, dtype=torch.bfloat16)
    w = dict(a_u=torch.randn(16, 16, device=dev) / 4, a_v=torch.randn(16, 16, device=dev) / 4,
             a_o=torch.randn(16, 16, device=dev) / 4, b_u=torch.randn(2, 64, 128, device=dev) / 8,
             b_v=torch.randn(2, 64, 128, device=dev) / 8, b_o=torch.randn(2, 128, 64, device=dev) / 11)
    w = {k: v.to(torch.bfloat16) for k, v in w.items()}
    gamma = torch.randn(128, device=dev, dtype=torch.float32)
    with torch.no_grad():
        a = bigemm(x=x, plan=plan, gamma=gamma, backend="cuda", **w)
        b = bigemm(x=x, plan=plan, gamma=2 * gamma, backend="cuda", **w)
    assert a.dtype == torch.float32
    assert torch.equal(2 * a, b)
    assert torch.isfinite(a).all()


def test_unsupported_raises(cuda_device):
    from omniwave_b200 import bigemm, build_route_plan

    plan = build_route_plan(8, 8, 32, 8, 32, "local")  # g = 8
    x = torch.randn(1, 8, 8, 32, device=cuda_device)
    w = dict(a_u=torch.eye(8, device=cuda_device), a_v=torch.eye(8, device=cuda_device),
             a_o=torch.eye(8, device=cuda_device), b_u=torch.zeros(1, 32, 64, device=cuda_device),
             b_v=torch.zeros(1, 32, 64, device=cuda_device), b_o=torch.zeros(1, 64, 32, device=cuda_device),
             gamma=torch.ones(32, device=cuda_device))
    with pytest.raises(RuntimeError, match="g=8"):
        bigemm(x=x, plan=plan, backend="cuda", **w)
    with pytest.raises(ValueError, match="unknown backend"):
        bigemm(x=x, plan=plan, backend="cuda_graphs", **w)

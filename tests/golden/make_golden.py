"""Generate golden vectors by running the reference ``omniweave`` package.

Usage::

    python tests/golden/make_golden.py --reference <checkout of QuackPhuc/omniwave>

Writes ``tests/golden/*.npz``.  Each case records the seeded inputs, the
reference's outputs and (where the case has them) the autograd gradients of
``sum(out * dout)``.  The fixtures are committed so that tests on a machine
without the reference checkout can still pin the oracle and the CUDA path.

Cases (reference file:line the setup follows):

* ``routes``            -- route tables of every BASELINE stage shape and
                           route plus padded shapes (routing.py:128-179).
* ``single_tile_f64``   -- tests/test_ops.py:45-72 setup (known answer).
* ``gradcheck_f64``     -- tests/test_ops.py:75-104 setup, with grads.
* ``radix1_pad_f64``    -- 7x7x70, d=64, radix level 1: token and channel pads.
* ``shifted_f64``       -- 8x8x128, d=64, shifted route.
* ``radix2_f32``        -- 14x14x512, d=128, radix level 2 (strided channels).
* ``config1_f32``       -- BASELINE config 1: X [8,14,14,512] from seed 0,
                           OmniWeaveBlock(14,14,512,128,"local",0) default
                           init under manual_seed(0); forward delta only.
* ``block_f64``         -- OmniWeaveBlock forward+backward (RMSNorm, residual).
* ``model_f32``         -- OmniWeave-T at 64x64 input, forward logits.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
NAMES = ("x", "a_u", "a_v", "a_o", "b_u", "b_v", "b_o", "gamma")


def _plan_arrays(plan):
    return dict(
        tok=plan.token_indices.numpy(), ch=plan.channel_indices.numpy(),
        tmask=plan.token_mask.numpy(), cmask=plan.channel_mask.numpy(),
        hwc=np.array([plan.height, plan.width, plan.channels]),
    )


def _param_digest(params):
    """Per-parameter fingerprint (shape, sums, leading values) instead of the
    full weights: the tests rebuild the weights from the same seed and check
    the fingerprint, which keeps the fixture small."""
    out = {}
    for k, v in params.items():
        a = v.detach().double().numpy()
        out[f"digest_{k}"] = np.concatenate([
            np.array(a.shape + (0,) * (4 - a.ndim), dtype=np.float64),
            [a.sum(), np.abs(a).sum(), (a * a).sum()], a.reshape(-1)[:8]])
    return out


def _op_case(ref, plan, tensors, with_grad=True, seed=0):
    vals = {k: v.detach().clone().requires_grad_(with_grad) for k, v in tensors.items()}
    out = ref.bigemm_delta_reference(plan=plan, **vals)
    rec = {f"in_{k}": v.detach().numpy() for k, v in vals.items()}
    rec["out"] = out.detach().numpy()
    if with_grad:
        g = torch.Generator().manual_seed(seed + 1000)
        dout = torch.randn(out.shape, generator=g, dtype=out.dtype)
        grads = torch.autograd.grad((out * dout).sum(), [vals[k] for k in NAMES])
        rec["dout"] = dout.numpy()
        for k, gr in zip(NAMES, grads):
            rec[f"grad_{k}"] = gr.numpy()
    rec.update(_plan_arrays(plan))
    return rec


def _rand_tensors(shape_hwc, b, g, d, rd, dtype, seed, gamma_scale=1.0):
    h, w, c = shape_hwc
    qc = -(-c // d)
    gen = torch.Generator().manual_seed(seed)

    def r(*s):
        return torch.randn(*s, generator=gen, dtype=dtype)

    return dict(
        x=r(b, h, w, c), a_u=r(g, g) / 4, a_v=r(g, g) / 4, a_o=r(g, g) / 4,
        b_u=r(qc, d, rd) / d ** 0.5, b_v=r(qc, d, rd) / d ** 0.5,
        b_o=r(qc, rd, d) / rd ** 0.5, gamma=r(c) * gamma_scale,
    )


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the omniweave checkout")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from omniweave.models import routing as R
    from omniweave.models.block import OmniWeaveBlock
    from omniweave.models.registry import create_model
    from omniweave.ops import reference as ref

    torch.backends.cuda.matmul.allow_tf32 = False

    # --- route tables -----------------------------------------------------
    routes = {}
    shapes = [(56, 56, 128, 64), (28, 28, 256, 64), (14, 14, 512, 128), (7, 7, 1024, 128),
              (7, 7, 70, 64), (8, 8, 128, 64), (4, 4, 32, 32), (5, 9, 48, 16)]
    kinds = [("local", 0), ("shifted", 0), ("radix", 0), ("radix", 1), ("radix", 2)]
    for h, w, c, d in shapes:
        for route, lvl in kinds:
            p = R.build_route_plan(h, w, c, 16, d, route, lvl)
            key = f"{h}x{w}x{c}_d{d}_{route}{lvl}"
            routes[f"{key}__tok"] = p.token_indices.numpy().astype(np.int32)
            routes[f"{key}__ch"] = p.channel_indices.numpy().astype(np.int32)
            routes[f"{key}__tmask"] = p.token_mask.numpy()
            routes[f"{key}__cmask"] = p.channel_mask.numpy()
    np.savez_compressed(os.path.join(HERE, "routes.npz"), **routes)

    # --- single tile, known answer (tests/test_ops.py:45-72) --------------
    torch.manual_seed(7)
    g, d, rd = 16, 4, 8
    x = torch.randn(1, 4, 4, 4, dtype=torch.float64)
    plan = R.build_route_plan(4, 4, 4, g, d, "local")
    t = dict(x=x, a_u=torch.randn(g, g, dtype=torch.float64),
             a_v=torch.randn(g, g, dtype=torch.float64),
             a_o=torch.randn(g, g, dtype=torch.float64),
             b_u=torch.randn(1, d, rd, dtype=torch.float64),
             b_v=torch.randn(1, d, rd, dtype=torch.float64),
             b_o=torch.randn(1, rd, d, dtype=torch.float64),
             gamma=torch.ones(d, dtype=torch.float64))
    np.savez_compressed(os.path.join(HERE, "single_tile_f64.npz"), **_op_case(ref, plan, t, seed=7))

    # --- gradcheck setup (tests/test_ops.py:75-104) ------------------------
    torch.manual_seed(42)
    x = torch.randn(1, 4, 4, 4, dtype=torch.float64)
    t = dict(x=x, a_u=torch.randn(g, g, dtype=torch.float64),
             a_v=torch.randn(g, g, dtype=torch.float64),
             a_o=torch.randn(g, g, dtype=torch.float64),
             b_u=torch.randn(1, d, rd, dtype=torch.float64),
             b_v=torch.randn(1, d, rd, dtype=torch.float64),
             b_o=torch.randn(1, rd, d, dtype=torch.float64),
             gamma=torch.randn(d, dtype=torch.float64))
    np.savez_compressed(os.path.join(HERE, "gradcheck_f64.npz"), **_op_case(ref, plan, t, seed=42))

    # --- padded radix-1, shifted, strided radix-2 -------------------------
    plan = R.build_route_plan(7, 7, 70, 16, 64, "radix", 1)
    t = _rand_tensors((7, 7, 70), 2, 16, 64, 128, torch.float64, seed=11)
    np.savez_compressed(os.path.join(HERE, "radix1_pad_f64.npz"), **_op_case(ref, plan, t, seed=11))

    plan = R.build_route_plan(8, 8, 128, 16, 64, "shifted", 0)
    t = _rand_tensors((8, 8, 128), 2, 16, 64, 128, torch.float64, seed=12)
    np.savez_compressed(os.path.join(HERE, "shifted_f64.npz"), **_op_case(ref, plan, t, seed=12))

    plan = R.build_route_plan(14, 14, 512, 16, 128, "radix", 2)
    t = _rand_tensors((14, 14, 512), 1, 16, 128, 256, torch.float32, seed=13)
    np.savez_compressed(os.path.join(HERE, "radix2_f32.npz"), **_op_case(ref, plan, t, seed=13))

    # --- BASELINE config 1 --------------------------------------------------
    x = torch.randn(8, 14, 14, 512, generator=torch.Generator().manual_seed(0))
    torch.manual_seed(0)
    blk = OmniWeaveBlock(14, 14, 512, 128, "local", 0)
    with torch.no_grad():
        delta = ref.bigemm_delta_reference(
            x=x, plan=blk.plan, a_u=blk.a_u, a_v=blk.a_v, a_o=blk.a_o,
            b_u=blk.b_u, b_v=blk.b_v, b_o=blk.b_o, gamma=blk.gamma)
    np.savez_compressed(
        os.path.join(HERE, "config1_f32.npz"), out=delta.numpy(),
        **_param_digest(dict(blk.named_parameters())))

    # --- block forward + backward (RMSNorm, residual) ----------------------
    torch.manual_seed(21)
    blk = OmniWeaveBlock(8, 8, 128, 64, "shifted", 0, layer_scale_init=0.5).double()
    with torch.no_grad():
        blk.norm_weight.uniform_(0.5, 1.5)
        blk.gamma.normal_()
    x = torch.randn(2, 8, 8, 128, dtype=torch.float64, requires_grad=True)
    out = blk(x)
    dout = torch.randn_like(out)
    params = dict(blk.named_parameters())
    grads = torch.autograd.grad((out * dout).sum(), [x] + list(params.values()))
    rec = dict(in_x=x.detach().numpy(), out=out.detach().numpy(), dout=dout.numpy(),
               grad_x=grads[0].numpy())
    for (k, v), gr in zip(params.items(), grads[1:]):
        rec[f"param_{k}"] = v.detach().numpy()
        rec[f"grad_{k}"] = gr.numpy()
    rec.update(_plan_arrays(blk.plan))
    np.savez_compressed(os.path.join(HERE, "block_f64.npz"), **rec)

    # --- OmniWeave-T forward at 64x64 --------------------------------------
    torch.manual_seed(5)
    model = create_model("omniweave_t", input_size=64, layer_scale_init=0.5).eval()
    inp = torch.randn(2, 3, 64, 64, generator=torch.Generator().manual_seed(6))
    with torch.no_grad():
        logits = model(inp)
    np.savez_compressed(
        os.path.join(HERE, "model_f32.npz"), inp=inp.numpy(), logits=logits.numpy(),
        **_param_digest(model.state_dict()))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()

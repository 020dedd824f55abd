"""The numpy oracle against golden vectors produced by the reference itself.

These pin the oracle before it is trusted as the GPU checker: forward, all
eight operator gradients, and the RMSNorm block's forward and gradients.
Also carries the reference's closed-form single-tile check
(tests/test_ops.py:45-72) and pack/unpack round trips (:12-42).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import load_golden, rel_err
from oracle import bigemm as O

NAMES = ("x", "a_u", "a_v", "a_o", "b_u", "b_v", "b_o", "gamma")


def _plan(z):
    h, w, c = (int(v) for v in z["hwc"])
    return O.Plan(z["tok"], z["ch"], z["tmask"], z["cmask"], h, w, c)


@pytest.mark.parametrize("name,tol", [("single_tile_f64", 1e-12), ("gradcheck_f64", 1e-12),
                                      ("radix1_pad_f64", 1e-12), ("shifted_f64", 1e-12),
                                      ("radix2_f32", 5e-6)])
def test_oracle_matches_reference(name, tol):
    z = load_golden(name)
    p = _plan(z)
    ws = [z[f"in_{k}"] for k in NAMES[1:]]
    assert rel_err(O.forward(z["in_x"], p, *ws), z["out"]) <= tol
    g = O.backward(z["dout"], z["in_x"], p, *ws)
    for k in NAMES:
        assert rel_err(g[k], z[f"grad_{k}"]) <= tol, k


def test_oracle_block_matches_reference():
    z = load_golden("block_f64")
    p = _plan(z)
    names = ("norm_weight", "a_u", "a_v", "a_o", "b_u", "b_v", "b_o", "gamma")
    ws = [z[f"param_{k}"] for k in names]
    # float32 variance in the reference bounds agreement at ~1e-7.
    assert rel_err(O.block_forward(z["in_x"], p, *ws), z["out"]) <= 1e-8
    g = O.block_backward(z["dout"], z["in_x"], p, *ws)
    assert rel_err(g["x"], z["grad_x"]) <= 1e-8
    for k in names:
        assert rel_err(g[k], z[f"grad_{k}"]) <= 1e-6, k


def test_single_tile_closed_form():
    z = load_golden("single_tile_f64")
    x = z["in_x"]
    tile = x.reshape(16, 4)
    silu = lambda u: u / (1 + np.exp(-u))  # noqa: E731
    exp = (z["in_a_o"] @ (silu(z["in_a_u"] @ tile @ z["in_b_u"][0]) * (z["in_a_v"] @ tile @ z["in_b_v"][0]))
           @ z["in_b_o"][0]).reshape(x.shape)
    assert rel_err(O.forward(x, _plan(z), *[z[f"in_{k}"] for k in NAMES[1:]]), exp) <= 1e-12


@pytest.mark.parametrize("shape,route,lvl", [((7, 7, 70, 64), "radix", 1), ((8, 8, 128, 64), "local", 0),
                                             ((8, 8, 128, 64), "shifted", 0), ((14, 14, 512, 128), "radix", 2)])
def test_pack_unpack_round_trip(shape, route, lvl):
    h, w, c, d = shape
    p = O.make_plan(h, w, c, 16, d, route, lvl)
    x = np.arange(2 * h * w * c, dtype=np.float64).reshape(2, h, w, c)
    t = O.pack(x, p)
    assert t.shape == (2, p.tok.shape[0], p.ch.shape[0], 16, d)
    assert np.array_equal(O.unpack(t, p), x)
    mask = p.tmask[:, None, :, None] & p.cmask[None, :, None, :]
    assert np.count_nonzero(t[:, ~mask]) == 0


def test_oracle_gradient_finite_difference():
    """Independent of the golden files: central differences on a small case."""
    rng = np.random.default_rng(0)
    p = O.make_plan(4, 4, 8, 16, 4, "local")
    x = rng.standard_normal((1, 4, 4, 8))
    ws = [rng.standard_normal((16, 16)) / 4 for _ in range(3)] + \
         [rng.standard_normal((2, 4, 8)) / 2 for _ in range(2)] + \
         [rng.standard_normal((2, 8, 4)) / 2, rng.standard_normal(8)]
    dy = rng.standard_normal(x.shape)
    g = O.backward(dy, x, p, *ws)
    f = lambda xx: float((O.forward(xx, p, *ws) * dy).sum())  # noqa: E731
    eps = 1e-6
    for idx in [(0, 0, 0, 0), (0, 1, 2, 3), (0, 3, 3, 7)]:
        xp = x.copy(); xp[idx] += eps
        xm = x.copy(); xm[idx] -= eps
        assert abs((f(xp) - f(xm)) / (2 * eps) - g["x"][idx]) < 1e-6

"""Model glue on CPU: module tree, parameter names/shapes/count, seeded init
identical to the reference, and the reference's shape/schedule checks
(tests/test_model.py).  Forward passes need the GPU and live in
test_gpu_block_model.py."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from omniwave_b200 import OmniWeaveBackbone, OmniWeaveBlock, create_model, space_to_depth_nhwc


def _digest(t):
    a = t.detach().double().numpy()
    return np.concatenate([np.array(a.shape + (0,) * (4 - a.ndim), dtype=np.float64),
                           [a.sum(), np.abs(a).sum(), (a * a).sum()], a.reshape(-1)[:8]])


def test_param_count_matches_reference():
    m = create_model("omniweave_t")
    assert sum(p.numel() for p in m.parameters()) == 10_232_040


def test_seeded_model_init_is_identical_to_reference():
    z = load_golden("model_f32")
    torch.manual_seed(5)
    sd = create_model("omniweave_t", input_size=64, layer_scale_init=0.5).state_dict()
    keys = {k[len("digest_"):] for k in z if k.startswith("digest_")}
    assert keys == set(sd)
    for k in keys:
        assert np.array_equal(_digest(sd[k]), z[f"digest_{k}"]), k


def test_seeded_block_init_is_identical_to_reference():
    z = load_golden("config1_f32")
    torch.manual_seed(0)
    blk = OmniWeaveBlock(14, 14, 512, 128, "local", 0)
    for k, v in blk.named_parameters():
        assert np.array_equal(_digest(v), z[f"digest_{k}"]), k


def test_block_parameter_shapes():
    blk = OmniWeaveBlock(14, 14, 512, 128, "radix", 2)
    shapes = {k: tuple(v.shape) for k, v in blk.named_parameters()}
    assert shapes == {"norm_weight": (512,), "a_u": (16, 16), "a_v": (16, 16), "a_o": (16, 16),
                      "b_u": (4, 128, 256), "b_v": (4, 128, 256), "b_o": (4, 256, 128),
                      "gamma": (512,)}
    assert torch.allclose(blk.a_o, torch.eye(16))
    assert torch.allclose(blk.a_u @ blk.a_u.T, torch.eye(16), atol=1e-5)


def test_stage_schedules_and_anchors():
    m = create_model("omniweave_t")
    routes = [[(b.plan.route, b.plan.radix_level) for b in s.blocks] for s in m.stages]
    assert routes[2] == [("local", 0), ("shifted", 0), ("radix", 0), ("radix", 1), ("radix", 2),
                         ("local", 0), ("shifted", 0), ("radix", 0)]
    assert [s.anchor is not None for s in m.stages] == [False, False, True, True]
    assert [s.blocks[0].plan.height for s in m.stages] == [56, 28, 14, 7]


def test_space_to_depth():
    x = torch.arange(2 * 4 * 4 * 3, dtype=torch.float32).reshape(2, 4, 4, 3)
    y = space_to_depth_nhwc(x, 2)
    assert y.shape == (2, 2, 2, 12)
    assert torch.equal(y[0, 0, 0], torch.cat([x[0, 0, 0], x[0, 0, 1], x[0, 1, 0], x[0, 1, 1]]))
    with pytest.raises(ValueError):
        space_to_depth_nhwc(torch.zeros(1, 5, 4, 3), 2)


def test_registry_errors_and_drop_path_validation():
    with pytest.raises(ValueError, match="unknown model"):
        create_model("omniweave_xl")
    with pytest.raises(NotImplementedError):
        create_model("omniweave_t", pretrained=True)
    with pytest.raises(ValueError):
        OmniWeaveBlock(8, 8, 128, 64, "local", 0, drop_path_rate=1.0)
    with pytest.raises(ValueError):
        OmniWeaveBackbone(widths=[1, 2, 3])


def test_drop_path_schedule():
    m = create_model("omniweave_t", drop_path_rate=0.1)
    rates = [b.drop_path_rate for s in m.stages for b in s.blocks]
    assert rates[0] == 0.0 and abs(rates[-1] - 0.1) < 1e-12
    assert all(b >= a for a, b in zip(rates, rates[1:]))


def test_cpu_forward_raises_instead_of_falling_back():
    blk = OmniWeaveBlock(8, 8, 128, 64, "local", 0)
    with pytest.raises(RuntimeError):
        blk(torch.randn(1, 8, 8, 128))

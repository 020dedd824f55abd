"""The standalone ``omniwave_b200.OmniWeaveBlock`` on CPU: parameter names,
shapes and seeded init identical to the reference block (block.py:54-78),
and no host fallback.  Forward passes need the GPU (test_gpu_block_model.py)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from omniwave_b200 import OmniWeaveBlock


def _digest(t):
    a = t.detach().double().numpy()
    return np.concatenate([np.array(a.shape + (0,) * (4 - a.ndim), dtype=np.float64),
                           [a.sum(), np.abs(a).sum(), (a * a).sum()], a.reshape(-1)[:8]])


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


def test_drop_path_validation():
    with pytest.raises(ValueError):
        OmniWeaveBlock(8, 8, 128, 64, "local", 0, drop_path_rate=1.0)


def test_cpu_forward_raises_instead_of_falling_back():
    blk = OmniWeaveBlock(8, 8, 128, 64, "local", 0)
    with pytest.raises(RuntimeError):
        blk(torch.randn(1, 8, 8, 128))

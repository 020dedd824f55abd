"""Route plans: the reference's own routing tests plus bit-exact tables.

The first group mirrors the reference's tests/test_routing.py:10-74 on this
package's builder.  The golden group compares every BASELINE stage shape and
route (plus padded shapes) with tables the reference itself produced, for
both the vectorised builder and the loop-level oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from omniwave_b200.routing import build_route_plan, build_stage_schedule, radix_order
from oracle.routing import build_plan


def test_local_route_covers_tokens_once():
    plan = build_route_plan(8, 8, 128, 16, 64, "local")
    valid = plan.token_indices[plan.token_mask]
    assert torch.equal(torch.sort(valid).values, torch.arange(64))
    assert plan.token_indices.shape == (4, 16)
    assert plan.channel_indices.shape == (2, 64)


def test_shifted_route_is_a_permutation():
    local = build_route_plan(8, 8, 128, 16, 64, "local")
    shifted = build_route_plan(8, 8, 128, 16, 64, "shifted")
    assert not torch.equal(local.token_indices, shifted.token_indices)
    assert torch.equal(torch.sort(shifted.token_indices[shifted.token_mask]).values, torch.arange(64))


def test_stage_schedule():
    assert build_stage_schedule(8) == [
        ("local", 0), ("shifted", 0), ("radix", 0), ("radix", 1), ("radix", 2),
        ("local", 0), ("shifted", 0), ("radix", 0),
    ]
    assert build_stage_schedule(1) == [("local", 0)]


def test_padding_masks_non_divisible_shapes():
    plan = build_route_plan(7, 7, 70, 16, 64, "radix", radix_level=1)
    assert plan.token_mask.sum().item() == 49
    assert plan.channel_mask.sum().item() == 70
    assert plan.token_indices.max().item() == 49
    assert plan.channel_indices.max().item() == 70


def test_radix_route_covers_tokens():
    plan = build_route_plan(8, 8, 128, 16, 64, "radix", radix_level=0)
    assert torch.equal(torch.sort(plan.token_indices[plan.token_mask]).values, torch.arange(64))


def test_local_route_small_spatial():
    plan = build_route_plan(4, 4, 32, 16, 32, "local")
    assert torch.equal(torch.sort(plan.token_indices[plan.token_mask]).values, torch.arange(16))
    assert plan.token_indices.shape == (1, 16)


def test_unknown_route_rejected():
    with pytest.raises(ValueError, match="unknown route"):
        build_route_plan(8, 8, 128, 16, 64, "spiral")


def test_plans_are_cached_and_int64():
    a = build_route_plan(14, 14, 512, 16, 128, "shifted", 0)
    assert a is build_route_plan(14, 14, 512, 16, 128, "shifted", 0)
    assert a.token_indices.dtype == torch.int64 and a.channel_mask.dtype == torch.bool


def _golden_keys():
    z = load_golden("routes")
    return sorted({k.split("__")[0] for k in z})


@pytest.mark.parametrize("key", _golden_keys())
def test_tables_bit_exact_vs_reference(key):
    z = load_golden("routes")
    hwc, dpart, rl = key.split("_")
    h, w, c = (int(v) for v in hwc.split("x"))
    d = int(dpart[1:])
    route, lvl = rl[:-1], int(rl[-1])
    plan = build_route_plan(h, w, c, 16, d, route, lvl)
    tok, ch, tm, cm = build_plan(h, w, c, 16, d, route, lvl)
    for ours, orc, name in ((plan.token_indices, tok, "tok"), (plan.channel_indices, ch, "ch"),
                            (plan.token_mask, tm, "tmask"), (plan.channel_mask, cm, "cmask")):
        ref = z[f"{key}__{name}"]
        assert np.array_equal(ours.numpy(), ref), name
        assert np.array_equal(orc, ref), f"oracle {name}"


def test_radix_order_list_api():
    assert radix_order(20, 16, 0) == list(range(20))
    assert radix_order(40, 4, 1)[:8] == [0, 4, 8, 12, 1, 5, 9, 13]


def test_large_plan_is_a_permutation():
    plan = build_route_plan(256, 256, 128, 16, 64, "shifted")
    v = plan.token_indices[plan.token_mask]
    assert v.numel() == 65536 and torch.unique(v).numel() == 65536

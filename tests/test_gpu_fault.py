"""Bounded waits on the GPU: a wait that runs out is reported, and the
context stays usable.

Every mbarrier wait in the pipelined kernels gives up after a time limit,
sets the CTA's abort flag and the library's one per-device fault word.
``ow_debug_wait_probe`` makes each such kernel first wait on a barrier that
nothing arrives on, before it issues any copy or MMA, so the wait runs out
with nothing in flight -- no GPU fault is caused.  The test checks that the
forward kernel and the backward role kernel (two translation units) both
report through the same word, that reading it with reset clears it, and that
a normal call afterwards matches the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import bigemm as O

pytestmark = pytest.mark.gpu

NAMES = ("x", "a_u", "a_v", "a_o", "b_u", "b_v", "b_o", "gamma")


def _case(dev):
    from omniwave_b200 import build_route_plan

    rng = np.random.default_rng(21)
    h, w, c, d = 14, 14, 512, 128
    arr = dict(x=rng.standard_normal((2, h, w, c)), a_u=rng.standard_normal((16, 16)) / 4,
               a_v=rng.standard_normal((16, 16)) / 4, a_o=rng.standard_normal((16, 16)) / 4,
               b_u=rng.standard_normal((4, d, 2 * d)) / np.sqrt(d),
               b_v=rng.standard_normal((4, d, 2 * d)) / np.sqrt(d),
               b_o=rng.standard_normal((4, 2 * d, d)) / np.sqrt(2 * d), gamma=rng.standard_normal(c))
    arr = {k: torch.tensor(v).to(torch.bfloat16) for k, v in arr.items()}
    dy = torch.tensor(rng.standard_normal((2, h, w, c))).to(torch.bfloat16)
    plan = build_route_plan(h, w, c, 16, d, "radix", 1)
    ts = {k: v.to(dev).requires_grad_(True) for k, v in arr.items()}
    return plan, arr, ts, dy.to(dev)


def test_wait_timeout_is_reported_and_the_context_survives(cuda_device):
    from omniwave_b200 import _lib, bigemm

    lib = _lib.load()
    dev = cuda_device
    assert _lib.device_fault(0, reset=True) == 0
    plan, arr, ts, dy = _case(dev)
    try:
        # Forward kernel (ow_tc.cu).
        assert lib.ow_debug_wait_probe(1_000_000) == 0
        bigemm(plan=plan, backend="cuda", **ts)
        torch.cuda.synchronize(dev)
        assert _lib.device_fault(0) == 1
        assert _lib.device_fault(0, reset=True) == 1
        assert _lib.device_fault(0) == 0
        # Backward role kernel (ow_tc_bwd.cu) reports through the same word.
        assert lib.ow_debug_wait_probe(0) == 0
        out = bigemm(plan=plan, backend="cuda", **ts)
        assert lib.ow_debug_wait_probe(1_000_000) == 0
        torch.autograd.grad(out, [ts[k] for k in NAMES], dy)
        torch.cuda.synchronize(dev)
        with pytest.raises(_lib.DeviceFaultError):
            _lib.check_device_fault(0)
        assert _lib.device_fault(0) == 0
    finally:
        lib.ow_debug_wait_probe(0)
    # The limit of the self-check is enforced.
    assert lib.ow_debug_wait_probe(2_000_000_000) == _lib.OW_OK + 1
    # The context is intact: a normal call matches the oracle, with no fault.
    out = bigemm(plan=plan, backend="cuda", **ts)
    grads = torch.autograd.grad(out, [ts[k] for k in NAMES], dy)
    p = O.Plan(plan.token_indices.numpy(), plan.channel_indices.numpy(), plan.token_mask.numpy(),
               plan.channel_mask.numpy(), 14, 14, 512)
    a = {k: v.double().numpy() for k, v in arr.items()}
    ws = [a[k] for k in NAMES[1:]]
    assert rel_err(out.detach().double().cpu().numpy(), O.forward(a["x"], p, *ws)) <= 2e-2
    ref = O.backward(dy.double().cpu().numpy(), a["x"], p, *ws)
    for k, g in zip(NAMES, grads):
        assert rel_err(g.double().cpu().numpy(), ref[k]) <= 2e-2, k
    assert _lib.device_fault(0) == 0

"""Backend dispatch policy (mirrors the reference's tests/test_dispatch.py:13-66
with ``"cuda"`` in the role of ``"triton"``) and the operator's argument checks."""

from __future__ import annotations

import logging

import pytest
import torch

from omniwave_b200 import bigemm, build_route_plan, cuda_is_supported, select_backend


def test_auto_falls_back_on_cpu(caplog):
    with caplog.at_level(logging.INFO):
        backend, reason = select_backend(torch.randn(1), "auto", lambda _: (False, "CUDA is unavailable"))
    assert backend == "reference"
    assert reason == "CUDA is unavailable"
    assert "CUDA is unavailable" in caplog.text


def test_forced_cuda_fails():
    with pytest.raises(RuntimeError, match="CUDA is unavailable"):
        select_backend(torch.randn(1), "cuda", lambda _: (False, "CUDA is unavailable"))


@pytest.mark.parametrize("name", ["reference", "compile", "triton"])
def test_passthrough(name):
    assert select_backend(torch.randn(1), name, lambda _: (True, None)) == (name, None)


def test_auto_selects_cuda_when_supported():
    assert select_backend(torch.randn(1), "auto", lambda _: (True, None)) == ("cuda", None)


def test_unknown_backend_rejected():
    with pytest.raises(ValueError, match="unknown backend"):
        select_backend(torch.randn(1), "cuda_graphs", lambda _: (True, None))


def _ops_args(c=128, d=64):
    qc = c // d
    return dict(a_u=torch.eye(16), a_v=torch.eye(16), a_o=torch.eye(16),
                b_u=torch.zeros(qc, d, 2 * d), b_v=torch.zeros(qc, d, 2 * d),
                b_o=torch.zeros(qc, 2 * d, d), gamma=torch.ones(c))


def test_cpu_tensor_is_unsupported_and_never_computed_on_host():
    plan = build_route_plan(8, 8, 128, 16, 64, "local")
    x = torch.randn(1, 8, 8, 128)
    ok, reason = cuda_is_supported(x, plan, torch.zeros(2, 64, 128))
    assert not ok and reason == "CUDA is unavailable"
    with pytest.raises(RuntimeError, match="CUDA is unavailable"):
        bigemm(x=x, plan=plan, backend="cuda", **_ops_args())


def test_reference_backends_go_to_the_reference_package(omniweave):
    """``"reference"`` (the default, as in bigemm.py:35) and an unsupported
    ``"auto"`` run the reference package's own code, never this package's."""
    from omniweave.ops.reference import bigemm_delta_reference

    plan = build_route_plan(8, 8, 128, 16, 64, "local")
    x = torch.randn(1, 8, 8, 128)
    ref = bigemm_delta_reference(x=x, plan=plan, **_ops_args())
    assert torch.equal(bigemm(x=x, plan=plan, **_ops_args()), ref)
    assert torch.equal(bigemm(x=x, plan=plan, backend="reference", **_ops_args()), ref)
    assert torch.equal(bigemm(x=x, plan=plan, backend="auto", **_ops_args()), ref)


def test_reference_backends_without_the_reference_package(monkeypatch):
    import sys

    monkeypatch.setitem(sys.modules, "omniweave", None)
    monkeypatch.setitem(sys.modules, "omniweave.ops", None)
    plan = build_route_plan(8, 8, 128, 16, 64, "local")
    with pytest.raises(RuntimeError, match="belong to the omniweave package"):
        bigemm(x=torch.randn(1, 8, 8, 128), plan=plan, backend="reference", **_ops_args())


def test_unknown_backend_in_bigemm():
    plan = build_route_plan(8, 8, 128, 16, 64, "local")
    with pytest.raises(ValueError, match="unknown backend"):
        bigemm(x=torch.randn(1, 8, 8, 128), plan=plan, backend="tpu", **_ops_args())


def test_plan_validation_rejects_duplicates():
    from omniwave_b200.ops import _validate_plan
    from omniwave_b200.routing import RoutePlan

    good = build_route_plan(8, 8, 128, 16, 64, "local")
    _validate_plan(good)
    tok = good.token_indices.clone()
    tok[0, 1] = tok[0, 0]
    bad = RoutePlan(tok, good.channel_indices, good.token_mask, good.channel_mask, 8, 8, 128, "x", 0)
    with pytest.raises(ValueError, match="exactly once"):
        _validate_plan(bad)

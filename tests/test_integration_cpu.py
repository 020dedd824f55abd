"""The cuda backend installed into the reference package (CPU side).

``omniwave_b200.integration.install()`` patches the reference ``omniweave``
package in place (dispatch.py:13-49, bigemm.py:24-73, block.py:80-108).
These tests check, without a GPU, that the patched reference keeps its own
behaviour for its own backends, accepts ``"cuda"`` with the reference's
forced-backend rule, never computes a cuda call on the host, and that models
built for either backend share one state-dict format (names, shapes, seeded
values) so checkpoints interchange.
"""

from __future__ import annotations

import io
import logging

import numpy as np
import pytest
import torch

from conftest import load_golden


def _digest(t):
    a = t.detach().double().numpy()
    return np.concatenate([np.array(a.shape + (0,) * (4 - a.ndim), dtype=np.float64),
                           [a.sum(), np.abs(a).sum(), (a * a).sum()], a.reshape(-1)[:8]])


def test_install_is_idempotent(omniweave):
    from omniwave_b200 import integration

    assert integration.installed()
    assert integration.install() is omniweave
    import omniweave.ops.bigemm as ob
    import omniweave.models.block as mb

    assert ob.bigemm is mb.bigemm


def test_select_backend_accepts_cuda_with_the_forced_backend_rule(omniweave):
    from omniweave.ops.dispatch import select_backend

    assert select_backend(torch.randn(1), "cuda", lambda _: (True, None)) == ("cuda", None)
    with pytest.raises(RuntimeError, match="CUDA is unavailable"):
        select_backend(torch.randn(1), "cuda", lambda _: (False, "CUDA is unavailable"))
    # The reference's own rules are unchanged (its tests/test_dispatch.py).
    assert select_backend(torch.randn(1), "reference", lambda _: (True, None)) == ("reference", None)
    assert select_backend(torch.randn(1), "compile", lambda _: (False, "x")) == ("compile", None)
    assert select_backend(torch.randn(1), "triton", lambda _: (True, None)) == ("triton", None)
    with pytest.raises(RuntimeError, match="nope"):
        select_backend(torch.randn(1), "triton", lambda _: (False, "nope"))
    with pytest.raises(ValueError, match="unknown backend"):
        select_backend(torch.randn(1), "tpu", lambda _: (True, None))


def test_auto_on_cpu_falls_back_to_reference(omniweave, caplog):
    from omniweave.models.block import OmniWeaveBlock
    from omniweave.ops.bigemm import bigemm

    torch.manual_seed(0)
    blk = OmniWeaveBlock(8, 8, 128, 64, "shifted", 0, layer_scale_init=0.5)
    x = torch.randn(2, 8, 8, 128)
    kw = dict(x=x, plan=blk.plan, a_u=blk.a_u, a_v=blk.a_v, a_o=blk.a_o, b_u=blk.b_u,
              b_v=blk.b_v, b_o=blk.b_o, gamma=blk.gamma)
    ref = bigemm(backend="reference", **kw)
    with caplog.at_level(logging.INFO):
        auto = bigemm(backend="auto", **kw)
    assert torch.equal(auto, ref)
    with pytest.raises(RuntimeError, match="CUDA is unavailable"):
        bigemm(backend="cuda", **kw)
    with pytest.raises(ValueError, match="unknown backend"):
        bigemm(backend="tpu", **kw)


def test_block_with_cuda_backend_never_runs_on_the_host(omniweave):
    from omniweave.models.block import OmniWeaveBlock

    blk = OmniWeaveBlock(8, 8, 128, 64, "local", 0, backend="cuda")
    with pytest.raises(RuntimeError, match="CUDA is unavailable"):
        blk(torch.randn(1, 8, 8, 128))
    torch.manual_seed(1)
    a = OmniWeaveBlock(8, 8, 128, 64, "radix", 1, backend="auto", layer_scale_init=0.5)
    torch.manual_seed(1)
    r = OmniWeaveBlock(8, 8, 128, 64, "radix", 1, backend="reference", layer_scale_init=0.5)
    x = torch.randn(2, 8, 8, 128)
    assert torch.equal(a(x), r(x))


def test_standalone_bigemm_mirror_delegates_reference_backends(omniweave):
    from omniweave.ops.reference import bigemm_delta_reference

    from omniwave_b200 import OmniWeaveBlock, bigemm

    torch.manual_seed(2)
    blk = OmniWeaveBlock(8, 8, 128, 64, "local", 0, layer_scale_init=0.5)
    x = torch.randn(1, 8, 8, 128)
    kw = dict(x=x, plan=blk.plan, a_u=blk.a_u, a_v=blk.a_v, a_o=blk.a_o, b_u=blk.b_u,
              b_v=blk.b_v, b_o=blk.b_o, gamma=blk.gamma)
    ref = bigemm_delta_reference(**kw)
    assert torch.equal(bigemm(**kw), ref)  # default backend is "reference", as in the reference
    assert torch.equal(bigemm(backend="auto", **kw), ref)


def test_models_for_both_backends_share_one_state_dict_format(omniweave):
    from omniweave.models.registry import create_model

    torch.manual_seed(5)
    ref = create_model("omniweave_t", input_size=64, layer_scale_init=0.5)
    torch.manual_seed(5)
    cud = create_model("omniweave_t", input_size=64, layer_scale_init=0.5, backend="cuda")
    sr, sc = ref.state_dict(), cud.state_dict()
    assert list(sr) == list(sc)
    for k in sr:
        assert torch.equal(sr[k], sc[k]), k
    # The seeded values are the ones the reference drew when the golden file was made.
    z = load_golden("model_f32")
    assert {k[len("digest_"):] for k in z if k.startswith("digest_")} == set(sr)
    for k in sr:
        assert np.array_equal(_digest(sc[k]), z[f"digest_{k}"]), k
    assert sum(p.numel() for p in create_model("omniweave_t", backend="cuda").parameters()) == 10_232_040


def test_checkpoint_round_trip_between_backends(omniweave):
    """A state dict saved from either backend's model loads strictly into the other."""
    from omniweave.models.registry import create_model

    torch.manual_seed(6)
    src = create_model("omniweave_t", input_size=64, backend="cuda")
    with torch.no_grad():
        for p in src.parameters():
            p.add_(torch.randn_like(p) * 0.01)
    buf = io.BytesIO()
    torch.save(src.state_dict(), buf)
    buf.seek(0)
    dst = create_model("omniweave_t", input_size=64, backend="reference")
    dst.load_state_dict(torch.load(buf), strict=True)
    back = create_model("omniweave_t", input_size=64, backend="cuda")
    back.load_state_dict(dst.state_dict(), strict=True)
    for (k, a), (_, b) in zip(src.state_dict().items(), back.state_dict().items()):
        assert torch.equal(a, b), k


def test_standalone_block_state_dict_interchanges_with_reference(omniweave):
    from omniweave.models.block import OmniWeaveBlock as RefBlock

    from omniwave_b200 import OmniWeaveBlock

    torch.manual_seed(0)
    ours = OmniWeaveBlock(14, 14, 512, 128, "local", 0)
    torch.manual_seed(0)
    ref = RefBlock(14, 14, 512, 128, "local", 0)
    for (k, a), (k2, b) in zip(ours.state_dict().items(), ref.state_dict().items()):
        assert k == k2 and torch.equal(a, b), k
    ref.load_state_dict(ours.state_dict(), strict=True)
    ours.load_state_dict(ref.state_dict(), strict=True)
    assert torch.equal(ours.plan.token_indices, ref.plan.token_indices)
    assert torch.equal(ours.plan.channel_indices, ref.plan.channel_indices)

"""Data-parallel host logic on CPU with the gloo backend (world size 2).

The model here is a small MLP stand-in -- as in the reference's own training
tests (tests/test_training.py:29-36) -- because the BiGEMM blocks need a GPU;
what is tested is the host-side plumbing: rank-0 broadcast of the init, DDP's
gradient all-reduce matching single-process training on the global batch,
batch sharding, the device-side fail-fast flag, and a rank that raises.
"""

from __future__ import annotations

import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _mlp(seed: int) -> nn.Module:
    torch.manual_seed(seed)
    return nn.Sequential(nn.Linear(12, 16), nn.GELU(), nn.Linear(16, 5))


def _worker(rank: int, world: int, port: int, mode: str, q) -> None:
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    from omniwave_b200.train import TrainStep, init_distributed, shard_range

    try:
        info = init_distributed(backend="gloo", timeout_s=20)
        g = torch.Generator().manual_seed(123)
        x = torch.randn(8, 12, generator=g)
        y = torch.randint(0, 5, (8,), generator=g)
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 failed before its first step")
        model = _mlp(seed=rank)  # different init per rank; broadcast must fix it
        ts = TrainStep(model, amp_dtype=None)
        a, b = shard_range(8, info.rank, info.world_size)
        for _ in range(3):
            ts.step(x[a:b], y[a:b])
        ts.check_finite()
        q.put((rank, [p.detach().numpy().copy() for p in model.parameters()]))
    except Exception as exc:  # reported to the parent, never hangs it
        q.put((rank, repr(exc)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(mode: str):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        rank, val = q.get(timeout=120)
        out[rank] = val
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_ddp_matches_single_process_on_global_batch():
    out = _run("ok")
    assert isinstance(out[0], list) and isinstance(out[1], list), out
    for p0, p1 in zip(out[0], out[1]):
        assert (p0 == p1).all()  # replicas stay identical
    # Single process, same init (rank 0's), whole batch.
    sys.path.insert(0, ROOT)
    from omniwave_b200.train import TrainStep

    g = torch.Generator().manual_seed(123)
    x = torch.randn(8, 12, generator=g)
    y = torch.randint(0, 5, (8,), generator=g)
    model = _mlp(seed=0)
    ts = TrainStep(model, amp_dtype=None)
    for _ in range(3):
        ts.step(x, y)
    for p, q in zip(model.parameters(), out[0]):
        torch.testing.assert_close(p.detach(), torch.from_numpy(q), rtol=1e-5, atol=1e-6)


def test_failing_rank_is_reported_not_hung():
    out = _run("fail")
    assert "rank 1 failed" in str(out[1])
    # Rank 0 leaves with an error (its collective times out or sees the peer
    # gone) instead of waiting forever.
    assert isinstance(out[0], str)


def test_shard_range_covers_batch():
    from omniwave_b200.train import shard_range

    for n in (0, 1, 7, 128, 257):
        for w in (1, 2, 3, 8):
            parts = [shard_range(n, r, w) for r in range(w)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
            assert max(b - a for a, b in parts) - min(b - a for a, b in parts) <= 1


def test_nonfinite_loss_skips_the_update_and_fails_fast():
    """A non-finite loss leaves weights (and the EMA) untouched without a host
    sync; check_finite then raises, as the reference raises at engine.py:205."""
    from omniwave_b200.train import TrainStep

    model = _mlp(0)
    ts = TrainStep(model, amp_dtype=None, ema_decay=0.9)
    before = [p.detach().clone() for p in model.parameters()]
    ema_before = {k: v.clone() for k, v in ts.ema.state.items()}
    x = torch.full((4, 12), float("nan"))
    ts.step(x, torch.zeros(4, dtype=torch.long))
    for p, b in zip(model.parameters(), before):
        assert torch.equal(p.detach(), b)
    for k, v in ts.ema.state.items():
        assert torch.equal(v, ema_before[k]), k
    with pytest.raises(FloatingPointError):
        ts.check_finite()
    # A later finite step updates normally.
    g = torch.Generator().manual_seed(1)
    ts.step(torch.randn(4, 12, generator=g), torch.zeros(4, dtype=torch.long))
    assert any(not torch.equal(p.detach(), b) for p, b in zip(model.parameters(), before))


def test_step_with_clip_and_ema_matches_reference_engine_semantics():
    """clip_grad_norm_ then AdamW then EMAModel.update, as engine.py:243-257."""
    from omniwave_b200.train import TrainStep

    g = torch.Generator().manual_seed(7)
    x = torch.randn(6, 12, generator=g) * 10
    y = torch.randint(0, 5, (6,), generator=g)
    model = _mlp(3)
    ts = TrainStep(model, amp_dtype=None, clip_norm=0.5, ema_decay=0.8)
    ref = _mlp(3)
    opt = torch.optim.AdamW(ref.parameters(), lr=1e-3, weight_decay=0.05)
    ema = {k: v.detach().clone() for k, v in ref.state_dict().items()}
    for _ in range(3):
        ts.step(x, y)
        loss = nn.functional.cross_entropy(ref(x), y)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        nn.utils.clip_grad_norm_(ref.parameters(), 0.5)
        opt.step()
        with torch.no_grad():
            for k, p in ref.named_parameters():
                ema[k].lerp_(p, 1 - 0.8)
    for p, q in zip(model.parameters(), ref.parameters()):
        torch.testing.assert_close(p.detach(), q.detach(), rtol=1e-6, atol=1e-7)
    for k, v in ts.ema.state_dict().items():
        torch.testing.assert_close(v, ema[k], rtol=1e-6, atol=1e-7)

"""Data-parallel training and batch-sharded inference around the B200 blocks.

Covers the parts of the reference training engine that sit on the BiGEMM
path (``omniweave/training/engine.py``, ``training/distributed.py``), not its
data pipeline, checkpointing or logging:

* ``init_distributed`` -- one process per GPU from ``RANK`` / ``WORLD_SIZE``
  / ``LOCAL_RANK`` (reference ``distributed.py:24-51``), with a bounded
  process-group timeout so ranks that lose a peer fail instead of hanging.
* ``broadcast_parameters`` -- rank 0's random init to every rank.
* ``TrainStep`` -- one optimisation step as in ``train_one_epoch``
  (``engine.py:134-300``): bf16 autocast forward, cross-entropy, backward
  with DDP's bucketed NCCL all-reduce overlapped, AdamW step, optional
  gradient clipping and EMA.  The reference's per-step host syncs
  (``_is_finite(loss)`` at :205 and a per-parameter finite check at
  :229-232) become one device-side flag that makes the optimizer and the
  EMA skip their update; it is read on the host only when the caller asks
  (``check_finite``), so steps queue without host round trips.  On one GPU
  the whole step can run as one CUDA graph.
* ``EMA`` -- the reference's ``EMAModel`` (engine.py:106-131), sync-free.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F
from torch import Tensor

__all__ = ["DistInfo", "EMA", "init_distributed", "broadcast_parameters", "shard_range", "TrainStep"]


@dataclass(frozen=True)
class DistInfo:
    rank: int
    world_size: int
    local_rank: int
    device: torch.device


def init_distributed(backend: str | None = None, timeout_s: float = 120.0) -> DistInfo:
    """Join the process group described by the launcher's environment.

    ``backend`` defaults to ``"nccl"`` when CUDA is available, else
    ``"gloo"``.  A single process (no ``WORLD_SIZE`` or ``WORLD_SIZE=1``)
    does not create a group.
    """
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    use_cuda = torch.cuda.is_available() and backend != "gloo"
    device = torch.device("cuda", local) if use_cuda else torch.device("cpu")
    if use_cuda:
        torch.cuda.set_device(device)
    if world > 1 and not dist.is_initialized():
        backend = backend or ("nccl" if use_cuda else "gloo")
        kwargs = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kwargs["device_id"] = device
        dist.init_process_group(**kwargs)
    return DistInfo(rank, world, local, device)


@torch.no_grad()
def broadcast_parameters(module: nn.Module, src: int = 0) -> None:
    """Copy ``src``'s parameters and buffers to every rank."""
    if not (dist.is_available() and dist.is_initialized()):
        return
    for t in list(module.parameters()) + list(module.buffers()):
        dist.broadcast(t.data, src=src)


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous ``[start, stop)`` share of ``n`` items for ``rank``."""
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class EMA:
    """Exponential moving average of a model's state (reference ``EMAModel``,
    engine.py:106-131): parameters move by ``lerp(param, 1 - decay)``, buffers
    are copied.  ``update`` takes an optional device flag; when it is nonzero
    the update is skipped without a host sync (a step that was skipped for a
    non-finite loss leaves the average untouched, as the reference's
    fail-fast would)."""

    def __init__(self, model: nn.Module, decay: float = 0.9999) -> None:
        self.decay = decay
        self.state = {k: v.detach().clone() for k, v in model.state_dict().items()}
        self._pnames = [k for k, _ in model.named_parameters() if k in self.state]
        self._bnames = [k for k, _ in model.named_buffers() if k in self.state]

    @torch.no_grad()
    def update(self, model: nn.Module, skip: Tensor | None = None) -> None:
        src = model.module if hasattr(model, "module") else model
        params = dict(src.named_parameters())
        dst = [self.state[k] for k in self._pnames]
        cur = [params[k].detach().to(self.state[k].dtype) for k in self._pnames]
        if dst:
            if skip is None:
                torch._foreach_lerp_(dst, cur, 1.0 - self.decay)
            else:
                w = (1.0 - skip.to(torch.float32)) * (1.0 - self.decay)
                torch._foreach_lerp_(dst, cur, [w.to(t.dtype) for t in dst])
        bufs = dict(src.named_buffers())
        for k in self._bnames:
            self.state[k].copy_(bufs[k])

    def state_dict(self) -> dict[str, Tensor]:
        return {k: v.clone() for k, v in self.state.items()}


class TrainStep:
    """One data-parallel optimisation step of a classifier.

    Parameters mirror the reference defaults used by BASELINE config 5:
    AdamW(lr=1e-3, weight_decay=0.05), bf16 autocast, cross-entropy.  The
    reference engine's other step features are options with its semantics:
    ``clip_norm`` (``clip_grad_norm_``, engine.py:243-244) and ``ema_decay``
    (``EMAModel``, engine.py:256-257).

    Non-finite values never reach the weights, and no host sync is needed
    to guarantee it: one device flag collects ``~isfinite`` of the loss and
    of every gradient (the reference's checks at engine.py:205 and
    :229-240), the fused AdamW kernel skips its update when the flag is set
    (its ``found_inf`` input), and so does the EMA.  ``check_finite()``
    raises ``FloatingPointError`` afterwards, as the reference raises at
    the step itself.

    ``cuda_graph=True`` (single process only) captures the whole step --
    forward, backward, finite check, optimizer and EMA -- into one CUDA
    graph after ``graph_warmup`` eager steps; later steps copy the batch
    into the graph's input buffers and replay it.
    """

    def __init__(
        self,
        model: nn.Module,
        *,
        lr: float = 1e-3,
        weight_decay: float = 0.05,
        amp_dtype: torch.dtype | None = torch.bfloat16,
        bucket_cap_mb: float = 25.0,
        broadcast: bool = True,
        clip_norm: float | None = None,
        ema_decay: float | None = None,
        cuda_graph: bool = False,
        graph_warmup: int = 3,
    ) -> None:
        self.device = next(model.parameters()).device
        distributed = dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1
        if distributed and broadcast:
            broadcast_parameters(model)
        if cuda_graph and (distributed or self.device.type != "cuda"):
            raise ValueError("cuda_graph=True needs a single process on a CUDA device")
        self.module = model
        if distributed:
            self.model: nn.Module = nn.parallel.DistributedDataParallel(
                model,
                device_ids=[self.device.index] if self.device.type == "cuda" else None,
                bucket_cap_mb=bucket_cap_mb,
                gradient_as_bucket_view=True,
                broadcast_buffers=False,
            )
        else:
            self.model = model
        on_cuda = self.device.type == "cuda"
        self.optimizer = torch.optim.AdamW(
            model.parameters(), lr=lr, weight_decay=weight_decay, fused=on_cuda,
            capturable=cuda_graph)
        self.amp_dtype = amp_dtype if on_cuda else None
        self.clip_norm = clip_norm
        self.ema = EMA(model, ema_decay) if ema_decay is not None else None
        self._params = [p for p in model.parameters() if p.requires_grad]
        # 1.0 when this step saw a non-finite loss or gradient (fused AdamW's
        # found_inf input), and a sticky flag over all steps for check_finite.
        self._found = torch.zeros((), dtype=torch.float32, device=self.device)
        self._bad = torch.zeros((), dtype=torch.bool, device=self.device)
        self._one = torch.ones((), dtype=torch.float32, device=self.device)
        self._graph = None
        self._graph_warmup = graph_warmup if cuda_graph else -1
        self._nsteps = 0
        self._static: tuple[Tensor, Tensor, Tensor] | None = None

    def _body(self, images: Tensor, labels: Tensor) -> Tensor:
        self.model.train()
        if self.amp_dtype is not None:
            with torch.autocast(self.device.type, dtype=self.amp_dtype, cache_enabled=False):
                loss = F.cross_entropy(self.model(images), labels)
        else:
            loss = F.cross_entropy(self.model(images), labels)
        self.optimizer.zero_grad(set_to_none=True)
        loss.backward()
        loss = loss.detach()
        self._found.copy_((~torch.isfinite(loss)).to(torch.float32))
        grads = [p.grad for p in self._params if p.grad is not None]
        if self.device.type == "cuda":
            # One multi-tensor pass: sets _found when any gradient is inf/nan.
            torch._amp_foreach_non_finite_check_and_unscale_(grads, self._found, self._one)
        else:
            for g in grads:
                self._found.logical_or_(~torch.isfinite(g).all())
        if self.clip_norm is not None:
            nn.utils.clip_grad_norm_(self._params, self.clip_norm, foreach=True)
        if self.device.type == "cuda":
            self.optimizer.found_inf = self._found  # the fused kernel skips the update when set
            self.optimizer.step()
        else:
            snapshot = [p.detach().clone() for p in self._params]
            self.optimizer.step()
            with torch.no_grad():
                keep = self._found.bool()
                for p, old in zip(self._params, snapshot):
                    p.copy_(torch.where(keep, old, p))
        if self.ema is not None:
            self.ema.update(self.module, skip=self._found)
        self._bad |= self._found.bool()
        return loss

    def step(self, images: Tensor, labels: Tensor) -> Tensor:
        """Forward, backward (gradients all-reduced by DDP), optimizer step.

        Returns the loss as a device tensor; nothing here waits for the GPU.
        """
        self._nsteps += 1
        if self._graph_warmup < 0:
            return self._body(images, labels)
        if self._graph is None and self._nsteps <= self._graph_warmup:
            # Warm-up runs eagerly on a side stream, as graph capture requires.
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                loss = self._body(images, labels)
            torch.cuda.current_stream(self.device).wait_stream(side)
            return loss
        if self._graph is None:
            si, sl = images.clone(), labels.clone()
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                sloss = self._body(si, sl)
            self._graph, self._static = g, (si, sl, sloss)
        si, sl, sloss = self._static
        si.copy_(images, non_blocking=True)
        sl.copy_(labels, non_blocking=True)
        self._graph.replay()
        return sloss

    def check_finite(self) -> None:
        """Raise ``FloatingPointError`` if any step so far saw a non-finite loss
        or gradient (the reference's fail-fast, engine.py:205-240); those steps
        left the weights and the EMA unchanged.  Syncs the device."""
        if bool(self._bad.item()):
            raise FloatingPointError("non-finite loss or gradient in a training step (update skipped)")

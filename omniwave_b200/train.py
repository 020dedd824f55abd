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
  with DDP's bucketed NCCL all-reduce overlapped, AdamW step.  The
  reference's per-step host syncs (``_is_finite(loss)`` at :205 and a
  per-parameter finite check at :229-232) become one device-side flag that
  is read only when the caller asks (``check_finite``), so steps queue
  without host round trips; the fail-fast behaviour (``FloatingPointError``)
  is kept.
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

__all__ = ["DistInfo", "init_distributed", "broadcast_parameters", "shard_range", "TrainStep"]


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


class TrainStep:
    """One data-parallel optimisation step of a classifier.

    Parameters mirror the reference defaults used by BASELINE config 5:
    AdamW(lr=1e-3, weight_decay=0.05), bf16 autocast, cross-entropy.
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
    ) -> None:
        self.device = next(model.parameters()).device
        distributed = dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1
        if distributed and broadcast:
            broadcast_parameters(model)
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
        fused = self.device.type == "cuda"
        self.optimizer = torch.optim.AdamW(
            model.parameters(), lr=lr, weight_decay=weight_decay, fused=fused)
        self.amp_dtype = amp_dtype if self.device.type == "cuda" else None
        self._bad = torch.zeros((), dtype=torch.bool, device=self.device)

    def step(self, images: Tensor, labels: Tensor) -> Tensor:
        """Forward, backward (gradients all-reduced by DDP), optimizer step.

        Returns the loss as a device tensor; nothing here waits for the GPU.
        """
        self.model.train()
        if self.amp_dtype is not None:
            with torch.autocast(self.device.type, dtype=self.amp_dtype):
                loss = F.cross_entropy(self.model(images), labels)
        else:
            loss = F.cross_entropy(self.model(images), labels)
        self.optimizer.zero_grad(set_to_none=True)
        loss.backward()
        self._bad |= ~torch.isfinite(loss.detach())
        self.optimizer.step()
        return loss.detach()

    def check_finite(self) -> None:
        """Raise ``FloatingPointError`` if any step so far had a non-finite loss
        (the reference's fail-fast, ``engine.py:205-210``); syncs the device."""
        if bool(self._bad.item()):
            raise FloatingPointError("non-finite loss in a training step")

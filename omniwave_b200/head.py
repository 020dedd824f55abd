"""Global average pool + classifier head of the OmniWeave backbone on the B200 kernel.

The reference classifies with ``pooled = stage4.mean(dim=(1, 2))`` followed by
``self.head(pooled)``, an ``nn.Linear(C4, num_classes)`` with bias
(omniweave/models/backbone.py:190-197).  ``ow_pool_head_fwd`` does both in one
kernel: a cluster of eight CTAs pools a group of images from HBM straight into
the tensor-core operand of the head GEMM (shared memory), so the pooled matrix
is written out only when the weight gradient needs it.

The fused path takes 16-bit compute (autocast bf16/f16, or a 16-bit model), as
the rest of the cuda backbone does: the f32 mean is rounded to the compute type
and the weight and bias are cast to it, which is what autocast does to the
reference's ``nn.Linear``.  The backward is the autograd of those reference
ops, on PyTorch GEMMs: ``dpooled = g W``, ``dW = g^T pooled``, ``db = sum g``
and the mean's gradient ``dpooled / (H W)`` broadcast over the tokens.
"""

from __future__ import annotations

from typing import Any

import torch
from torch import Tensor

from omniwave_b200 import _lib
from omniwave_b200.s2d import _compute

__all__ = ["pool_head", "pool_head_backward", "pool_head_supported", "head_supported"]

_C16 = (torch.bfloat16, torch.float16)


def _kernel_x_dtype(x_dtype: torch.dtype, compute: torch.dtype) -> torch.dtype:
    """x as is when the kernel takes it (f32 or the compute type), else cast to compute."""
    return x_dtype if x_dtype in (torch.float32, compute) else compute


def _kernel_w_dtype(w_dtype: torch.dtype, compute: torch.dtype) -> torch.dtype:
    return w_dtype if w_dtype in (torch.float32, compute) else torch.float32


def _args(x: Tensor | None, shape: tuple[int, int, int], x_dtype: torch.dtype, weight: Tensor | None,
          w_dtype: torch.dtype, classes: int, bias: Tensor | None, b_dtype: torch.dtype | None,
          compute: torch.dtype, out: Tensor | None, pooled: Tensor | None) -> _lib.PoolHead:
    b, t, c = shape
    return _lib.PoolHead(
        _lib.ptr(x), _lib.DTYPE_CODE.get(x_dtype, -1), b, t, c,
        _lib.ptr(weight), _lib.DTYPE_CODE.get(w_dtype, -1),
        _lib.ptr(bias), _lib.DTYPE_CODE.get(b_dtype, -1) if b_dtype is not None else -1,
        classes, _lib.DTYPE_CODE.get(compute, -1),
        _lib.ptr(out), _lib.ptr(pooled), None, 0,
    )


def pool_head_supported(x: Tensor, weight: Tensor, bias: Tensor | None = None,
                        compute: torch.dtype | None = None) -> tuple[bool, str | None]:
    """``(is_supported, reason_if_not)`` for ``pool_head`` on these arguments."""
    if x.device.type != "cuda":
        return False, "CUDA is unavailable"
    compute = compute or _compute(x, weight)
    if compute not in _C16:
        return False, f"compute dtype {compute} is not 16-bit"
    if x.dim() != 4 or weight.dim() != 2:
        return False, "x must be [B, H, W, C] and the weight 2-D"
    if weight.shape[1] != x.shape[3]:
        return False, f"weight must be [N, {x.shape[3]}], got {tuple(weight.shape)}"
    if bias is not None and tuple(bias.shape) != (weight.shape[0],):
        return False, f"bias must be [{weight.shape[0]}], got {tuple(bias.shape)}"
    try:
        lib = _lib.load()
    except _lib.NativeLibraryError as exc:
        return False, str(exc)
    idx = x.device.index if x.device.index is not None else torch.cuda.current_device()
    if not lib.ow_device_supported(idx):
        return False, f"device {idx} is not sm_100 (B200-class)"
    b, h, w, c = x.shape
    args = _args(None, (b, h * w, c), _kernel_x_dtype(x.dtype, compute), None,
                 _kernel_w_dtype(weight.dtype, compute), weight.shape[0], None,
                 None if bias is None else bias.dtype, compute, None, None)
    if lib.ow_pool_head_workspace_size(args) == 0:
        return False, "shape or dtype not supported by ow_pool_head_fwd"
    return True, None


def _fwd(x: Tensor, weight: Tensor, bias: Tensor | None, compute: torch.dtype,
         want_pooled: bool) -> tuple[Tensor, Tensor | None]:
    lib = _lib.load()
    b, h, w, c = x.shape
    x = x.to(_kernel_x_dtype(x.dtype, compute)).contiguous()
    weight = weight.to(_kernel_w_dtype(weight.dtype, compute)).contiguous()
    if bias is not None and bias.dtype not in (torch.float32, *_C16):
        bias = bias.float()
    bias = None if bias is None else bias.contiguous()
    n = weight.shape[0]
    out = torch.empty((b, n), dtype=compute, device=x.device)
    pooled = torch.empty((b, c), dtype=compute, device=x.device) if want_pooled else None
    args = _args(x, (b, h * w, c), x.dtype, weight, weight.dtype, n, bias,
                 None if bias is None else bias.dtype, compute, out, pooled)
    stream = _lib.stream_handle(x.device)
    nbytes = lib.ow_pool_head_workspace_size(args)
    if nbytes == 0:  # unsupported: the call reports why
        _lib.check(lib.ow_pool_head_fwd(args, stream), "ow_pool_head_fwd")
    ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    args.workspace, args.workspace_bytes = ws.data_ptr(), nbytes
    with torch.cuda.device(x.device):  # the library launches on the current device
        _lib.check(lib.ow_pool_head_fwd(args, stream), "ow_pool_head_fwd")
    del ws
    return out, pooled


class _PoolHead(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, compute):
        out, pooled = _fwd(x.detach(), weight.detach(), None if bias is None else bias.detach(), compute,
                           want_pooled=ctx.needs_input_grad[1])
        ctx.save_for_backward(pooled, weight.detach())
        ctx.compute, ctx.x_dtype, ctx.x_shape = compute, x.dtype, tuple(x.shape)
        ctx.b_dtype = None if bias is None else bias.dtype
        return out

    @staticmethod
    def backward(ctx, g):
        pooled, weight = ctx.saved_tensors
        return (*pool_head_backward(g, pooled, weight, ctx.x_shape, ctx.x_dtype, ctx.b_dtype, ctx.compute,
                                    ctx.needs_input_grad[:3]), None)


def pool_head_backward(g: Tensor, pooled: Tensor | None, weight: Tensor, x_shape: tuple[int, ...],
                       x_dtype: torch.dtype, b_dtype: torch.dtype | None, compute: torch.dtype,
                       needs: tuple[bool, ...] = (True, True, True)):
    """Gradients ``(dx, dW, db)`` of ``linear(x.mean(dim=(1, 2)), W, b)`` taken in ``compute``.

    The autograd of the reference's ops under autocast: the linear's input
    gradient ``g W`` in the compute type, cast back to the mean's dtype
    (x's), then the mean's gradient ``grad / (H W)`` on every token (returned
    as a broadcast view); ``dW = g^T pooled`` and ``db = sum_b g`` in the
    compute type, cast to the parameters' dtypes.  ``pooled`` is the forward's
    rounded mean (needed for ``dW`` only).
    """
    g = g.to(compute)
    dx = dw = db = None
    with torch.autocast(g.device.type, enabled=False):
        if needs[0]:
            b, h, w, c = x_shape
            dp = (g @ weight.to(compute)).to(x_dtype) / (h * w)
            dx = dp.view(b, 1, 1, c).expand(b, h, w, c)
        if needs[1]:
            dw = (g.t() @ pooled).to(weight.dtype)
        if needs[2] and b_dtype is not None:
            db = g.sum(0).to(b_dtype)
    return dx, dw, db


def pool_head(x: Tensor, weight: Tensor, bias: Tensor | None = None) -> Tensor:
    """``linear(x.mean(dim=(1, 2)), weight, bias)`` for NHWC ``x`` [B, H, W, C].

    Returns ``[B, N]`` logits in the compute dtype: the autocast dtype when
    autocast is on, else x's dtype when it is 16-bit.  Raises
    ``RuntimeError`` when the kernel does not support the arguments (float32
    compute included).
    """
    compute = _compute(x, weight)
    ok, why = pool_head_supported(x, weight, bias, compute)
    if not ok:
        raise RuntimeError(f"pool_head not supported: {why}")
    return _PoolHead.apply(x, weight, bias, compute)


def head_supported(model: Any, stage4: Tensor) -> tuple[bool, str | None]:
    """Whether ``model.head`` (an ``nn.Linear``) can run fused with the pool on ``stage4``."""
    head = getattr(model, "head", None)
    if not isinstance(head, torch.nn.Linear):
        return False, "the head is not an nn.Linear"
    return pool_head_supported(stage4, head.weight, head.bias)

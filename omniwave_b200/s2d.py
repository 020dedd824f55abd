"""Stem and downsamples of the OmniWeave-T backbone on the B200 kernels.

The reference backbone rearranges space into channels and projects
(omniweave/models/backbone.py:14-27 ``space_to_depth_nhwc``, the stem
``Linear(48, C1)`` at :121, the downsamples ``Linear(4 C_i, C_{i+1})`` at
:128-132, called at :173-187).  Here each ``Linear(space_to_depth(x))`` is one
tensor-core GEMM (``ow_s2d_linear_fwd``) that reads the rearranged rows
straight from ``x``: the stem from the NCHW image batch (the reference's
``permute(0, 2, 3, 1)`` at :173 is folded in too), the downsamples from the
NHWC stage output.

A stage anchor ``Linear(C, C)`` (backbone.py:50, :76-77) directly follows the
space-to-depth projection that feeds its stage, so it is folded into that
GEMM: ``y = s2d(x) (W_a W_d)^T``, the product of the two 16-bit weights
formed once per call.  The backward recovers both weight
gradients from the gradient of the folded weight
``dW = dy^T s2d(x)``: ``dW_a = dW W_d^T``, ``dW_d = W_a^T dW`` (PyTorch
GEMMs), and the input gradient from ``dy (W_a W_d)`` with the space-to-depth
inverted: for the downsamples one kernel (``ow_d2s_linear_fwd``) whose
epilogue stores each output chunk at its place in the NHWC image, so neither
the GEMM's output nor a rearranging copy goes through memory.

The fused path takes 16-bit compute (autocast bf16/f16, or a 16-bit model),
which is how the reference trains; float32 compute stays on the reference
modules.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Any

import torch
from torch import Tensor

from omniwave_b200 import _lib

__all__ = [
    "space_to_depth_nhwc",
    "depth_to_space_nhwc",
    "s2d_linear",
    "s2d_linear_backward",
    "d2s_linear",
    "s2d_linear_supported",
    "forward_features",
    "features_supported",
]

_C16 = (torch.bfloat16, torch.float16)


def space_to_depth_nhwc(x: Tensor, factor: int) -> Tensor:
    """``[B, H, W, C] -> [B, H/f, W/f, f f C]`` with channel index ``(dy f + dx) C + c``.

    Same rearrangement (and error) as backbone.py:14-27.
    """
    b, h, w, c = x.shape
    if h % factor or w % factor:
        raise ValueError(f"height {h} and width {w} must be divisible by factor {factor}")
    y = x.reshape(b, h // factor, factor, w // factor, factor, c).permute(0, 1, 3, 2, 4, 5)
    return y.reshape(b, h // factor, w // factor, factor * factor * c)


def depth_to_space_nhwc(y: Tensor, factor: int) -> Tensor:
    """Inverse of ``space_to_depth_nhwc``: ``[B, Ho, Wo, f f C] -> [B, Ho f, Wo f, C]``."""
    b, ho, wo, k = y.shape
    c = k // (factor * factor)
    t = y.reshape(b, ho, wo, factor, factor, c).permute(0, 1, 3, 2, 4, 5)
    return t.reshape(b, ho * factor, wo * factor, c)


def _compute(x: Tensor, weight: Tensor) -> torch.dtype:
    """The autocast dtype when autocast is on, else a 16-bit x's dtype, else the promotion."""
    if x.is_cuda and torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    if x.dtype in _C16:
        return x.dtype
    return torch.promote_types(x.dtype, weight.dtype)


def _args(x: Tensor | None, shape: tuple[int, int, int, int], x_dtype: torch.dtype, layout: int,
          factor: int, weight: Tensor, out: Tensor | None, compute: torch.dtype) -> _lib.S2dLinear:
    if layout == _lib.LAYOUT_NCHW:
        b, c, h, w = shape
    else:
        b, h, w, c = shape
    return _lib.S2dLinear(
        _lib.ptr(x), _lib.DTYPE_CODE.get(x_dtype, -1), layout, b, h, w, c, factor,
        _lib.ptr(weight), _lib.DTYPE_CODE.get(weight.dtype, -1), weight.shape[0],
        _lib.ptr(out), _lib.DTYPE_CODE.get(compute, -1), None, 0,
    )


def _kernel_dtypes(x_dtype: torch.dtype, w_dtype: torch.dtype, nchw: bool,
                   compute: torch.dtype) -> tuple[torch.dtype, torch.dtype]:
    """The dtypes the kernel is handed: x as is when it takes it, else the compute dtype."""
    xk = x_dtype if (x_dtype == compute or (nchw and x_dtype == torch.float32)) else compute
    wk = w_dtype if w_dtype in (torch.float32, compute) else torch.float32
    return xk, wk


def _shape_supported(device: torch.device, shape: tuple[int, ...], x_dtype: torch.dtype,
                     weight: Tensor, factor: int, nchw: bool,
                     compute: torch.dtype) -> tuple[bool, str | None]:
    if device.type != "cuda":
        return False, "CUDA is unavailable"
    if compute not in _C16:
        return False, f"compute dtype {compute} is not 16-bit"
    if len(shape) != 4 or weight.dim() != 2:
        return False, "x must be 4-D and the weight 2-D"
    try:
        lib = _lib.load()
    except _lib.NativeLibraryError as exc:
        return False, str(exc)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if not lib.ow_device_supported(idx):
        return False, f"device {idx} is not sm_100 (B200-class)"
    k = factor * factor * (shape[1] if nchw else shape[3])
    if weight.shape[1] != k:
        return False, f"weight must be [N, {k}], got {tuple(weight.shape)}"
    xk, wk = _kernel_dtypes(x_dtype, weight.dtype, nchw, compute)
    args = _args(None, tuple(shape), xk, _lib.LAYOUT_NCHW if nchw else _lib.LAYOUT_NHWC, factor,
                 weight, None, compute)
    args.weight, args.w_dtype = None, _lib.DTYPE_CODE[wk]  # a size query reads no pointer
    if lib.ow_s2d_linear_workspace_size(args) == 0:
        return False, "shape or dtype not supported by ow_s2d_linear_fwd"
    return True, None


def s2d_linear_supported(x: Tensor, weight: Tensor, factor: int, nchw: bool = False,
                         compute: torch.dtype | None = None) -> tuple[bool, str | None]:
    """``(is_supported, reason_if_not)`` for ``s2d_linear`` on these arguments."""
    compute = compute or _compute(x, weight)
    return _shape_supported(x.device, tuple(x.shape), x.dtype, weight, factor, nchw, compute)


def _fwd(x: Tensor, weight: Tensor, factor: int, nchw: bool,
         compute: torch.dtype) -> tuple[Tensor, Tensor]:
    """Runs the kernel; returns the output and x as the kernel read it."""
    lib = _lib.load()
    xk, wk = _kernel_dtypes(x.dtype, weight.dtype, nchw, compute)
    x = x.to(xk).contiguous()
    weight = weight.to(wk).contiguous()
    if nchw:
        b, c, h, w = x.shape
    else:
        b, h, w, c = x.shape
    out = torch.empty((b, h // factor, w // factor, weight.shape[0]), dtype=compute, device=x.device)
    layout = _lib.LAYOUT_NCHW if nchw else _lib.LAYOUT_NHWC
    args = _args(x, tuple(x.shape), x.dtype, layout, factor, weight, out, compute)
    stream = _lib.stream_handle(x.device)
    n = lib.ow_s2d_linear_workspace_size(args)
    if n == 0:  # unsupported: the call reports why
        _lib.check(lib.ow_s2d_linear_fwd(args, stream), "ow_s2d_linear_fwd")
    ws = torch.empty(n, dtype=torch.uint8, device=x.device)
    args.workspace, args.workspace_bytes = ws.data_ptr(), n
    with torch.cuda.device(x.device):  # the library launches on the current device
        _lib.check(lib.ow_s2d_linear_fwd(args, stream), "ow_s2d_linear_fwd")
    del ws
    return out, x


class _S2dLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w_d, w_a, factor, nchw, compute):
        wd = w_d.detach()
        if w_a is not None:
            # The folded weight is the product of the 16-bit weights both
            # reference GEMMs would use (f32 accumulation, one rounding).
            with torch.autocast("cuda", enabled=False):
                w_eff = w_a.detach().to(compute) @ wd.to(compute)
        else:
            w_eff = wd
        out, xk = _fwd(x.detach(), w_eff, factor, nchw, compute)
        # The backward needs x in the compute type: a 16-bit copy made for the
        # kernel is kept instead of x (half the bytes, no second cast).
        ctx.save_for_backward(xk if xk.dtype == compute else x.detach(), wd,
                              None if w_a is None else w_a.detach(), w_eff)
        ctx.factor, ctx.nchw, ctx.compute, ctx.x_dtype = factor, nchw, compute, x.dtype
        return out

    @staticmethod
    def backward(ctx, dy):
        x, wd, wa, w_eff = ctx.saved_tensors
        return (*s2d_linear_backward(dy, x, wd, wa, w_eff, ctx.factor, ctx.nchw, ctx.compute,
                                     ctx.needs_input_grad[:3], ctx.x_dtype), None, None, None)


def s2d_linear_backward(dy: Tensor, x: Tensor, wd: Tensor, wa: Tensor | None, w_eff: Tensor,
                        factor: int, nchw: bool, compute: torch.dtype,
                        needs: tuple[bool, ...] = (True, True, True),
                        x_dtype: torch.dtype | None = None):
    """Gradients ``(dx, dW_d, dW_a)`` of ``y = s2d(x) w_eff^T``, ``w_eff = W_a W_d``.

    ``dx`` is returned in ``x_dtype`` (default: x's dtype).

    Every product is taken in ``compute`` (the forward's dtype, f32
    accumulation on the GPU), as the reference's autocast GEMMs take theirs:
    the folded weight's gradient ``dW = dy^T s2d(x)``, then ``dW_d = W_a^T dW``
    and ``dW_a = dW W_d^T`` (``dW_d = dW`` without an anchor).
    """
    dy = dy.to(compute)
    n = dy.shape[-1]
    dy2 = dy.reshape(-1, n)
    xn = x.permute(0, 2, 3, 1) if nchw else x
    a = space_to_depth_nhwc(xn.to(compute), factor).reshape(dy2.shape[0], -1)
    acc = compute
    dw_eff = dy2.t() @ a
    dx = dwd = dwa = None
    if needs[0] and not nchw and _d2s_supported(dy, w_eff, factor, x_dtype or x.dtype)[0]:
        # one kernel: the GEMM stores through the inverse rearrangement
        dx = _d2s(dy, w_eff, factor, x_dtype or x.dtype)
    elif needs[0]:
        b, ho, wo = dy.shape[:3]
        f = factor
        c = w_eff.shape[1] // (f * f)
        da = (dy2 @ w_eff.to(compute)).view(b, ho, wo, f, f, c)  # [b, i, j, dy, dx, c]
        # One copy: the inverse rearrangement and the cast in the same pass.
        if nchw:
            dx = torch.empty((b, c, ho * f, wo * f), dtype=x_dtype or x.dtype, device=da.device)
            dx.view(b, c, ho, f, wo, f).copy_(da.permute(0, 5, 1, 3, 2, 4))
        else:
            dx = torch.empty((b, ho * f, wo * f, c), dtype=x_dtype or x.dtype, device=da.device)
            dx.view(b, ho, f, wo, f, c).copy_(da.permute(0, 1, 3, 2, 4, 5))
    if wa is None:
        if needs[1]:
            dwd = dw_eff.to(wd.dtype)
    else:
        if needs[1]:
            dwd = (wa.to(acc).t() @ dw_eff).to(wd.dtype)
        if needs[2]:
            dwa = (dw_eff @ wd.to(acc).t()).to(wa.dtype)
    return dx, dwd, dwa


def _d2s_args(y: Tensor | None, shape: tuple[int, int, int, int], y_dtype: torch.dtype, weight: Tensor,
              factor: int, out: Tensor | None, out_dtype: torch.dtype) -> _lib.D2sLinear:
    b, ho, wo, n = shape
    c = weight.shape[1] // (factor * factor)
    return _lib.D2sLinear(
        _lib.ptr(y), _lib.DTYPE_CODE.get(y_dtype, -1), b, ho * factor, wo * factor, c, factor, n,
        _lib.ptr(weight), _lib.DTYPE_CODE.get(weight.dtype, -1),
        _lib.ptr(out), _lib.DTYPE_CODE.get(out_dtype, -1), None, 0,
    )


def _d2s_supported(y: Tensor, weight: Tensor, factor: int,
                   out_dtype: torch.dtype) -> tuple[bool, str | None]:
    if y.device.type != "cuda":
        return False, "CUDA is unavailable"
    if y.dim() != 4 or weight.dim() != 2 or weight.shape[0] != y.shape[3]:
        return False, "y must be [B, Ho, Wo, N] and the weight [N, f^2 C]"
    if weight.shape[1] % (factor * factor):
        return False, "weight columns must be a multiple of factor^2"
    if weight.dtype not in (torch.float32, y.dtype):
        return False, f"weight dtype {weight.dtype} is neither float32 nor y's dtype"
    try:
        lib = _lib.load()
    except _lib.NativeLibraryError as exc:
        return False, str(exc)
    idx = y.device.index if y.device.index is not None else torch.cuda.current_device()
    if not lib.ow_device_supported(idx):
        return False, f"device {idx} is not sm_100 (B200-class)"
    args = _d2s_args(None, tuple(y.shape), y.dtype, weight, factor, None, out_dtype)
    args.weight = None  # a size query reads no pointer
    if lib.ow_d2s_linear_workspace_size(args) == 0:
        return False, "shape or dtype not supported by ow_d2s_linear_fwd"
    return True, None


def _d2s(y: Tensor, weight: Tensor, factor: int, out_dtype: torch.dtype) -> Tensor:
    lib = _lib.load()
    y = y.contiguous()
    weight = weight.contiguous()
    b, ho, wo, _ = y.shape
    c = weight.shape[1] // (factor * factor)
    out = torch.empty((b, ho * factor, wo * factor, c), dtype=out_dtype, device=y.device)
    args = _d2s_args(y, tuple(y.shape), y.dtype, weight, factor, out, out_dtype)
    n = lib.ow_d2s_linear_workspace_size(args)
    ws = torch.empty(max(n, 1), dtype=torch.uint8, device=y.device)
    args.workspace, args.workspace_bytes = ws.data_ptr(), n
    with torch.cuda.device(y.device):  # the library launches on the current device
        _lib.check(lib.ow_d2s_linear_fwd(args, _lib.stream_handle(y.device)), "ow_d2s_linear_fwd")
    del ws
    return out


def d2s_linear(y: Tensor, weight: Tensor, factor: int, out_dtype: torch.dtype | None = None) -> Tensor:
    """``depth_to_space_nhwc(y @ weight, factor)`` as one kernel (``ow_d2s_linear_fwd``).

    The input gradient of the downsample ``Linear(space_to_depth_nhwc(x))``
    (backbone.py:14-27, :128-132): ``y`` is the 16-bit gradient
    ``[B, Ho, Wo, N]``, ``weight`` the projection's ``[N, f^2 C]`` (f32 or
    y's dtype); the result is ``[B, f Ho, f Wo, C]`` in ``out_dtype`` (y's
    dtype by default, or float32 holding the values rounded to y's dtype).
    Raises ``RuntimeError`` when the kernel does not support the arguments.
    """
    out_dtype = out_dtype or y.dtype
    ok, why = _d2s_supported(y, weight, factor, out_dtype)
    if not ok:
        raise RuntimeError(f"d2s_linear not supported: {why}")
    return _d2s(y, weight, factor, out_dtype)


def s2d_linear(x: Tensor, weight: Tensor, factor: int, *, nchw: bool = False,
               anchor: Tensor | None = None) -> Tensor:
    """``Linear(space_to_depth(x, factor))`` (bias-free), then ``anchor`` if given.

    ``x`` is NHWC, or NCHW with ``nchw=True`` (the stem's image batch; the
    rearrangement then reads ``x.permute(0, 2, 3, 1)``).  ``weight`` is
    ``[N, factor^2 C]`` and ``anchor`` an optional ``[N, N]`` weight applied
    after it.  Returns NHWC ``[B, H/f, W/f, N]`` in the compute dtype: the
    autocast dtype when autocast is on, else x's dtype when it is 16-bit (the
    weights are rounded to it).  Raises ``RuntimeError`` when the kernel does
    not support the arguments (float32 compute included).
    """
    compute = _compute(x, weight)
    ok, why = s2d_linear_supported(x, weight, factor, nchw, compute)
    if not ok:
        raise RuntimeError(f"s2d_linear not supported: {why}")
    if anchor is not None and anchor.shape != (weight.shape[0], weight.shape[0]):
        raise ValueError(f"anchor must be [{weight.shape[0]}, {weight.shape[0]}], got {tuple(anchor.shape)}")
    return _S2dLinear.apply(x, weight, anchor, factor, nchw, compute)


# ---------------------------------------------------------------------------
# Backbone features (backbone.py:166-187) with the fused projections
# ---------------------------------------------------------------------------
def _anchor(stage: Any) -> Tensor | None:
    a = getattr(stage, "anchor", None)
    return None if a is None else a.weight


def features_supported(model: Any, x: Tensor) -> tuple[bool, str | None]:
    """Whether ``forward_features`` can run every projection of ``model`` on ``x``."""
    if x.dim() != 4:
        return False, "input must be [B, 3, H, W]"
    compute = _compute(x, model.stem_proj.weight)
    ok, why = s2d_linear_supported(x, model.stem_proj.weight, 4, True, compute)
    if not ok:
        return False, f"stem: {why}"
    b, _, h, w = x.shape
    h, w, c = h // 4, w // 4, model.stem_proj.weight.shape[0]
    for i, ds in enumerate(model.downsamples):
        ok, why = _shape_supported(x.device, (b, h, w, c), compute, ds.weight, 2, False, compute)
        if not ok:
            return False, f"downsample {i}: {why}"
        h, w, c = h // 2, w // 2, ds.weight.shape[0]
    return True, None


def forward_features(model: Any, x: Tensor) -> "OrderedDict[str, Tensor]":
    """``OmniWeaveBackbone.forward_features`` with fused stem and downsamples.

    Same outputs (four NHWC feature maps ``stage1`` .. ``stage4``) and the same
    modules as backbone.py:166-187; each stage's blocks run as the stage
    would run them, with its anchor folded into the projection before it.
    """
    stages = list(model.stages)
    x = s2d_linear(x, model.stem_proj.weight, 4, nchw=True, anchor=_anchor(stages[0]))
    features: OrderedDict[str, Tensor] = OrderedDict()
    for i, stage in enumerate(stages):
        for block in stage.blocks:
            x = block(x)
        features[f"stage{i + 1}"] = x
        if i < len(stages) - 1:
            x = s2d_linear(x, model.downsamples[i].weight, 2, anchor=_anchor(stages[i + 1]))
    return features

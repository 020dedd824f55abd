"""BiGEMM operator API and the ``cuda`` backend.

Mirrors the reference operator surface:

* ``bigemm(*, x, plan, a_u, a_v, a_o, b_u, b_v, b_o, gamma, backend)``
  (omniweave/ops/bigemm.py:24-73) -- returns the residual delta;
* ``select_backend(x, requested, support_check)`` (omniweave/ops/dispatch.py:13-49)
  -- the same policy with ``"cuda"`` in the role the reference gives
  ``"triton"``;
* ``cuda_is_supported(x, plan, b_u)`` -- the support check, in the shape of
  ``triton_is_supported`` (omniweave/ops/triton.py:26-55).

The ``cuda`` backend calls the C ABI of ``libomniwave_b200.so`` through
``torch.autograd.Function``s: forward and backward are both CUDA kernels
(there is no Triton, no PyTorch recompute and no CPU fallback on this path).
``block_forward`` is the fused ``OmniWeaveBlock.forward`` (RMSNorm prologue,
residual epilogue) used by ``omniwave_b200.block``.
"""

from __future__ import annotations

import logging
import threading
from collections.abc import Callable

import torch
from torch import Tensor

from omniwave_b200 import _lib
from omniwave_b200.routing import RoutePlan

logger = logging.getLogger(__name__)

__all__ = [
    "bigemm",
    "bigemm_delta_cuda",
    "block_forward",
    "cuda_is_supported",
    "drop_path_scale",
    "select_backend",
    "VALID_BACKENDS",
]

VALID_BACKENDS = ("reference", "compile", "triton", "cuda", "auto")
RMS_EPS = 1e-6  # omniweave/models/block.py:84


# ---------------------------------------------------------------------------
# Dispatch policy (reference omniweave/ops/dispatch.py:13-49)
# ---------------------------------------------------------------------------
def select_backend(
    x: Tensor,
    requested: str,
    support_check: Callable[[Tensor], tuple[bool, str | None]],
) -> tuple[str, str | None]:
    """Choose the execution backend.

    ``"reference"``, ``"compile"`` and ``"triton"`` pass through unchanged.
    ``"cuda"`` and ``"auto"`` consult ``support_check``: when it passes the
    answer is ``"cuda"``; a forced ``"cuda"`` that is unsupported raises
    ``RuntimeError(reason)``; ``"auto"`` logs the reason and answers
    ``"reference"`` (the reference's own fallback policy, which lives in the
    caller's ``omniweave`` install -- this package computes only ``"cuda"``).
    Unknown names raise ``ValueError``.
    """
    if requested not in VALID_BACKENDS:
        raise ValueError(f"unknown backend: {requested!r}")
    if requested in ("reference", "compile", "triton"):
        return requested, None
    supported, reason = support_check(x)
    if supported:
        return "cuda", None
    if requested == "cuda":
        raise RuntimeError(reason)
    logger.info("falling back to reference backend: %s", reason)
    return "reference", reason


# ---------------------------------------------------------------------------
# Support check
# ---------------------------------------------------------------------------
_SUPPORTED_DTYPES = (torch.float32, torch.float64, torch.bfloat16, torch.float16)


def _device_ok(device: torch.device) -> tuple[bool, str | None]:
    try:
        lib = _lib.load()
    except _lib.NativeLibraryError as exc:
        return False, str(exc)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if not lib.ow_device_supported(idx):
        return False, f"device {idx} is not sm_100 (B200-class)"
    return True, None


def cuda_is_supported(x: Tensor, plan: RoutePlan, b_u: Tensor) -> tuple[bool, str | None]:
    """``(is_supported, reason_if_not)`` for the ``cuda`` backend."""
    if not x.is_cuda:
        return False, "CUDA is unavailable"
    if x.dtype not in _SUPPORTED_DTYPES:
        return False, f"unsupported dtype {x.dtype}"
    q_s, g = plan.token_indices.shape
    if g != 16:
        return False, f"unsupported spatial tile g={g}; expected 16"
    if b_u.dim() != 3 or b_u.shape[0] != plan.channel_indices.shape[0] \
            or b_u.shape[1] != plan.channel_indices.shape[1]:
        return False, "b_u shape does not match the plan's channel groups"
    return _device_ok(x.device)


# ---------------------------------------------------------------------------
# Device route tables: int32 copies, uploaded once per (plan, device)
# ---------------------------------------------------------------------------
_tables: dict[tuple[int, str], tuple[RoutePlan, Tensor, Tensor]] = {}
_tables_lock = threading.Lock()


def _validate_plan(plan: RoutePlan) -> None:
    n = plan.height * plan.width
    c = plan.channels
    tok, tm = plan.token_indices, plan.token_mask
    ch, cm = plan.channel_indices, plan.channel_mask
    if tok.dim() != 2 or ch.dim() != 2 or tok.shape != tm.shape or ch.shape != cm.shape:
        raise ValueError("route plan tables have inconsistent shapes")
    if not torch.equal(tok >= n, ~tm) or not torch.equal(ch >= c, ~cm):
        raise ValueError("route plan pads must be exactly the masked entries")
    if int(tok.min()) < 0 or int(ch.min()) < 0 or int(tok.max()) > n or int(ch.max()) > c:
        raise ValueError("route plan index out of range")
    vt, vc = tok[tm], ch[cm]
    if vt.numel() != n or vc.numel() != c or torch.unique(vt).numel() != n \
            or torch.unique(vc).numel() != c:
        raise ValueError("route plan must visit every token and channel exactly once")


def channel_stride_hint(plan: RoutePlan) -> int:
    """The route's channel-layout hint for the C ABI (``ow_route_t.ch_stride``):
    S when every channel group is ``c0 + S*k`` (S = 1: one run starting on a
    multiple of 8; S in {2, 4, 8}: the stride-Q_c groups of radix levels 1
    and 2 with c0 < S), else 0 (unknown)."""
    ch = plan.channel_indices
    q_c, d = ch.shape
    if plan.channels % 8 or not bool(plan.channel_mask.all()):
        return 0
    c0 = ch[:, :1]
    if d == 1:
        return 0
    steps = ch[:, 1:] - ch[:, :-1]
    s = int(steps[0, 0])
    if s not in (1, 2, 4, 8) or not bool((steps == s).all()):
        return 0
    if s == 1:
        return 1 if bool((c0 % 8 == 0).all()) else 0
    return s if bool((c0 < s).all()) and s * d <= plan.channels else 0


def route_tables(plan: RoutePlan, device: torch.device) -> tuple[Tensor, Tensor]:
    """int32 device copies of ``plan.token_indices`` / ``plan.channel_indices``."""
    key = (id(plan), str(device))
    hit = _tables.get(key)
    if hit is not None and hit[0] is plan:
        return hit[1], hit[2]
    with _tables_lock:
        hit = _tables.get(key)
        if hit is not None and hit[0] is plan:
            return hit[1], hit[2]
        _validate_plan(plan)
        tok = plan.token_indices.to(torch.int32).reshape(-1).to(device)
        ch = plan.channel_indices.to(torch.int32).reshape(-1).to(device)
        _tables[key] = (plan, tok, ch)  # keeps ``plan`` alive, so its id stays unique
        return tok, ch


_hints: dict[int, tuple[RoutePlan, int]] = {}


def _stride_hint(plan: RoutePlan) -> int:
    hit = _hints.get(id(plan))
    if hit is not None and hit[0] is plan:
        return hit[1]
    v = channel_stride_hint(plan)
    _hints[id(plan)] = (plan, v)  # keeps ``plan`` alive, so its id stays unique
    return v


# ---------------------------------------------------------------------------
# Argument marshalling
# ---------------------------------------------------------------------------
def _compute_dtype(x: Tensor) -> torch.dtype:
    if x.is_cuda and torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    return x.dtype


def _weights_common(ws: list[Tensor]) -> tuple[list[Tensor], torch.dtype]:
    dt = ws[0].dtype
    for w in ws[1:]:
        dt = torch.promote_types(dt, w.dtype)
    return [w.detach().to(dt).contiguous() for w in ws], dt


def _make_args(x, plan, tok, ch, weights, w_dtype, compute, rstd, norm_w, scale, residual,
               out, out_dtype) -> _lib.Args:
    b, h, w, c = x.shape
    a_u, a_v, a_o, b_u, b_v, b_o, gamma = weights
    q_c, d, rd = b_u.shape
    q_s, g = plan.token_indices.shape
    r = _lib.Route(b, h, w, c, q_s, q_c, g, d, rd, tok.data_ptr(), ch.data_ptr(), _stride_hint(plan))
    return _lib.Args(
        r, x.data_ptr(), _lib.DTYPE_CODE[x.dtype], _lib.DTYPE_CODE[compute],
        _lib.ptr(rstd), _lib.ptr(norm_w),
        a_u.data_ptr(), a_v.data_ptr(), a_o.data_ptr(),
        b_u.data_ptr(), b_v.data_ptr(), b_o.data_ptr(), gamma.data_ptr(),
        _lib.DTYPE_CODE[w_dtype], _lib.ptr(scale), int(residual),
        _lib.ptr(out), _lib.DTYPE_CODE[out_dtype], None, 0,
    )


def _workspace(lib, args: _lib.Args, device, backward: bool) -> Tensor:
    n = lib.ow_bigemm_workspace_size(args, 1 if backward else 0)
    if n == 0:
        _lib.check(1, "ow_bigemm_workspace_size")
    ws = torch.empty(n, dtype=torch.uint8, device=device)
    args.workspace = ws.data_ptr()
    args.workspace_bytes = n
    return ws


def _check_shapes(x: Tensor, plan: RoutePlan, weights: list[Tensor]) -> None:
    a_u, a_v, a_o, b_u, b_v, b_o, gamma = weights
    if x.dim() != 4:
        raise ValueError(f"x must be [B,H,W,C], got {tuple(x.shape)}")
    b, h, w, c = x.shape
    if (h, w, c) != (plan.height, plan.width, plan.channels):
        raise ValueError(f"x shape {tuple(x.shape)} does not match plan {plan.height}x{plan.width}x{plan.channels}")
    q_s, g = plan.token_indices.shape
    q_c, d = plan.channel_indices.shape
    for name, t in (("a_u", a_u), ("a_v", a_v), ("a_o", a_o)):
        if t.shape != (g, g):
            raise ValueError(f"{name} must be [{g},{g}], got {tuple(t.shape)}")
    if b_u.dim() != 3 or b_u.shape[:2] != (q_c, d) or b_v.shape != b_u.shape:
        raise ValueError("b_u/b_v must be [Q_c, d, rd] matching the plan")
    rd = b_u.shape[2]
    if b_o.shape != (q_c, rd, d):
        raise ValueError(f"b_o must be [{q_c},{rd},{d}], got {tuple(b_o.shape)}")
    if gamma.shape != (c,):
        raise ValueError(f"gamma must be [{c}], got {tuple(gamma.shape)}")


def _grad_buffers(x, weights, w_dtype, with_norm):
    dev = x.device
    g = [torch.empty(w.shape, dtype=w_dtype, device=dev) for w in weights]
    dnw = torch.empty(x.shape[-1], dtype=w_dtype, device=dev) if with_norm else None
    return g, dnw


# ---------------------------------------------------------------------------
# Operator autograd function
# ---------------------------------------------------------------------------
class _CudaBiGEMM(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, plan, compute, a_u, a_v, a_o, b_u, b_v, b_o, gamma):
        lib = _lib.load()
        x_c = x.detach().contiguous()
        weights, w_dtype = _weights_common([a_u, a_v, a_o, b_u, b_v, b_o, gamma])
        tok, ch = route_tables(plan, x.device)
        out_dtype = torch.promote_types(compute, gamma.dtype)
        out = torch.empty(x.shape, dtype=out_dtype, device=x.device)
        args = _make_args(x_c, plan, tok, ch, weights, w_dtype, compute, None, None, None,
                          False, out, out_dtype)
        ws = _workspace(lib, args, x.device, backward=False)
        with torch.cuda.device(x.device):  # the library launches on the current device
            _lib.check(lib.ow_bigemm_fwd(args, _lib.stream_handle(x.device)), "ow_bigemm_fwd")
        del ws
        ctx.save_for_backward(x_c, *weights)
        ctx.plan, ctx.compute, ctx.w_dtype, ctx.out_dtype = plan, compute, w_dtype, out_dtype
        ctx.in_dtypes = [t.dtype for t in (x, a_u, a_v, a_o, b_u, b_v, b_o, gamma)]
        return out

    @staticmethod
    def backward(ctx, dout):
        lib = _lib.load()
        x, *weights = ctx.saved_tensors
        plan = ctx.plan
        tok, ch = route_tables(plan, x.device)
        dout = dout.to(ctx.out_dtype).contiguous()
        args = _make_args(x, plan, tok, ch, weights, ctx.w_dtype, ctx.compute, None, None, None,
                          False, None, ctx.out_dtype)
        ws = _workspace(lib, args, x.device, backward=True)
        dx = torch.empty_like(x)
        gw, _ = _grad_buffers(x, weights, ctx.w_dtype, False)
        grads = _lib.Grads(dout.data_ptr(), dx.data_ptr(), *[g.data_ptr() for g in gw], None)
        with torch.cuda.device(x.device):
            _lib.check(lib.ow_bigemm_bwd(args, grads, _lib.stream_handle(x.device)), "ow_bigemm_bwd")
        del ws
        out = [dx] + gw
        out = [o.to(dt) for o, dt in zip(out, ctx.in_dtypes)]
        return (out[0], None, None, *out[1:])


def bigemm_delta_cuda(*, x, plan, a_u, a_v, a_o, b_u, b_v, b_o, gamma) -> Tensor:
    """BiGEMM delta on the B200 kernels (forward and backward)."""
    supported, reason = cuda_is_supported(x, plan, b_u)
    if not supported:
        raise RuntimeError(f"cuda backend not supported: {reason}")
    _check_shapes(x, plan, [a_u, a_v, a_o, b_u, b_v, b_o, gamma])
    return _CudaBiGEMM.apply(x, plan, _compute_dtype(x), a_u, a_v, a_o, b_u, b_v, b_o, gamma)


def _reference_bigemm():
    """The reference package's own ``bigemm`` (for its reference/compile/triton backends)."""
    try:
        from omniweave.ops import bigemm as ref_mod
    except ImportError as exc:
        raise RuntimeError(
            "the 'reference', 'compile' and 'triton' backends belong to the omniweave package, "
            "which is not importable here; omniwave_b200 implements 'cuda'"
        ) from exc
    # After omniwave_b200.integration.install() the module attribute is the
    # patched dispatcher; it passes these names on to the reference function.
    return ref_mod.bigemm


def bigemm(
    *,
    x: Tensor,
    plan: RoutePlan,
    a_u: Tensor,
    a_v: Tensor,
    a_o: Tensor,
    b_u: Tensor,
    b_v: Tensor,
    b_o: Tensor,
    gamma: Tensor,
    backend: str = "reference",
) -> Tensor:
    """Compute the BiGEMM residual delta (reference ``bigemm``, ops/bigemm.py:24-73).

    Same signature and default as the reference.  ``"cuda"`` runs this
    package's kernels; ``"auto"`` picks ``"cuda"`` when it is supported and
    otherwise applies the reference's own ``"auto"`` policy; ``"reference"``,
    ``"compile"`` and ``"triton"`` are passed to the installed ``omniweave``
    package.  Unknown names raise ``ValueError``.
    """
    kwargs = dict(x=x, plan=plan, a_u=a_u, a_v=a_v, a_o=a_o, b_u=b_u, b_v=b_v, b_o=b_o, gamma=gamma)
    if backend not in VALID_BACKENDS:
        raise ValueError(
            f"unknown backend: {backend!r}; expected 'reference', 'compile', 'triton', "
            f"'cuda', or 'auto'"
        )
    if backend == "auto":
        chosen, _ = select_backend(x, "auto", lambda t: cuda_is_supported(t, plan, b_u))
        if chosen == "cuda":
            return bigemm_delta_cuda(**kwargs)
        return _reference_bigemm()(backend="auto", **kwargs)
    if backend != "cuda":
        return _reference_bigemm()(backend=backend, **kwargs)
    return bigemm_delta_cuda(**kwargs)


# ---------------------------------------------------------------------------
# Fused block: x + scale * bigemm(rmsnorm(x))   (block.py:80-108)
# ---------------------------------------------------------------------------
class _CudaBlock(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, plan, compute, scale, norm_w, a_u, a_v, a_o, b_u, b_v, b_o, gamma):
        lib = _lib.load()
        x_c = x.detach().contiguous()
        b, h, w, c = x.shape
        dev = x.device
        weights, w_dtype = _weights_common([a_u, a_v, a_o, b_u, b_v, b_o, gamma])
        nw = norm_w.detach().to(w_dtype).contiguous()
        tok, ch = route_tables(plan, dev)
        stat_dtype = torch.float64 if compute == torch.float64 else torch.float32
        rstd = torch.empty(b * h * w, dtype=stat_dtype, device=dev)
        stream = _lib.stream_handle(dev)
        with torch.cuda.device(dev):
            _lib.check(lib.ow_rmsnorm_rstd(x_c.data_ptr(), _lib.DTYPE_CODE[x.dtype],
                                           _lib.DTYPE_CODE[compute], b * h * w, c, RMS_EPS,
                                           rstd.data_ptr(), stream), "ow_rmsnorm_rstd")
        delta_dtype = torch.promote_types(compute, gamma.dtype)
        out_dtype = torch.promote_types(x.dtype, delta_dtype)
        out = torch.empty(x.shape, dtype=out_dtype, device=dev)
        scale_c = None if scale is None else scale.to(torch.float32).contiguous()
        args = _make_args(x_c, plan, tok, ch, weights, w_dtype, compute, rstd, nw, scale_c,
                          True, out, out_dtype)
        ws = _workspace(lib, args, dev, backward=False)
        with torch.cuda.device(dev):
            _lib.check(lib.ow_bigemm_fwd(args, stream), "ow_bigemm_fwd")
        del ws
        ctx.save_for_backward(x_c, rstd, nw, *weights)
        ctx.scale = scale_c
        ctx.plan, ctx.compute, ctx.w_dtype, ctx.out_dtype = plan, compute, w_dtype, out_dtype
        ctx.in_dtypes = [t.dtype for t in (x, norm_w, a_u, a_v, a_o, b_u, b_v, b_o, gamma)]
        return out

    @staticmethod
    def backward(ctx, dout):
        lib = _lib.load()
        x, rstd, nw, *weights = ctx.saved_tensors
        plan = ctx.plan
        tok, ch = route_tables(plan, x.device)
        dout = dout.to(ctx.out_dtype).contiguous()
        args = _make_args(x, plan, tok, ch, weights, ctx.w_dtype, ctx.compute, rstd, nw,
                          ctx.scale, True, None, ctx.out_dtype)
        ws = _workspace(lib, args, x.device, backward=True)
        dx = torch.empty_like(x)
        gw, dnw = _grad_buffers(x, weights, ctx.w_dtype, True)
        grads = _lib.Grads(dout.data_ptr(), dx.data_ptr(), *[g.data_ptr() for g in gw],
                           dnw.data_ptr())
        with torch.cuda.device(x.device):
            _lib.check(lib.ow_bigemm_bwd(args, grads, _lib.stream_handle(x.device)), "ow_bigemm_bwd")
        del ws
        out = [dx, dnw] + gw
        out = [o.to(dt) for o, dt in zip(out, ctx.in_dtypes)]
        return (out[0], None, None, None, *out[1:])


def drop_path_scale(x: Tensor, gamma: Tensor, rate: float, training: bool) -> Tensor | None:
    """Per-sample drop-path scale ``keep_mask / keep_probability`` of block.py:99-107.

    Draws the same Bernoulli sample as the reference (a ``[B,1,1,1]`` tensor of
    the delta's dtype on ``x``'s device), so a seeded run keeps the same
    samples; ``None`` when drop-path is inactive.
    """
    if not (training and rate):
        return None
    keep = 1.0 - rate
    compute = torch.get_autocast_dtype("cuda") if (x.is_cuda and torch.is_autocast_enabled("cuda")) else x.dtype
    dtype = torch.promote_types(torch.promote_types(compute, gamma.dtype), x.dtype)
    mask = torch.empty((x.shape[0], 1, 1, 1), dtype=dtype, device=x.device).bernoulli_(keep)
    return (mask / keep).reshape(-1)


def block_forward(x: Tensor, plan: RoutePlan, norm_w: Tensor, a_u: Tensor, a_v: Tensor,
                  a_o: Tensor, b_u: Tensor, b_v: Tensor, b_o: Tensor, gamma: Tensor,
                  sample_scale: Tensor | None = None) -> Tensor:
    """Fused ``x + sample_scale[b] * bigemm(rmsnorm(x))`` on the B200 kernels."""
    supported, reason = cuda_is_supported(x, plan, b_u)
    if not supported:
        raise RuntimeError(f"cuda backend not supported: {reason}")
    _check_shapes(x, plan, [a_u, a_v, a_o, b_u, b_v, b_o, gamma])
    if norm_w.shape != (x.shape[-1],):
        raise ValueError("norm weight must be [C]")
    return _CudaBlock.apply(x, plan, _compute_dtype(x), sample_scale, norm_w,
                            a_u, a_v, a_o, b_u, b_v, b_o, gamma)

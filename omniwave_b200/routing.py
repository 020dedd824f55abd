"""Route plans for the BiGEMM operator: local, shifted and radix token routes.

A route plan says which 16 tokens form each spatial tile and which ``d``
channels form each channel group.  This module mirrors the reference's
``omniweave/models/routing.py`` API (``RoutePlan`` :17-33,
``build_route_plan`` :128-179, ``build_stage_schedule`` :182-198,
``radix_order`` :93-104) so that callers and state are interchangeable, but
the orders are built with vectorised integer arithmetic instead of nested
Python loops: the largest plans (65,536 tokens at 1024x1024 input) are built
in milliseconds.

Index conventions follow the reference: indices are int64 CPU tensors, the
token pad index is ``N = H*W`` and the channel pad index is ``C``.  The CUDA
backend uploads an int32 copy of each table once per (plan, device).
"""

from __future__ import annotations

import functools
import math
from dataclasses import dataclass

import numpy as np
import torch

__all__ = [
    "RoutePlan",
    "build_route_plan",
    "build_stage_schedule",
    "radix_order",
    "local_token_order",
    "shifted_token_order",
    "channel_order",
]

_WINDOW = 4
_SHIFT = 2


@dataclass(frozen=True)
class RoutePlan:
    """Immutable routing specification for one block invocation.

    Field meaning is identical to the reference ``RoutePlan``
    (``omniweave/models/routing.py:17-33``).
    """

    token_indices: torch.Tensor    # [Q_s, g] int64, pad index = N
    channel_indices: torch.Tensor  # [Q_c, d] int64, pad index = C
    token_mask: torch.Tensor       # [Q_s, g] bool
    channel_mask: torch.Tensor     # [Q_c, d] bool
    height: int
    width: int
    channels: int
    route: str
    radix_level: int


def local_token_order(height: int, width: int, window: int = _WINDOW) -> np.ndarray:
    """Tokens grouped by ``window x window`` windows, windows in raster order.

    Same order as ``_local_token_order`` (reference ``routing.py:57-65``):
    windows are visited row-major, tokens inside a window row-major, and
    windows at the right/bottom edge are clipped to the image.
    """
    rows, cols = np.meshgrid(np.arange(height), np.arange(width), indexing="ij")
    win_cols = -(-width // window)
    # Sort key: (window row, window col, row in window, col in window).
    key = (((rows // window) * win_cols + cols // window) * window + rows % window) * window + cols % window
    flat = (rows * width + cols).reshape(-1)
    return flat[np.argsort(key.reshape(-1), kind="stable")]


def shifted_token_order(
    height: int, width: int, window: int = _WINDOW, shift: int = _SHIFT
) -> np.ndarray:
    """Windows displaced by ``-shift`` with cyclic wrap, first occurrence kept.

    Same order as ``_shifted_token_order`` (reference ``routing.py:68-90``):
    every window origin in ``range(-shift, dim - shift, window)`` contributes a
    full ``window x window`` block of wrapped coordinates; a token that appears
    in more than one block keeps the position of its first appearance.
    """
    row_bases = np.arange(-shift, height - shift, window)
    col_bases = np.arange(-shift, width - shift, window)
    off = np.arange(window)
    # Shape [row_base, col_base, r, c] in the visiting order.
    r = (row_bases[:, None, None, None] + off[None, None, :, None]) % height
    c = (col_bases[None, :, None, None] + off[None, None, None, :]) % width
    seq = (r * width + c).reshape(-1)
    _, first = np.unique(seq, return_index=True)
    return seq[np.sort(first)]


def radix_order(token_count: int, group_size: int, level: int) -> list[int]:
    """Mixed-radix order: each group of ``group_size`` differs in digit ``level``.

    Same order as reference ``routing.py:93-104``: stride ``g**level``, block
    ``g**(level+1)``; indices at or beyond ``token_count`` are dropped.
    """
    return _radix_order_array(token_count, group_size, level).tolist()


def _radix_order_array(token_count: int, group_size: int, level: int) -> np.ndarray:
    stride = group_size ** level
    block = stride * group_size
    bases = np.arange(0, token_count, block, dtype=np.int64)
    offsets = np.arange(stride, dtype=np.int64)
    digits = np.arange(group_size, dtype=np.int64)
    idx = bases[:, None, None] + digits[None, None, :] * stride + offsets[None, :, None]
    idx = idx.reshape(-1)
    return idx[idx < token_count]


def channel_order(channels: int, channel_tile: int, radix_level: int) -> np.ndarray:
    """Channel order for a radix level (reference ``_channel_order`` :107-121).

    Level 0 (or a single group) is the identity.  Otherwise channel ``i`` is
    dealt to group ``i % Q_c`` and the list of groups is rotated left by
    ``radix_level % Q_c``; group ``q`` therefore holds the channels
    ``{(q + rot) % Q_c + Q_c * j}``.
    """
    n_groups = math.ceil(channels / channel_tile)
    ident = np.arange(channels, dtype=np.int64)
    if radix_level == 0 or n_groups <= 1:
        return ident
    rot = radix_level % n_groups
    parts = [ident[(q + rot) % n_groups :: n_groups] for q in range(n_groups)]
    return np.concatenate(parts)


def _pad_and_mask(order: np.ndarray, group_size: int, pad_value: int) -> tuple[torch.Tensor, torch.Tensor]:
    n = int(order.shape[0])
    groups = -(-n // group_size)
    total = groups * group_size
    idx = np.full(total, pad_value, dtype=np.int64)
    idx[:n] = order
    mask = np.zeros(total, dtype=bool)
    mask[:n] = True
    return (
        torch.from_numpy(idx.reshape(groups, group_size)),
        torch.from_numpy(mask.reshape(groups, group_size)),
    )


@functools.lru_cache(maxsize=256)
def build_route_plan(
    height: int,
    width: int,
    channels: int,
    spatial_tile: int,
    channel_tile: int,
    route: str,
    radix_level: int = 0,
) -> RoutePlan:
    """Build the cached route plan (reference ``build_route_plan`` :128-179).

    ``radix_level`` selects both the radix digit (route ``"radix"``) and the
    channel-group rotation (any route), as in the reference.
    """
    n_tokens = height * width
    if route == "local":
        tokens = local_token_order(height, width)
    elif route == "shifted":
        tokens = shifted_token_order(height, width)
    elif route == "radix":
        tokens = _radix_order_array(n_tokens, spatial_tile, radix_level)
    else:
        raise ValueError(f"unknown route type: {route!r}")
    token_indices, token_mask = _pad_and_mask(tokens, spatial_tile, n_tokens)
    channel_indices, channel_mask = _pad_and_mask(
        channel_order(channels, channel_tile, radix_level), channel_tile, channels
    )
    return RoutePlan(
        token_indices=token_indices,
        channel_indices=channel_indices,
        token_mask=token_mask,
        channel_mask=channel_mask,
        height=height,
        width=width,
        channels=channels,
        route=route,
        radix_level=radix_level,
    )


_SCHEDULE_CYCLE: tuple[tuple[str, int], ...] = (
    ("local", 0),
    ("shifted", 0),
    ("radix", 0),
    ("radix", 1),
    ("radix", 2),
)


def build_stage_schedule(depth: int) -> list[tuple[str, int]]:
    """Route schedule of a stage (reference ``build_stage_schedule`` :182-198).

    Cycles local, shifted, radix-0, radix-1, radix-2, starting with local.
    """
    return [_SCHEDULE_CYCLE[i % len(_SCHEDULE_CYCLE)] for i in range(depth)]

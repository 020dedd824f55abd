"""Loop-level restatement of the reference route plans (test oracle only).

Each function follows ``omniweave/models/routing.py`` of the reference at the
cited lines.  Plans are returned as numpy arrays:
``(token_indices [Q_s,g] int64, channel_indices [Q_c,d] int64,
token_mask [Q_s,g] bool, channel_mask [Q_c,d] bool)``.
"""

from __future__ import annotations

import math

import numpy as np


def local_order(height: int, width: int, window: int = 4) -> list[int]:
    """``_local_token_order`` -- reference routing.py:57-65."""
    out: list[int] = []
    for rb in range(0, height, window):
        for cb in range(0, width, window):
            for r in range(rb, min(rb + window, height)):
                for c in range(cb, min(cb + window, width)):
                    out.append(r * width + c)
    return out


def shifted_order(height: int, width: int, window: int = 4, shift: int = 2) -> list[int]:
    """``_shifted_token_order`` -- reference routing.py:68-90."""
    seq: list[int] = []
    for rb in range(-shift, height - shift, window):
        for cb in range(-shift, width - shift, window):
            for r in range(rb, rb + window):
                for c in range(cb, cb + window):
                    seq.append((r % height) * width + (c % width))
    seen: set[int] = set()
    out: list[int] = []
    for t in seq:
        if t not in seen:
            seen.add(t)
            out.append(t)
    return out


def radix_order(n: int, g: int, level: int) -> list[int]:
    """``radix_order`` -- reference routing.py:93-104."""
    stride = g ** level
    block = stride * g
    out: list[int] = []
    for base in range(0, n, block):
        for off in range(stride):
            for digit in range(g):
                t = base + digit * stride + off
                if t < n:
                    out.append(t)
    return out


def channel_order(c: int, d: int, level: int) -> list[int]:
    """``_channel_order`` -- reference routing.py:107-121."""
    groups = math.ceil(c / d)
    if level == 0 or groups <= 1:
        return list(range(c))
    buckets: list[list[int]] = [[] for _ in range(groups)]
    for i in range(c):
        buckets[i % groups].append(i)
    rot = level % groups
    buckets = buckets[rot:] + buckets[:rot]
    return [i for b in buckets for i in b]


def pad_and_mask(order: list[int], size: int, pad: int) -> tuple[np.ndarray, np.ndarray]:
    """``_pad_and_mask`` -- reference routing.py:40-54."""
    n = len(order)
    groups = math.ceil(n / size)
    total = groups * size
    idx = np.array(order + [pad] * (total - n), dtype=np.int64).reshape(groups, size)
    mask = np.zeros(total, dtype=bool)
    mask[:n] = True
    return idx, mask.reshape(groups, size)


def build_plan(h: int, w: int, c: int, g: int, d: int, route: str, level: int = 0):
    """``build_route_plan`` -- reference routing.py:128-179."""
    n = h * w
    if route == "local":
        order = local_order(h, w)
    elif route == "shifted":
        order = shifted_order(h, w)
    elif route == "radix":
        order = radix_order(n, g, level)
    else:
        raise ValueError(route)
    tok, tmask = pad_and_mask(order, g, n)
    ch, cmask = pad_and_mask(channel_order(c, d, level), d, c)
    return tok, ch, tmask, cmask

"""numpy restatement of the reference BiGEMM operator (test oracle only).

Follows ``omniweave/ops/reference.py`` of the reference:

* ``pack``     -- ``pack_tiles`` :16-64 (pad row/channel, two gathers, mask)
* ``unpack``   -- ``unpack_tiles`` :67-117 (two scatter-adds, trim)
* ``forward``  -- ``bigemm_delta_reference`` :120-173
  ``U = A_u T B_u``, ``V = A_v T B_v``, ``Z = silu(U) * V``,
  ``delta = A_o Z B_o``, then mask and LayerScale ``gamma[ch_idx] * ch_mask``.
* ``backward`` -- the gradients torch autograd takes through that graph,
  written out by hand (chain rule through the einsums, silu and gathers).
* ``block_forward`` / ``block_backward`` -- ``OmniWeaveBlock.forward``
  (``omniweave/models/block.py:80-108``): RMSNorm with eps 1e-6, BiGEMM,
  optional per-sample drop-path scale, residual add.

All arithmetic happens in the dtype of the inputs (use float64 for a tight
reference, float32 to time the CPU baseline).  Contractions are arranged as
large matrix products so numpy's BLAS uses every host core.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

EPS = 1e-6  # omniweave/models/block.py:84


@dataclass
class Plan:
    tok: np.ndarray    # [Q_s, g] int64, pad = N
    ch: np.ndarray     # [Q_c, d] int64, pad = C
    tmask: np.ndarray  # [Q_s, g] bool
    cmask: np.ndarray  # [Q_c, d] bool
    h: int
    w: int
    c: int

    @property
    def n(self) -> int:
        return self.h * self.w

    def unique(self) -> bool:
        t = self.tok[self.tmask]
        c = self.ch[self.cmask]
        return len(np.unique(t)) == len(t) and len(np.unique(c)) == len(c)


def make_plan(h, w, c, g, d, route, level=0) -> Plan:
    from oracle.routing import build_plan

    tok, ch, tm, cm = build_plan(h, w, c, g, d, route, level)
    return Plan(tok, ch, tm, cm, h, w, c)


def _mask(p: Plan) -> np.ndarray:
    # [Q_s, Q_c, g, d], reference.py:51-59
    return p.tmask[:, None, :, None] & p.cmask[None, :, None, :]


def pack(x: np.ndarray, p: Plan) -> np.ndarray:
    """reference.py:16-64 -> tiles [B, Q_s, Q_c, g, d] (mask applied)."""
    b = x.shape[0]
    n, c = p.n, p.c
    flat = np.zeros((b, n + 1, c + 1), dtype=x.dtype)
    flat[:, :n, :c] = x.reshape(b, n, c)
    qs, g = p.tok.shape
    qc, d = p.ch.shape
    t = flat[:, p.tok.reshape(-1), :][:, :, p.ch.reshape(-1)]
    t = t.reshape(b, qs, g, qc, d).transpose(0, 1, 3, 2, 4)
    return t * _mask(p).astype(x.dtype)


def unpack(tiles: np.ndarray, p: Plan) -> np.ndarray:
    """reference.py:67-117 -> [B, H, W, C] (scatter-add, then trim)."""
    b, qs, qc, g, d = tiles.shape
    n, c = p.n, p.c
    vals = tiles.transpose(0, 1, 3, 2, 4).reshape(b, qs * g, qc * d)
    out = np.zeros((b, n + 1, c + 1), dtype=tiles.dtype)
    ti = p.tok.reshape(-1)
    ci = p.ch.reshape(-1)
    if p.unique():
        # Valid positions are distinct, so scatter-add equals assignment there;
        # pad entries land in row N / column C, which are trimmed.
        vm = (p.tmask.reshape(-1)[:, None] & p.cmask.reshape(-1)[None, :])
        sub = out[:, ti[:, None], ci[None, :]]
        sub = np.where(vm[None], vals, sub)
        out[:, ti[:, None], ci[None, :]] = sub
    else:
        np.add.at(out, (slice(None), ti[:, None], ci[None, :]), vals)
    return out[:, :n, :c].reshape(b, p.h, p.w, c)


def _mix(a: np.ndarray, t: np.ndarray) -> np.ndarray:
    """Token mix ``a @ tile`` for every tile: a [g,g], t [..., g, k]."""
    g = t.shape[-2]
    moved = np.moveaxis(t, -2, 0)
    out = a @ moved.reshape(g, -1)
    return np.moveaxis(out.reshape(moved.shape), 0, -2)


def _chan(t: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Per-channel-group product ``tile @ w[q]``: t [B,Qs,Qc,g,k], w [Qc,k,e]."""
    b, qs, qc, g, k = t.shape
    e = w.shape[2]
    out = np.empty((b, qs, qc, g, e), dtype=np.result_type(t, w))
    for q in range(qc):
        out[:, :, q] = (t[:, :, q].reshape(-1, k) @ w[q]).reshape(b, qs, g, e)
    return out


def _chan_wgrad(l: np.ndarray, r: np.ndarray) -> np.ndarray:
    """Sum over tiles of ``l_tile^T @ r_tile`` per channel group -> [Qc, kl, kr]."""
    qc = l.shape[2]
    return np.stack([
        l[:, :, q].reshape(-1, l.shape[-1]).T @ r[:, :, q].reshape(-1, r.shape[-1])
        for q in range(qc)
    ])


def _tok_wgrad(l: np.ndarray, r: np.ndarray) -> np.ndarray:
    """Sum over tiles of ``l_tile @ r_tile^T`` -> [g, g]."""
    g = l.shape[-2]
    lm = np.moveaxis(l, -2, 0).reshape(g, -1)
    rm = np.moveaxis(r, -2, 0).reshape(g, -1)
    return lm @ rm.T


def _sigmoid(u):
    return 1.0 / (1.0 + np.exp(-u))


def grouped_gamma(gamma: np.ndarray, p: Plan) -> np.ndarray:
    """reference.py:168-170: ``gamma[ch_idx.clamp_max(C-1)] * ch_mask``."""
    return gamma[np.minimum(p.ch, p.c - 1)] * p.cmask.astype(gamma.dtype)


def forward(x, p: Plan, a_u, a_v, a_o, b_u, b_v, b_o, gamma, keep: bool = False):
    """Delta of ``bigemm_delta_reference`` (reference.py:120-173).

    With ``keep=True`` also returns the intermediates the backward needs.
    """
    t = pack(x, p)
    pu = _mix(a_u, t)
    pv = _mix(a_v, t)
    u = _chan(pu, b_u)
    v = _chan(pv, b_v)
    su = u * _sigmoid(u)
    z = su * v
    y = _chan(z, b_o)
    du = _mix(a_o, y)
    mask = _mask(p).astype(x.dtype)
    gg = grouped_gamma(gamma, p)
    delta = du * mask[None] * gg[None, None, :, None, :]
    out = unpack(delta, p)
    if keep:
        return out, dict(t=t, pu=pu, pv=pv, u=u, v=v, z=z, y=y, du=du)
    return out


def backward(dout, x, p: Plan, a_u, a_v, a_o, b_u, b_v, b_o, gamma):
    """Gradients of ``sum(forward(...) * dout)`` w.r.t. all eight inputs."""
    _, s = forward(x, p, a_u, a_v, a_o, b_u, b_v, b_o, gamma, keep=True)
    graw = pack(dout, p)                          # mask applied
    gg = grouped_gamma(gamma, p)
    g_ = graw * gg[None, None, :, None, :]
    dgg = (graw * s["du"]).sum(axis=(0, 1, 3))    # [Qc, d]
    dgamma = np.zeros_like(gamma)
    np.add.at(dgamma, np.minimum(p.ch, p.c - 1)[p.cmask], dgg[p.cmask])
    dy = _mix(a_o.T, g_)
    da_o = _tok_wgrad(g_, s["y"])
    dz = _chan(dy, np.transpose(b_o, (0, 2, 1)))
    db_o = _chan_wgrad(s["z"], dy)
    sig = _sigmoid(s["u"])
    du_ = dz * s["v"] * sig * (1.0 + s["u"] * (1.0 - sig))
    dv_ = dz * s["u"] * sig
    dpu = _chan(du_, np.transpose(b_u, (0, 2, 1)))
    dpv = _chan(dv_, np.transpose(b_v, (0, 2, 1)))
    db_u = _chan_wgrad(s["pu"], du_)
    db_v = _chan_wgrad(s["pv"], dv_)
    da_u = _tok_wgrad(dpu, s["t"])
    da_v = _tok_wgrad(dpv, s["t"])
    dt = (_mix(a_u.T, dpu) + _mix(a_v.T, dpv)) * _mask(p).astype(x.dtype)[None]
    dx = unpack(dt, p)
    return dict(x=dx, a_u=da_u, a_v=da_v, a_o=da_o, b_u=db_u, b_v=db_v, b_o=db_o, gamma=dgamma)


def rms_stats(x):
    """Per-token reciprocal RMS, block.py:83-84.

    As in the reference, the mean of squares is taken in float32
    (``x.float().square().mean(-1)``) and then cast back to ``x``'s dtype
    before ``+ eps`` and the reciprocal square root.
    """
    x32 = x.astype(np.float32)
    var = np.mean(x32 * x32, axis=-1, keepdims=True, dtype=np.float32).astype(x.dtype)
    return 1.0 / np.sqrt(var + x.dtype.type(EPS))


def block_forward(x, p: Plan, norm_w, a_u, a_v, a_o, b_u, b_v, b_o, gamma, scale=None):
    """``OmniWeaveBlock.forward`` (block.py:80-108): x + s_b * delta(rmsnorm(x))."""
    r = rms_stats(x)
    xn = x * r * norm_w
    delta = forward(xn, p, a_u, a_v, a_o, b_u, b_v, b_o, gamma)
    if scale is not None:
        delta = delta * scale.reshape(-1, 1, 1, 1)
    return x + delta


def block_backward(dout, x, p: Plan, norm_w, a_u, a_v, a_o, b_u, b_v, b_o, gamma, scale=None):
    """Gradients of ``sum(block_forward(...) * dout)``."""
    r = rms_stats(x)
    xn = x * r * norm_w
    dd = dout if scale is None else dout * scale.reshape(-1, 1, 1, 1)
    gr = backward(dd, xn, p, a_u, a_v, a_o, b_u, b_v, b_o, gamma)
    dxn = gr["x"]
    c = x.shape[-1]
    dnorm_w = (dxn * x * r).reshape(-1, c).sum(axis=0)
    inner = np.sum(dxn * norm_w * x, axis=-1, keepdims=True)
    dx = dout + r * norm_w * dxn - x * (r ** 3) * inner / c
    out = dict(gr)
    out["x"] = dx
    out["norm_weight"] = dnorm_w
    return out

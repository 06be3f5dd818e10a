"""Float64 oracle of the max and smooth pooling operators — TEST INFRASTRUCTURE ONLY.

Restates the reference's operators on Mode-A tensors (Mode B through the equivalent Mode-A
expansion): pytorch_reference.py:29-48 (pre-activations) and :51-98 (``pool``):

* max: the maximum of act(z) over each group's valid slots, the winner being the smallest slot
  attaining it (kernels/triton_fused.py:129-140), with the backward of the winner-event kernel
  (triton_fused.py:476-520): per (token, group) one event dz = dy * act'(z_winner);
* logmeanexp: tau (logsumexp(a / tau) - log n); dz = dy softmax(a / tau) act'(z);
* softmax_weighted: sum softmax(beta a) a; dz = dy p (1 + beta (a - y)) act'(z);
* power_mean (a = relu(z)): max-scaled (mean a^p)^(1/p); dz = dy a^(p-1) y^(1-p) / n for z > 0,
  the derivatives the reference's dense backward uses (kernels/triton_fused.py:365-399);
* topk_mean: the k valid slots with the largest z (a stable descending sort: ties keep the
  smaller slot), pre = sum act(z) / min(k, n); dz = dy act'(z) / min(k, n) on those slots
  (pytorch_reference.py:66-77).

Pinned by tests/test_oracle_golden.py to fixtures made by the reference itself
(tests/golden/fwdbwd_max_*.npz, fwdbwd_smooth_*.npz, fwdbwd_topk_*.npz).  Materialises z [B, G, slots]: small cases
only.
"""
from __future__ import annotations

import numpy as np
from scipy.special import erf


def _act(z, act):
    if act == "relu":
        return np.maximum(z, 0.0)
    if act == "gelu":
        return 0.5 * z * (1.0 + erf(z / np.sqrt(2.0)))
    return z


def _dact(z, act):
    if act == "relu":
        return (z > 0).astype(np.float64)
    if act == "gelu":
        return 0.5 * (1.0 + erf(z / np.sqrt(2.0))) + z * np.exp(-0.5 * z * z) / np.sqrt(2.0 * np.pi)
    return np.ones_like(z)


def _z(x, idx, w, b):
    G = idx.shape[0]
    i = idx.reshape(G, -1, 8).astype(np.int64)            # [G, slots, 8]
    wv = w.reshape(G, -1, 8).astype(np.float64)
    bv = b.reshape(G, -1).astype(np.float64)
    xg = np.asarray(x, np.float64)[:, i]                   # [B, G, slots, 8]
    return (xg * wv[None]).sum(-1) + bv[None], xg, i, wv


def max_forward(x, idx, w, b, counts, act="relu"):
    """(y [B, G], winner [B, G]): max of act(z) over valid slots, smallest winning slot."""
    z, _, i, _ = _z(x, idx, w, b)
    valid = np.arange(i.shape[1])[None, :] < np.asarray(counts).reshape(-1, 1)
    a = np.where(valid[None], _act(z, act), -np.inf)
    win = np.argmax(a, axis=-1)
    return np.take_along_axis(a, win[..., None], -1)[..., 0], win


def max_backward(x, idx, w, b, counts, gy, act="relu", winner=None):
    """(dx, dw, db) float64 of the max operator for upstream gy [B, G] (dw, db in idx's layout)."""
    z, xg, i, wv = _z(x, idx, w, b)
    if winner is None:
        winner = max_forward(x, idx, w, b, counts, act)[1]
    B, G = winner.shape
    t = np.repeat(np.arange(B), G)
    g = np.tile(np.arange(G), B)
    s = winner.reshape(-1)
    dz = np.asarray(gy, np.float64).reshape(-1) * _dact(z[t, g, s], act)
    dx = np.zeros(np.asarray(x).shape)
    dw = np.zeros_like(wv)
    db = np.zeros(wv.shape[:2])
    np.add.at(db, (g, s), dz)
    np.add.at(dw, (g, s), dz[:, None] * xg[t, g, s])
    for k in range(8):
        np.add.at(dx, (t, i[g, s, k]), dz * wv[g, s, k])
    return dx, dw.reshape(np.asarray(w).shape), db.reshape(np.asarray(b).shape)


def _valid(i, counts):
    return np.arange(i.shape[1])[None, :] < np.asarray(counts).reshape(-1, 1)


def smooth_forward(x, idx, w, b, counts, kind, act, tau=1.0, beta=1.0, p=2.0):
    """y [B, G] (float64) of the logmeanexp / softmax_weighted / power_mean operators."""
    z, _, i, _ = _z(x, idx, w, b)
    valid = _valid(i, counts)[None]
    a = _act(z, act)
    n = np.asarray(counts, np.float64)[None, :]
    if kind == "power_mean":
        am = np.where(valid, a, 0.0)
        m = am.max(-1)
        safe = np.where(m > 0, m, 1.0)
        s = ((am / safe[..., None]) ** p).sum(-1) / n
        return np.where(m > 0, safe * s ** (1.0 / p), 0.0)
    u = np.where(valid, a / tau if kind == "logmeanexp" else beta * a, -np.inf)
    m = u.max(-1, keepdims=True)
    e = np.exp(u - m)
    lse = m[..., 0] + np.log(e.sum(-1))
    if kind == "logmeanexp":
        return tau * (lse - np.log(n))
    pw = e / e.sum(-1, keepdims=True)
    return (pw * np.where(valid, a, 0.0)).sum(-1)


def smooth_backward(x, idx, w, b, counts, gy, kind, act, tau=1.0, beta=1.0, p=2.0):
    """(dx, dw, db) float64 of the smooth operators for upstream gy = dL/dpre [B, G]."""
    z, xg, i, wv = _z(x, idx, w, b)
    valid = _valid(i, counts)[None]
    a = _act(z, act)
    gy = np.asarray(gy, np.float64)[..., None]
    if kind == "power_mean":
        y = smooth_forward(x, idx, w, b, counts, kind, act, p=p)[..., None]
        n = np.asarray(counts, np.float64)[None, :, None]
        ys = np.where(y > 0, y, 1.0)
        h = np.where((z > 0) & (y > 0), (np.maximum(a, 0.0) / ys) ** (p - 1.0) / n, 0.0)
        dz = np.where(valid, gy * h, 0.0)
    else:
        u = np.where(valid, a / tau if kind == "logmeanexp" else beta * a, -np.inf)
        e = np.exp(u - u.max(-1, keepdims=True))
        pw = e / e.sum(-1, keepdims=True)
        if kind == "logmeanexp":
            h = pw
        else:
            y = (pw * np.where(valid, a, 0.0)).sum(-1, keepdims=True)
            h = pw * (1.0 + beta * (a - y))
        dz = np.where(valid, gy * h * _dact(z, act), 0.0)
    db = dz.sum(0)                                                   # [G, slots]
    dw = (dz[..., None] * xg).sum(0)                                 # [G, slots, 8]
    B = dz.shape[0]
    dx = np.zeros(np.asarray(x).shape)
    contrib = dz[..., None] * wv[None]                               # [B, G, slots, 8]
    tt = np.broadcast_to(np.arange(B)[:, None, None, None], contrib.shape)
    np.add.at(dx, (tt.reshape(-1), np.broadcast_to(i[None], contrib.shape).reshape(-1)), contrib.reshape(-1))
    return dx, dw.reshape(np.asarray(w).shape), db.reshape(np.asarray(b).shape)


def topk_forward(x, idx, w, b, counts, k, act="identity"):
    """(y [B, G], slots [B, G, k] with -1 past min(k, n)) of the top-K mean operator."""
    z, _, i, _ = _z(x, idx, w, b)
    valid = _valid(i, counts)[None]
    zm = np.where(valid, z, -np.inf)
    order = np.argsort(-zm, axis=-1, kind="stable")[..., :k]
    n = np.asarray(counts).reshape(1, -1, 1)
    kk = np.minimum(n, k)
    sel = np.arange(order.shape[-1])[None, None, :] < kk
    a = np.take_along_axis(_act(z, act), order, -1)
    y = np.where(sel, a, 0.0).sum(-1) / kk[..., 0]
    return y, np.where(sel, order, -1)


def topk_backward(x, idx, w, b, counts, gy, k, act="identity", slots=None):
    """(dx, dw, db) float64 of the top-K mean operator for upstream gy [B, G]."""
    z, xg, i, wv = _z(x, idx, w, b)
    if slots is None:
        slots = topk_forward(x, idx, w, b, counts, k, act)[1]
    B, G, K = slots.shape
    t, g, j = np.nonzero(slots >= 0)
    s = slots[t, g, j]
    kk = np.minimum(np.asarray(counts), k).astype(np.float64)
    dz = np.asarray(gy, np.float64)[t, g] / kk[g] * _dact(z[t, g, s], act)
    dx = np.zeros(np.asarray(x).shape)
    dw = np.zeros_like(wv)
    db = np.zeros(wv.shape[:2])
    np.add.at(db, (g, s), dz)
    np.add.at(dw, (g, s), dz[:, None] * xg[t, g, s])
    for q in range(8):
        np.add.at(dx, (t, i[g, s, q]), dz * wv[g, s, q])
    return dx, dw.reshape(np.asarray(w).shape), db.reshape(np.asarray(b).shape)

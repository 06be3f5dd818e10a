"""Float64 oracle of max pooling — TEST INFRASTRUCTURE ONLY.

Restates the reference's max operator on Mode-A tensors (Mode B through the equivalent Mode-A
expansion): pytorch_reference.py:29-48 (pre-activations) and :51-75 (``pool``, "max": the
maximum of act(z) over each group's valid slots, the winner being the smallest slot attaining
it, kernels/triton_fused.py:129-140), with the backward of the winner-event kernel
(triton_fused.py:476-520): per (token, group) one event dz = dy * act'(z_winner) on the winning
neuron only.  Pinned by tests/test_oracle_golden.py to fixtures made by the reference itself
(tests/golden/fwdbwd_max_*.npz).  Materialises z [B, G, slots]: small cases only.
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

"""numpy wrapper of the C oracle ``libgl_oracle.so`` — TEST INFRASTRUCTURE ONLY.

Every function restates the reference's algorithm (file:line in gl_oracle.c and
below) in double precision on the CPU.  Parity is pinned by
``tests/test_oracle_golden.py`` against fixtures generated from the reference
itself (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libgl_oracle.so"
_lib = None

_i64, _int, _dbl = ctypes.c_int64, ctypes.c_int, ctypes.c_double
_p = ctypes.c_void_p


def build():
    """Compile libgl_oracle.so with the Makefile (gcc, OpenMP when available)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def load():
    global _lib
    if _lib is None:
        if not LIB.exists() or LIB.stat().st_mtime < (HERE / "gl_oracle.c").stat().st_mtime:
            build()
        lib = ctypes.CDLL(str(LIB))
        lib.glo_fwd.argtypes = [_p, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _int, _int, _p, _int]
        lib.glo_bwd.argtypes = [_p, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _int, _int, _p, _p, _p, _p, _int,
                                _p, _p, _p]
        lib.glo_adam.argtypes = [_p, _p, _p, _p, _i64, _dbl, _dbl, _dbl, _dbl, _dbl, _i64]
        for f in (lib.glo_fwd, lib.glo_bwd, lib.glo_adam):
            f.restype = _int
        _lib = lib
    return _lib


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _threads(n):
    return n if n else (os.cpu_count() or 1)


POOL = {"mean": 0, "sum": 1}
ACT = {"identity": 0, "relu": 1, "gelu": 2}


def forward(x, idx, w, b, counts, pool="mean", act="relu", nthreads=0):
    """pre [B, G] (float64) for Mode-A parameters idx [G, NB, 8, 8], w, b [G, NB, 8]."""
    lib = load()
    x = _c(x, np.float32)
    idx = _c(idx, np.int16)
    w = _c(w, np.float32)
    b = _c(b, np.float32)
    counts = _c(counts, np.int32)
    G, NB = idx.shape[0], idx.shape[1]
    B, D = x.shape
    pre = np.zeros((B, G), np.float64)
    rc = lib.glo_fwd(x.ctypes.data, B, D, D, idx.ctypes.data, w.ctypes.data, b.ctypes.data, counts.ctypes.data,
                     G, NB, POOL[pool], ACT[act], pre.ctypes.data, _threads(nthreads))
    if rc:
        raise RuntimeError(f"glo_fwd failed {rc}")
    return pre


def backward(x, idx, w, b, counts, gpre, pool="mean", act="relu", nthreads=0, slack=False):
    """(dx [B, D], dw like w, db like b), float64, for upstream dL/dpre ``gpre`` [B, G].

    With ``slack=True`` also returns (sdx, sdw, sdb): per element, the magnitude of
    the contributions of (token, neuron) pairs whose ReLU argument is within
    rounding of 0, where an fp32 kernel may legitimately take the other side of
    the derivative's jump (zero for identity/GELU)."""
    lib = load()
    x = _c(x, np.float32)
    idx = _c(idx, np.int16)
    w = _c(w, np.float32)
    b = _c(b, np.float32)
    counts = _c(counts, np.int32)
    gpre = _c(gpre, np.float64)
    G, NB = idx.shape[0], idx.shape[1]
    B, D = x.shape
    dx = np.zeros((B, D), np.float64)
    dw = np.zeros(w.shape, np.float64)
    db = np.zeros(b.shape, np.float64)
    sl = [np.zeros_like(a) for a in (dx, dw, db)] if slack else [None, None, None]
    ptr = [a.ctypes.data if a is not None else None for a in sl]
    nt = _threads(nthreads)
    if slack:  # the slack pass keeps a second private dx copy per thread
        nt = max(1, min(nt, int(2e9 // max(1, B * D * 16))))
    rc = lib.glo_bwd(x.ctypes.data, B, D, D, idx.ctypes.data, w.ctypes.data, b.ctypes.data, counts.ctypes.data,
                     G, NB, POOL[pool], ACT[act], gpre.ctypes.data, dx.ctypes.data, dw.ctypes.data, db.ctypes.data,
                     nt, *ptr)
    if rc:
        raise RuntimeError(f"glo_bwd failed {rc}")
    return (dx, dw, db, *sl) if slack else (dx, dw, db)


def adam_step(p, g, m, v, lr, beta1, beta2, eps, weight_decay, step):
    """One Adam(W) step (optim.py:39-42) in double; returns new (p, m, v)."""
    lib = load()
    p = _c(p, np.float64).copy()
    g = _c(g, np.float64)
    m = _c(m, np.float64).copy()
    v = _c(v, np.float64).copy()
    lib.glo_adam(p.ctypes.data, g.ctypes.data, m.ctypes.data, v.ctypes.data, p.size, lr, beta1, beta2, eps,
                 weight_decay, step)
    return p, m, v

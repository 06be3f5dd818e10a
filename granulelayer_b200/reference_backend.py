"""A backend for the reference's own ``Level1Runtime`` on the B200 library (maintainer-side binding).

This file is written to be copied unchanged into the reference as ``sparse_pooling/backends/b200.py``;
it imports nothing from this package, only ``ctypes`` and ``torch``.  The reference's runtime calls
a backend object at two sites (sparse_pooling/autograd.py:221 and :267):

    out = backend.forward(rt, x, w, b, track_ids)                     -> {"pre": [B, U] fp32}
    dx  = backend.backward(rt, x, w, b, g_pre, stats, dw_buf, db_buf) -> dx [B, D] fp32

with ``dw_buf`` / ``db_buf`` fp32 buffers that the backward accumulates into (the reference's
``main_grad`` semantics).  ``B200Backend`` serves single-level mean layers (the reference's pooling
operator of the hot path, any activation) with fp32 or bf16 parameters: Mode A through ``gl_fwd_f32`` /
``gl_bwd_f32``, Mode B (``shared_neurons=C``, canonical or fragment-packed) through
``gl_fwd_shared_f32`` / ``gl_bwd_shared_f32``; other layers raise ``NotImplementedError``, so a runtime
that routes only these layers here keeps its own kernels for the rest.

Loading follows the reference's ctypes bridge (backends/cuda/runtime.py:34-121): the library path comes
from ``GRANULE_B200_LIB`` (default: ``_lib/libgranule_b200.so`` beside this file), and the load refuses
a library whose ABI version, argument-struct sizes, field offsets or field names differ from the
declarations below (``gl_struct_layout`` / ``gl_struct_fields``).  Calls run on the current CUDA stream
of the tensors' device; a failed call raises ``RuntimeError`` with the library's status string.

Wiring (a maintainer's change to the reference): in ``SparsePoolingLayer._runtime``
(sparse_pooling/layer.py:106-131) pass ``B200Backend()`` as the runtime's ``backend`` for the layers it
serves, and make ``Level1Runtime.resolve`` report ``"cuda"`` for them (backends/dispatch.py:124-125
routes Mode A to Triton today).
"""
import ctypes
import os
from pathlib import Path

import torch

ABI_VERSION = 17
P, I64, I32, F32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float


class GlFwdArgs(ctypes.Structure):
    _fields_ = [("x", P), ("idx", P), ("w", P), ("b", P), ("counts", P), ("pre", P),
                ("B", I64), ("D", I64), ("NB", I64), ("g0", I64), ("g1", I64), ("ldx", I64), ("ldp", I64),
                ("pool", I32), ("act", I32), ("tokens", I32), ("groups_per_cta", I32), ("wabsmax", P),
                ("order", P), ("lidx", P), ("fmap", P), ("nfeat", P), ("fcap", I64), ("winners", P),
                ("ldwin", I64), ("stat", P), ("ldstat", I64), ("param", F32), ("k", I32), ("wdtype", I32),
                ("reserved3", I32)]


class GlBwdArgs(ctypes.Structure):
    _fields_ = [("x", P), ("idx", P), ("w", P), ("b", P), ("counts", P), ("gpre", P), ("dx", P), ("dw", P),
                ("db", P), ("B", I64), ("D", I64), ("NB", I64), ("g0", I64), ("g1", I64), ("ldx", I64),
                ("ldg", I64), ("lddx", I64), ("pool", I32), ("act", I32), ("tokens", I32),
                ("groups_per_cta", I32), ("wabsmax", P), ("rowmax", P), ("order", P), ("lidx", P),
                ("fmap", P), ("nfeat", P), ("fcap", I64), ("c2", P), ("c3", P), ("param", F32),
                ("wdtype", I32)]


class GlSharedArgs(ctypes.Structure):
    _fields_ = [(n, P) for n in ("x", "idx", "w", "b", "counts", "pre", "gpre", "dx", "dw", "db")] + \
               [(n, I64) for n in ("B", "D", "NB", "C", "g0", "g1", "ldx", "ldp", "ldg", "lddx")] + \
               [(n, I32) for n in ("pool", "act", "packed", "tokens", "groups_per_cta", "wdtype")] + \
               [("winners", P), ("ldwin", I64), ("stat", P), ("ldstat", I64), ("c2", P), ("c3", P),
                ("param", F32), ("k", I32)]


STRUCT_IDS = {GlFwdArgs: 0, GlBwdArgs: 1, GlSharedArgs: 3}     # ids of gl_struct_layout
POOL_MEAN = 0
ACT = {"identity": 0, "relu": 1, "gelu": 2}
DTYPE = {torch.float32: 0, torch.bfloat16: 1}


def load_library(path=None):
    """The B200 library, after checking its ABI version and the structs above against it."""
    p = Path(path or os.environ.get("GRANULE_B200_LIB") or Path(__file__).resolve().parent / "_lib" /
             "libgranule_b200.so")
    lib = ctypes.CDLL(str(p))
    lib.gl_abi_version.restype = ctypes.c_int
    if lib.gl_abi_version() != ABI_VERSION:
        raise RuntimeError(f"{p}: ABI version {lib.gl_abi_version()} != {ABI_VERSION}")
    lib.gl_struct_layout.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int64), ctypes.c_int]
    lib.gl_struct_layout.restype = ctypes.c_int
    lib.gl_struct_fields.argtypes = [ctypes.c_int]
    lib.gl_struct_fields.restype = ctypes.c_char_p
    for st, which in STRUCT_IDS.items():
        buf = (ctypes.c_int64 * 64)()
        n = lib.gl_struct_layout(which, buf, 64)
        want = [ctypes.sizeof(st)] + [getattr(st, f).offset for f, _ in st._fields_]
        names = (lib.gl_struct_fields(which) or b"").decode().rstrip(",").split(",")
        if n != len(want) or list(buf[:n]) != want or names != [f for f, _ in st._fields_]:
            raise RuntimeError(f"{p}: {st.__name__} differs from the library's (offsets {list(buf[:max(n, 0)])}, "
                               f"fields {names})")
    lib.gl_status_string.argtypes, lib.gl_status_string.restype = [ctypes.c_int], ctypes.c_char_p
    for name, st in (("gl_fwd_f32", GlFwdArgs), ("gl_bwd_f32", GlBwdArgs), ("gl_fwd_shared_f32", GlSharedArgs),
                     ("gl_bwd_shared_f32", GlSharedArgs)):
        getattr(lib, name).argtypes, getattr(lib, name).restype = [ctypes.POINTER(st), P], ctypes.c_int
    lib.gl_group_index_maxcount.argtypes = [P, P, I64, I64, I64, I64, P, P]
    lib.gl_group_index_maxcount.restype = ctypes.c_int
    return lib


class B200Backend:
    """``Level1Runtime`` backend on the B200 library for single-level mean layers (Mode A or B)."""

    def __init__(self, lib=None):
        self.lib = lib or load_library()
        self._rowmax = {}     # per index tensor: records per feature bound of the fixed-point backward

    def build_info(self):
        return {"library": "libgranule_b200", "abi": ABI_VERSION}

    def _check(self, rc, what):
        if rc:
            raise RuntimeError(f"{what}: {self.lib.gl_status_string(rc).decode()} [{rc}]")

    @staticmethod
    def _serves(rt, w):
        lv = rt.level
        if lv.type != "mean" or lv.activation not in ACT or w.dtype not in DTYPE:
            raise NotImplementedError(f"B200Backend serves mean layers with fp32/bf16 parameters, not "
                                      f"{lv.type}/{lv.activation}/{w.dtype}")

    def forward(self, rt, x, w, b, track_ids):
        """{"pre": [B, G] fp32}: the mean over each group's valid neurons of act(z)."""
        self._serves(rt, w)
        L, G = rt.layout, rt.layout.groups
        x = x.float().contiguous()
        B, D = x.shape
        pre = torch.empty(B, G, device=x.device, dtype=torch.float32)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        act = ACT[rt.level.activation]
        ptr = lambda t: t.data_ptr()  # noqa: E731
        with torch.cuda.device(x.device):
            if L.shared_indices:
                a = GlSharedArgs()
                a.x, a.idx, a.w, a.b, a.counts, a.pre = map(ptr, (x, rt.idx, w, b, rt.counts_i32, pre))
                a.B, a.D, a.NB, a.C, a.g0, a.g1, a.ldx, a.ldp = B, D, L.blocks_per_group, L.block, 0, G, D, G
                a.pool, a.act, a.packed, a.wdtype = POOL_MEAN, act, int(L.packed), DTYPE[w.dtype]
                self._check(self.lib.gl_fwd_shared_f32(ctypes.byref(a), stream), "gl_fwd_shared_f32")
            else:
                a = GlFwdArgs()
                a.x, a.idx, a.w, a.b, a.counts, a.pre = map(ptr, (x, rt.idx, w, b, rt.counts_i32, pre))
                a.B, a.D, a.NB, a.g0, a.g1, a.ldx, a.ldp = B, D, L.blocks_per_group, 0, G, D, G
                a.pool, a.act, a.wdtype = POOL_MEAN, act, DTYPE[w.dtype]
                self._check(self.lib.gl_fwd_f32(ctypes.byref(a), stream), "gl_fwd_f32")
        return {"pre": pre}

    def backward(self, rt, x, w, b, g_pre, stats, dw_buf, db_buf):
        """dx [B, D] fp32; dw_buf / db_buf (fp32, the parameters' layout) += the weight / bias gradients."""
        self._serves(rt, w)
        L, G = rt.layout, rt.layout.groups
        x = x.float().contiguous()
        g_pre = g_pre.float().contiguous()
        B, D = x.shape
        dx = torch.zeros(B, D, device=x.device, dtype=torch.float32)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        act = ACT[rt.level.activation]
        ptr = lambda t: t.data_ptr()  # noqa: E731
        with torch.cuda.device(x.device):
            if L.shared_indices:
                a = GlSharedArgs()
                a.x, a.idx, a.w, a.b, a.counts = map(ptr, (x, rt.idx, w, b, rt.counts_i32))
                a.gpre, a.dx, a.dw, a.db = map(ptr, (g_pre, dx, dw_buf, db_buf))
                a.B, a.D, a.NB, a.C, a.g0, a.g1 = B, D, L.blocks_per_group, L.block, 0, G
                a.ldx, a.ldg, a.lddx = D, G, D
                a.pool, a.act, a.packed, a.wdtype = POOL_MEAN, act, int(L.packed), DTYPE[w.dtype]
                self._check(self.lib.gl_bwd_shared_f32(ctypes.byref(a), stream), "gl_bwd_shared_f32")
                return dx
            key = (rt.idx.data_ptr(), rt.idx._version)
            rowmax = self._rowmax.get(key)
            if rowmax is None:      # once per layer: the largest number of a group's records on one feature
                rowmax = torch.empty(G, device=x.device, dtype=torch.int32)
                self._check(self.lib.gl_group_index_maxcount(ptr(rt.idx), ptr(rt.counts_i32), D, L.blocks_per_group,
                                                             0, G, ptr(rowmax), stream), "gl_group_index_maxcount")
                self._rowmax = {key: rowmax}
            # per-group bound max |w| (padding slots hold zeros, so the whole group's maximum is the same)
            wabsmax = w.detach().reshape(G, -1).abs().amax(1).float().contiguous()
            a = GlBwdArgs()
            a.x, a.idx, a.w, a.b, a.counts = map(ptr, (x, rt.idx, w, b, rt.counts_i32))
            a.gpre, a.dx, a.dw, a.db = map(ptr, (g_pre, dx, dw_buf, db_buf))
            a.B, a.D, a.NB, a.g0, a.g1, a.ldx, a.ldg, a.lddx = B, D, L.blocks_per_group, 0, G, D, G, D
            a.pool, a.act, a.wdtype = POOL_MEAN, act, DTYPE[w.dtype]
            a.wabsmax, a.rowmax = ptr(wabsmax), ptr(rowmax)
            self._check(self.lib.gl_bwd_f32(ctypes.byref(a), stream), "gl_bwd_f32")
        return dx

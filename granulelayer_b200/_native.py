"""ctypes binding of the C ABI in ``include/granule_b200.h``.

The library is loaded from ``granulelayer_b200/_lib/libgranule_b200.so`` (built
in-tree by ``granulelayer_b200.build``).  There is no fallback: if the library
is missing or its ABI version differs, every GPU entry point raises
``NativeLibraryError``.  Launch helpers take torch tensors only to read their
device pointers, strides and the current CUDA stream of their device; the
library itself sees plain pointers and sizes.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

ABI_VERSION = 17
LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libgranule_b200.so"

POOL_MEAN, POOL_SUM, POOL_MAX, POOL_LME, POOL_POWER, POOL_SOFTMAX, POOL_TOPK = 0, 1, 2, 3, 4, 5, 6
ACT_IDS = {"identity": 0, "relu": 1, "gelu": 2}
DTYPE_F32, DTYPE_BF16 = 0, 1


def _wdtype(t) -> int:
    """GL_DTYPE_* of a parameter tensor (fp32 or bf16 storage)."""
    if t.dtype == torch.float32:
        return DTYPE_F32
    if t.dtype == torch.bfloat16:
        return DTYPE_BF16
    raise ValueError(f"parameters must be float32 or bfloat16, not {t.dtype}")

# The exported entry points, in header order (checked by the CPU test suite).
EXPORTS = ("gl_abi_version", "gl_status_string", "gl_last_cuda_error", "gl_fwd_f32", "gl_bwd_f32",
           "gl_adam_f32", "gl_group_absmax_f32", "gl_group_index_maxcount", "gl_group_feature_map",
           "gl_group_order", "gl_launch_count",
           "gl_fwd_auto_tokens", "gl_bwd_auto_tokens", "gl_fwd_shared_f32", "gl_fwd_shared_tc", "gl_bwd_shared_tc", "gl_bwd_shared_tc_sets",
           "gl_fwd_shared_tc_sets", "gl_shared_tc_auto_tokens",
           "gl_bwd_shared_f32",
           "gl_bwd_events_f32",
           "gl_shared_auto_tokens", "gl_bwd_shared_det_f32", "gl_bwd_shared_det_static_f32", "gl_k16_fwd_f32",
           "gl_k16_bwd_f32", "gl_k16_auto_tokens", "gl_k16_fwd_tc", "gl_k16_bwd_tc", "gl_k16_fwd_tc_f32",
           "gl_k16_bwd_tc_f32", "gl_struct_layout", "gl_struct_fields", "gl_group_octets", "gl_fwd_octet_f32",
           "gl_bwd_octet_f32", "gl_k16_fwd_t5", "gl_k16_fwd_t5_f32", "gl_k16_bwd_t5", "gl_k16_bwd_t5_f32",
           "gl_bwd_octet_prefix_f32", "gl_group_feature_prefix")


class GlSetArgs(ctypes.Structure):
    _fields_ = [("feat", ctypes.c_void_p), ("buckets", ctypes.c_void_p), ("chunks", ctypes.c_void_p),
                ("rowmax", ctypes.c_void_p), ("wabsmax", ctypes.c_void_p), ("S", ctypes.c_int64),
                ("nchunks", ctypes.c_int64), ("max_chunk", ctypes.c_int64)]


class NativeLibraryError(RuntimeError):
    """The sm_100a library is missing, stale or failed a call."""


class GlFwdArgs(ctypes.Structure):
    _fields_ = [("x", ctypes.c_void_p), ("idx", ctypes.c_void_p), ("w", ctypes.c_void_p), ("b", ctypes.c_void_p),
                ("counts", ctypes.c_void_p), ("pre", ctypes.c_void_p),
                ("B", ctypes.c_int64), ("D", ctypes.c_int64), ("NB", ctypes.c_int64),
                ("g0", ctypes.c_int64), ("g1", ctypes.c_int64), ("ldx", ctypes.c_int64), ("ldp", ctypes.c_int64),
                ("pool", ctypes.c_int32), ("act", ctypes.c_int32), ("tokens", ctypes.c_int32),
                ("groups_per_cta", ctypes.c_int32), ("wabsmax", ctypes.c_void_p), ("order", ctypes.c_void_p),
                ("lidx", ctypes.c_void_p), ("fmap", ctypes.c_void_p), ("nfeat", ctypes.c_void_p),
                ("fcap", ctypes.c_int64), ("winners", ctypes.c_void_p), ("ldwin", ctypes.c_int64),
                ("stat", ctypes.c_void_p), ("ldstat", ctypes.c_int64), ("param", ctypes.c_float),
                ("k", ctypes.c_int32), ("wdtype", ctypes.c_int32), ("reserved3", ctypes.c_int32)]


class GlBwdArgs(ctypes.Structure):
    _fields_ = [("x", ctypes.c_void_p), ("idx", ctypes.c_void_p), ("w", ctypes.c_void_p), ("b", ctypes.c_void_p),
                ("counts", ctypes.c_void_p), ("gpre", ctypes.c_void_p), ("dx", ctypes.c_void_p),
                ("dw", ctypes.c_void_p), ("db", ctypes.c_void_p),
                ("B", ctypes.c_int64), ("D", ctypes.c_int64), ("NB", ctypes.c_int64),
                ("g0", ctypes.c_int64), ("g1", ctypes.c_int64),
                ("ldx", ctypes.c_int64), ("ldg", ctypes.c_int64), ("lddx", ctypes.c_int64),
                ("pool", ctypes.c_int32), ("act", ctypes.c_int32), ("tokens", ctypes.c_int32),
                ("groups_per_cta", ctypes.c_int32), ("wabsmax", ctypes.c_void_p), ("rowmax", ctypes.c_void_p),
                ("order", ctypes.c_void_p), ("lidx", ctypes.c_void_p), ("fmap", ctypes.c_void_p),
                ("nfeat", ctypes.c_void_p), ("fcap", ctypes.c_int64), ("c2", ctypes.c_void_p),
                ("c3", ctypes.c_void_p), ("param", ctypes.c_float), ("wdtype", ctypes.c_int32)]


class GlAdamArgs(ctypes.Structure):
    _fields_ = [("p", ctypes.c_void_p), ("g", ctypes.c_void_p), ("m", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("n", ctypes.c_int64),
                ("lr", ctypes.c_float), ("beta1", ctypes.c_float), ("beta2", ctypes.c_float),
                ("eps", ctypes.c_float), ("weight_decay", ctypes.c_float), ("bc1", ctypes.c_float),
                ("bc2", ctypes.c_float), ("zero_grad", ctypes.c_int32), ("master", ctypes.c_void_p),
                ("pdtype", ctypes.c_int32), ("mdtype", ctypes.c_int32), ("stochastic", ctypes.c_int32),
                ("seed", ctypes.c_uint32)]


class GlSharedArgs(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("x", "idx", "w", "b", "counts", "pre", "gpre", "dx", "dw", "db")] + \
               [(n, ctypes.c_int64) for n in ("B", "D", "NB", "C", "g0", "g1", "ldx", "ldp", "ldg", "lddx")] + \
               [(n, ctypes.c_int32) for n in ("pool", "act", "packed", "tokens", "groups_per_cta", "wdtype")] + \
               [("winners", ctypes.c_void_p), ("ldwin", ctypes.c_int64), ("stat", ctypes.c_void_p),
                ("ldstat", ctypes.c_int64), ("c2", ctypes.c_void_p), ("c3", ctypes.c_void_p),
                ("param", ctypes.c_float), ("k", ctypes.c_int32)]


class GlEventArgs(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("x", "idx", "w", "b", "winners", "coef", "dx", "dw", "db")] + \
               [(n, ctypes.c_int64) for n in ("B", "D", "NB", "C", "g0", "g1", "ldx", "ldwin", "ldc", "lddx")] + \
               [(n, ctypes.c_int32) for n in ("shared", "packed", "act", "kev", "wdtype", "reserved")]


class GlK16Args(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("x", "env", "feat", "buckets", "q_off", "rec_off", "w", "b", "counts",
                                                "pre", "c1t", "dx", "dw", "db")] + \
               [(n, ctypes.c_int64) for n in ("B", "D", "G", "NB16", "Q", "S", "nbuckets", "ldx", "ldp",
                                                 "ldc", "lddx")] + \
               [("act", ctypes.c_int32), ("tokens", ctypes.c_int32)]


# gl_struct_layout ids 0 .. GL_STRUCT_COUNT-1, in header order.
STRUCTS = (GlFwdArgs, GlBwdArgs, GlAdamArgs, GlSharedArgs, GlSetArgs, GlEventArgs, GlK16Args)


def check_struct_layouts(lib, path="library"):
    """Refuse a library whose argument structs differ from these ctypes declarations: sizeof, every
    field's offset (gl_struct_layout) and every field's name (gl_struct_fields), in declaration order.
    The reference's bridge makes the same check with sp_struct_layout (backends/cuda/runtime.py:103-121)."""
    lib.gl_struct_layout.restype = ctypes.c_int
    lib.gl_struct_layout.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int64), ctypes.c_int]
    lib.gl_struct_fields.restype = ctypes.c_char_p
    lib.gl_struct_fields.argtypes = [ctypes.c_int]
    for which, st in enumerate(STRUCTS):
        buf = (ctypes.c_int64 * 64)()
        n = lib.gl_struct_layout(which, buf, 64)
        want = [ctypes.sizeof(st)] + [getattr(st, name).offset for name, _ in st._fields_]
        names = (lib.gl_struct_fields(which) or b"").decode().rstrip(",").split(",")
        if n != len(want) or list(buf[:n]) != want or names != [name for name, _ in st._fields_]:
            raise NativeLibraryError(f"{path}: {st.__name__} layout mismatch (native sizeof/offsets "
                                     f"{list(buf[:max(n, 0)])}, fields {names}; ctypes {want})")


_lock = threading.Lock()
_lib = None


def library_path() -> Path:
    return Path(os.environ.get("GRANULE_B200_LIB", LIB_PATH))


def load(path=None) -> ctypes.CDLL:
    """Load (once) and version-check the library; raise if unavailable."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path else library_path()
        if not p.exists():
            raise NativeLibraryError(f"{p} not found: build it with `python -m granulelayer_b200.build`")
        lib = ctypes.CDLL(str(p))
        lib.gl_abi_version.restype = ctypes.c_int
        if lib.gl_abi_version() != ABI_VERSION:
            raise NativeLibraryError(f"{p}: ABI version {lib.gl_abi_version()} != {ABI_VERSION}; rebuild it")
        check_struct_layouts(lib, p)
        lib.gl_status_string.restype = ctypes.c_char_p
        lib.gl_status_string.argtypes = [ctypes.c_int]
        lib.gl_last_cuda_error.restype = ctypes.c_int
        lib.gl_launch_count.restype = ctypes.c_int64
        for name, st in (("gl_fwd_f32", GlFwdArgs), ("gl_bwd_f32", GlBwdArgs), ("gl_adam_f32", GlAdamArgs),
                         ("gl_fwd_octet_f32", GlFwdArgs), ("gl_bwd_octet_f32", GlBwdArgs),
                         ("gl_k16_fwd_f32", GlK16Args), ("gl_k16_bwd_f32", GlK16Args),
                         ("gl_k16_fwd_tc", GlK16Args), ("gl_k16_fwd_tc_f32", GlK16Args),
                         ("gl_fwd_shared_f32", GlSharedArgs), ("gl_bwd_shared_f32", GlSharedArgs),
                         ("gl_bwd_events_f32", GlEventArgs)):
            fn = getattr(lib, name)
            fn.restype = ctypes.c_int
            fn.argtypes = [ctypes.POINTER(st), ctypes.c_void_p]
        lib.gl_group_absmax_f32.restype = ctypes.c_int
        lib.gl_group_absmax_f32.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                            ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
        lib.gl_group_index_maxcount.restype = ctypes.c_int
        lib.gl_group_index_maxcount.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                                ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
        for name in ("gl_fwd_auto_tokens", "gl_bwd_auto_tokens"):
            getattr(lib, name).restype = ctypes.c_int
            getattr(lib, name).argtypes = [ctypes.c_int64]
        lib.gl_group_feature_map.restype = ctypes.c_int
        lib.gl_group_feature_map.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                             ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        lib.gl_bwd_octet_prefix_f32.restype = ctypes.c_int
        lib.gl_bwd_octet_prefix_f32.argtypes = [ctypes.POINTER(GlBwdArgs), ctypes.c_void_p, ctypes.c_void_p]
        lib.gl_group_feature_prefix.restype = ctypes.c_int
        lib.gl_group_feature_prefix.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                                ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
        lib.gl_group_octets.restype = ctypes.c_int
        lib.gl_group_octets.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                        ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_void_p]
        lib.gl_group_order.restype = ctypes.c_int
        lib.gl_group_order.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                       ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p,
                                       ctypes.c_void_p]
        lib.gl_shared_auto_tokens.restype = ctypes.c_int
        lib.gl_shared_auto_tokens.argtypes = [ctypes.c_int64, ctypes.c_int32]
        lib.gl_bwd_shared_det_f32.argtypes = [ctypes.POINTER(GlSharedArgs), ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_void_p, ctypes.c_void_p]
        lib.gl_bwd_shared_det_f32.restype = ctypes.c_int
        lib.gl_bwd_shared_det_static_f32.argtypes = [ctypes.POINTER(GlSharedArgs), ctypes.c_void_p, ctypes.c_void_p,
                                                     ctypes.c_void_p]
        lib.gl_bwd_shared_det_static_f32.restype = ctypes.c_int
        lib.gl_shared_tc_auto_tokens.restype = ctypes.c_int
        lib.gl_shared_tc_auto_tokens.argtypes = [ctypes.c_int64, ctypes.c_int32]
        lib.gl_fwd_shared_tc.argtypes = [ctypes.POINTER(GlSharedArgs), ctypes.c_void_p]
        lib.gl_fwd_shared_tc.restype = ctypes.c_int
        lib.gl_bwd_shared_tc.argtypes = [ctypes.POINTER(GlSharedArgs), ctypes.c_void_p, ctypes.c_void_p,
                                         ctypes.c_void_p]
        lib.gl_bwd_shared_tc.restype = ctypes.c_int
        for name in ("gl_k16_bwd_tc", "gl_k16_bwd_tc_f32"):
            getattr(lib, name).argtypes = [ctypes.POINTER(GlK16Args), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
            getattr(lib, name).restype = ctypes.c_int
        lib.gl_bwd_shared_tc_sets.argtypes = [ctypes.POINTER(GlSharedArgs), ctypes.POINTER(GlSetArgs), ctypes.c_void_p]
        lib.gl_bwd_shared_tc_sets.restype = ctypes.c_int
        lib.gl_fwd_shared_tc_sets.argtypes = [ctypes.POINTER(GlSharedArgs), ctypes.POINTER(GlSetArgs), ctypes.c_void_p]
        lib.gl_fwd_shared_tc_sets.restype = ctypes.c_int
        for name in ("gl_k16_fwd_t5", "gl_k16_fwd_t5_f32", "gl_k16_bwd_t5", "gl_k16_bwd_t5_f32"):
            getattr(lib, name).argtypes = [ctypes.POINTER(GlK16Args), ctypes.c_void_p, ctypes.c_void_p]
            getattr(lib, name).restype = ctypes.c_int
        lib.gl_k16_auto_tokens.restype = ctypes.c_int
        lib.gl_k16_auto_tokens.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32]
        if path is None:
            _lib = lib
        return lib


def launch_count() -> int:
    """Kernels the library has launched in this process (gl_launch_count)."""
    return int(load().gl_launch_count())


def _check(lib, rc: int, what: str):
    if rc != 0:
        msg = lib.gl_status_string(rc).decode()
        cu = lib.gl_last_cuda_error()
        extra = f" (cudaError {cu})" if cu else ""
        raise NativeLibraryError(f"{what} failed: {msg} [{rc}]{extra}")


def _ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise NativeLibraryError("the B200 kernels need CUDA tensors (no CPU fallback on this path)")


def fwd(x, idx, w, b, counts, pre, NB: int, g0: int, g1: int, pool: int, act: int, tokens: int = 0,
        groups_per_cta: int = 0, wabsmax=None, order=None, local=None, winners=None, stat=None,
        param: float = 0.0, k: int = 0):
    """pre[:, :g1-g0] = pooled act(z) of groups [g0, g1); optionally wabsmax[g-g0] = max |w|; ``order``
    is an optional processing order (group_order); ``local`` = (lidx, fmap, nfeat) from
    group_feature_map turns on the per-group input staging; ``winners`` [B, g1-g0] int32 receives
    the winning slots of max pooling; ``stat`` [B, g1-g0] the log2-normaliser of LME / softmax
    pooling, whose parameter (or power mean's p) is ``param``; top-K keeps ``k`` slots (``winners``
    then [B, (g1-g0) k]).  See GlFwdArgs."""
    lidx, fmap, nfeat = local if local is not None else (None, None, None)
    _require_cuda(x, idx, w, b, counts, pre, wabsmax, order, lidx, fmap, nfeat, winners, stat)
    lib = load()
    a = GlFwdArgs(_ptr(x), _ptr(idx), _ptr(w), _ptr(b), _ptr(counts), _ptr(pre), x.shape[0], x.shape[1], NB,
                  g0, g1, x.stride(0), pre.stride(0), pool, act, tokens, groups_per_cta, _ptr(wabsmax), _ptr(order),
                  _ptr(lidx), _ptr(fmap), _ptr(nfeat), fmap.shape[1] if fmap is not None else 0, _ptr(winners),
                  winners.stride(0) if winners is not None else 0, _ptr(stat),
                  stat.stride(0) if stat is not None else 0, float(param), int(k), _wdtype(w), 0)
    with torch.cuda.device(x.device):
        _check(lib, lib.gl_fwd_f32(ctypes.byref(a), _stream(x.device)), "gl_fwd_f32")


def bwd(x, idx, w, b, counts, gpre, dx, dw, db, NB: int, g0: int, g1: int, pool: int, act: int, tokens: int = 0,
        groups_per_cta: int = 0, wabsmax=None, rowmax=None, order=None, local=None, c2=None, c3=None,
        param: float = 0.0):
    """dx += ..., dw += ..., db += ... for groups [g0, g1); fixed-point dX tiles when the
    per-group bounds ``wabsmax``/``rowmax`` are given; optional processing ``order`` and input
    ``local``ity maps as in ``fwd``; the smooth pools take ``gpre`` = c1 and the coefficients
    ``c2``, ``c3`` (same strides as ``gpre``) and ``param``.  See GlBwdArgs."""
    lidx, fmap, nfeat = local if local is not None else (None, None, None)
    _require_cuda(x, idx, w, b, counts, gpre, dx, dw, db, wabsmax, rowmax, order, lidx, fmap, nfeat, c2, c3)
    for c in (c2, c3):
        if c is not None and c.stride(0) != gpre.stride(0):
            raise ValueError("c2/c3 must have gpre's row stride")
    lib = load()
    a = GlBwdArgs(_ptr(x), _ptr(idx), _ptr(w), _ptr(b), _ptr(counts), _ptr(gpre), _ptr(dx), _ptr(dw), _ptr(db),
                  x.shape[0], x.shape[1], NB, g0, g1, x.stride(0), gpre.stride(0), dx.stride(0), pool, act,
                  tokens, groups_per_cta, _ptr(wabsmax), _ptr(rowmax), _ptr(order), _ptr(lidx), _ptr(fmap),
                  _ptr(nfeat), fmap.shape[1] if fmap is not None else 0, _ptr(c2), _ptr(c3), float(param),
                  _wdtype(w))
    with torch.cuda.device(x.device):
        _check(lib, lib.gl_bwd_f32(ctypes.byref(a), _stream(x.device)), "gl_bwd_f32")


def _shared_args(x, idx, w, b, counts, NB, C, g0, g1, pool, act, packed, tokens, groups_per_cta):
    a = GlSharedArgs()
    a.x, a.idx, a.w, a.b, a.counts = _ptr(x), _ptr(idx), _ptr(w), _ptr(b), _ptr(counts)
    a.B, a.D, a.NB, a.C, a.g0, a.g1, a.ldx = x.shape[0], x.shape[1], NB, C, g0, g1, x.stride(0)
    a.pool, a.act, a.packed, a.tokens, a.groups_per_cta = pool, act, int(bool(packed)), tokens, groups_per_cta
    a.wdtype = _wdtype(w)
    return a


def fwd_shared(x, idx, w, b, counts, pre, NB: int, C: int, g0: int, g1: int, pool: int, act: int, packed: bool,
               tokens: int = 0, groups_per_cta: int = 0, winners=None, stat=None, param: float = 0.0, k: int = 0):
    """Mode B forward: pre[:, :g1-g0] = pooled act(z); ``winners``, ``stat`` and ``param`` as in
    ``fwd`` (GlSharedArgs)."""
    _require_cuda(x, idx, w, b, counts, pre, winners, stat)
    lib = load()
    a = _shared_args(x, idx, w, b, counts, NB, C, g0, g1, pool, act, packed, tokens, groups_per_cta)
    a.pre, a.ldp, a.param, a.k = _ptr(pre), pre.stride(0), float(param), int(k)
    if winners is not None:
        a.winners, a.ldwin = _ptr(winners), winners.stride(0)
    if stat is not None:
        a.stat, a.ldstat = _ptr(stat), stat.stride(0)
    with torch.cuda.device(x.device):
        _check(lib, lib.gl_fwd_shared_f32(ctypes.byref(a), _stream(x.device)), "gl_fwd_shared_f32")


def fwd_shared_tc(x, idx, w, b, counts, pre, NB: int, C: int, g0: int, g1: int, pool: int, act: int,
                  tokens: int = 0, groups_per_cta: int = 0, winners=None):
    """Mode B, bf16 fragment-packed parameters, on the tensor cores (gl_fwd_shared_tc): pre[:, :g1-g0] =
    mean / sum / max of act(z) with x rounded to bf16; ``winners`` as in ``fwd``."""
    _require_cuda(x, idx, w, b, counts, pre, winners)
    lib = load()
    a = _shared_args(x, idx, w, b, counts, NB, C, g0, g1, pool, act, True, tokens, groups_per_cta)
    a.pre, a.ldp = _ptr(pre), pre.stride(0)
    if winners is not None:
        a.winners, a.ldwin = _ptr(winners), winners.stride(0)
    with torch.cuda.device(x.device):
        _check(lib, lib.gl_fwd_shared_tc(ctypes.byref(a), _stream(x.device)), "gl_fwd_shared_tc")


def bwd_shared_tc(x, idx, w, b, counts, gpre, dx, dw, db, NB: int, C: int, g0: int, g1: int, pool: int, act: int,
                  tokens: int = 0, groups_per_cta: int = 0, wabsmax=None, rowmax=None):
    """Mode B, bf16 fragment-packed parameters, mean / sum backward on the tensor cores (gl_bwd_shared_tc):
    dx, dw, db += the gradients for dL/dpre ``gpre`` with x rounded to bf16 and dz in split precision.
    With ``wabsmax`` [g1-g0] fp32 and ``rowmax`` [g1-g0] int32 (both or neither) the dX tile is int32
    fixed point."""
    _require_cuda(x, idx, w, b, counts, gpre, dx, dw, db, wabsmax, rowmax)
    if (wabsmax is None) != (rowmax is None):
        raise ValueError("wabsmax and rowmax go together")
    lib = load()
    a = _shared_args(x, idx, w, b, counts, NB, C, g0, g1, pool, act, True, tokens, groups_per_cta)
    a.gpre, a.dx, a.dw, a.db = _ptr(gpre), _ptr(dx), _ptr(dw), _ptr(db)
    a.ldg, a.lddx = gpre.stride(0), dx.stride(0)
    with torch.cuda.device(x.device):
        _check(lib, lib.gl_bwd_shared_tc(ctypes.byref(a), _ptr(wabsmax), _ptr(rowmax), _stream(x.device)),
               "gl_bwd_shared_tc")


# Largest number of buckets in one chunk of gl_bwd_shared_tc_sets.
SET_MAX_CHUNK = 256


def fwd_shared_tc_sets(x, idx, w, b, counts, pre, NB: int, C: int, g0: int, g1: int, pool: int, act: int,
                       feat, buckets, chunks, max_chunk: int, tokens: int = 0):
    """Mode-B mean / sum forward of a bf16 fragment-packed layer with input-supergroup connectivity on the
    tensor cores over chunks of same-set buckets (gl_fwd_shared_tc_sets): pre[:, :g1-g0] is written."""
    _require_cuda(x, idx, w, b, counts, pre, feat, buckets, chunks)
    lib = load()
    a = _shared_args(x, idx, w, b, counts, NB, C, g0, g1, pool, act, True, tokens, 0)
    a.pre, a.ldp = _ptr(pre), pre.stride(0)
    sa = GlSetArgs(_ptr(feat), _ptr(buckets), _ptr(chunks), 0, 0, feat.shape[1], chunks.shape[0], int(max_chunk))
    with torch.cuda.device(x.device):
        _check(lib, lib.gl_fwd_shared_tc_sets(ctypes.byref(a), ctypes.byref(sa), _stream(x.device)),
               "gl_fwd_shared_tc_sets")


def bwd_shared_tc_sets(x, idx, w, b, counts, gpre, dx, dw, db, NB: int, C: int, g0: int, g1: int, pool: int, act: int,
                       feat, buckets, chunks, max_chunk: int, rowmax=None, wabsmax=None, tokens: int = 0):
    """Mode-B mean / sum backward of a bf16 fragment-packed layer with input-supergroup connectivity on the
    tensor cores, one CTA per token tile and chunk of same-set buckets (gl_bwd_shared_tc_sets): ``feat``
    [Q, S] int16, ``buckets`` [n, 4] int32, ``chunks`` [m, 3] int32 (set, first bucket, end bucket); with
    ``rowmax`` [n] int32 and ``wabsmax`` [G] fp32 the dX tile is int32 fixed point."""
    _require_cuda(x, idx, w, b, counts, gpre, dx, dw, db, feat, buckets, chunks, rowmax, wabsmax)
    if (rowmax is None) != (wabsmax is None):
        raise ValueError("rowmax and wabsmax go together")
    lib = load()
    a = _shared_args(x, idx, w, b, counts, NB, C, g0, g1, pool, act, True, tokens, 0)
    a.gpre, a.dx, a.dw, a.db = _ptr(gpre), _ptr(dx), _ptr(dw), _ptr(db)
    a.ldg, a.lddx = gpre.stride(0), dx.stride(0)
    sa = GlSetArgs(_ptr(feat), _ptr(buckets), _ptr(chunks), _ptr(rowmax), _ptr(wabsmax), feat.shape[1],
                   chunks.shape[0], int(max_chunk))
    with torch.cuda.device(x.device):
        _check(lib, lib.gl_bwd_shared_tc_sets(ctypes.byref(a), ctypes.byref(sa), _stream(x.device)),
               "gl_bwd_shared_tc_sets")


def shared_tc_tokens(D: int, backward: bool) -> int:
    """Token tile of the tensor-core kernels for input_dim D, or a negative status when D does not fit."""
    return load().gl_shared_tc_auto_tokens(D, int(backward))


def bwd_shared(x, idx, w, b, counts, gpre, dx, dw, db, NB: int, C: int, g0: int, g1: int, pool: int, act: int,
               packed: bool, tokens: int = 0, groups_per_cta: int = 0, c2=None, c3=None, param: float = 0.0):
    """Mode B backward: dx, dw, db += gradients for dL/dpre ``gpre`` (or, for the smooth pools, the
    coefficients ``gpre`` = c1, ``c2``, ``c3`` and ``param`` as in ``bwd``) (GlSharedArgs)."""
    _require_cuda(x, idx, w, b, counts, gpre, dx, dw, db, c2, c3)
    for c in (c2, c3):
        if c is not None and c.stride(0) != gpre.stride(0):
            raise ValueError("c2/c3 must have gpre's row stride")
    lib = load()
    a = _shared_args(x, idx, w, b, counts, NB, C, g0, g1, pool, act, packed, tokens, groups_per_cta)
    a.gpre, a.dx, a.dw, a.db = _ptr(gpre), _ptr(dx), _ptr(dw), _ptr(db)
    a.ldg, a.lddx = gpre.stride(0), dx.stride(0)
    a.c2, a.c3, a.param = _ptr(c2), _ptr(c3), float(param)
    with torch.cuda.device(x.device):
        _check(lib, lib.gl_bwd_shared_f32(ctypes.byref(a), _stream(x.device)), "gl_bwd_shared_f32")


def bwd_shared_det(x, idx, w, b, counts, gpre, dx, dw, db, NB: int, C: int, g0: int, g1: int, pool: int, act: int,
                   packed: bool, dxq, qscale, qinv):
    """Deterministic Mode-B backward (gl_bwd_shared_det_f32): dx, dw, db += the mean / sum gradients,
    bitwise repeatable; ``dxq`` a zeroed int64 [B, D] buffer, ``qscale`` / ``qinv`` [B] the per-token
    fixed-point scales 2^e and 2^-e."""
    _require_cuda(x, idx, w, b, counts, gpre, dx, dw, db, dxq, qscale, qinv)
    if dxq.dtype != torch.int64 or not dxq.is_contiguous() or tuple(dxq.shape) != tuple(x.shape):
        raise ValueError("dxq must be a contiguous int64 tensor shaped like x")
    lib = load()
    a = _shared_args(x, idx, w, b, counts, NB, C, g0, g1, pool, act, packed, 0, 0)
    a.gpre, a.dx, a.dw, a.db = _ptr(gpre), _ptr(dx), _ptr(dw), _ptr(db)
    a.ldg, a.lddx = gpre.stride(0), dx.stride(0)
    with torch.cuda.device(x.device):
        _check(lib, lib.gl_bwd_shared_det_f32(ctypes.byref(a), _ptr(dxq), _ptr(qscale), _ptr(qinv),
                                              _stream(x.device)), "gl_bwd_shared_det_f32")


# Largest B * D the allocation-free deterministic backward accepts (GL_DET_STATIC_MAX_ELEMS).
DET_STATIC_MAX_ELEMS = 1 << 20


def bwd_shared_det_static(x, idx, w, b, counts, gpre, dx, dw, db, NB: int, C: int, g0: int, g1: int, pool: int,
                          act: int, packed: bool, qscale, qinv):
    """Allocation-free deterministic Mode-B backward (gl_bwd_shared_det_static_f32): the results of
    ``bwd_shared_det`` without a caller scratch buffer, for B * D <= ``DET_STATIC_MAX_ELEMS``.  The
    library's fixed scratch is shared by every call on a device: calls must not overlap on the GPU."""
    _require_cuda(x, idx, w, b, counts, gpre, dx, dw, db, qscale, qinv)
    lib = load()
    a = _shared_args(x, idx, w, b, counts, NB, C, g0, g1, pool, act, packed, 0, 0)
    a.gpre, a.dx, a.dw, a.db = _ptr(gpre), _ptr(dx), _ptr(dw), _ptr(db)
    a.ldg, a.lddx = gpre.stride(0), dx.stride(0)
    with torch.cuda.device(x.device):
        _check(lib, lib.gl_bwd_shared_det_static_f32(ctypes.byref(a), _ptr(qscale), _ptr(qinv), _stream(x.device)),
               "gl_bwd_shared_det_static_f32")


def bwd_events(x, idx, w, b, winners, coef, dx, dw, db, NB: int, C: int, shared: bool, packed: bool, g0: int,
               g1: int, act: int, kev: int = 1):
    """Winner-event backward of max / top-K pooling (GlEventArgs): dx, dw, db += the gradients of the
    ``kev`` chosen slots per (token, group) in ``winners`` [B, (g1-g0) kev]."""
    _require_cuda(x, idx, w, b, winners, coef, dx, dw, db)
    lib = load()
    a = GlEventArgs(_ptr(x), _ptr(idx), _ptr(w), _ptr(b), _ptr(winners), _ptr(coef), _ptr(dx), _ptr(dw), _ptr(db),
                    x.shape[0], x.shape[1], NB, C, g0, g1, x.stride(0), winners.stride(0), coef.stride(0),
                    dx.stride(0), int(bool(shared)), int(bool(packed)), act, int(kev), _wdtype(w), 0)
    with torch.cuda.device(x.device):
        _check(lib, lib.gl_bwd_events_f32(ctypes.byref(a), _stream(x.device)), "gl_bwd_events_f32")


def group_absmax(w, counts, NB: int, g0: int, g1: int, out):
    """out[g-g0] = max |w| over the valid slots of group g (gl_group_absmax_f32)."""
    _require_cuda(w, counts, out)
    lib = load()
    with torch.cuda.device(w.device):
        _check(lib, lib.gl_group_absmax_f32(_ptr(w), _ptr(counts), NB, g0, g1, _ptr(out), _stream(w.device)),
               "gl_group_absmax_f32")


def group_index_maxcount(idx, counts, D: int, NB: int, g0: int, g1: int, out):
    """out[g-g0] = max records of group g sharing one feature (gl_group_index_maxcount)."""
    _require_cuda(idx, counts, out)
    lib = load()
    with torch.cuda.device(idx.device):
        _check(lib, lib.gl_group_index_maxcount(_ptr(idx), _ptr(counts), D, NB, g0, g1, _ptr(out),
                                                _stream(idx.device)), "gl_group_index_maxcount")


def group_feature_map(idx, counts, D: int, NB: int, g0: int, g1: int, nf, fmap=None, lidx=None):
    """nf[g-g0] = distinct features of group g; optionally the sorted lists ``fmap`` [g1-g0, cap] and
    the records as list positions ``lidx`` (gl_group_feature_map)."""
    _require_cuda(idx, counts, nf, fmap, lidx)
    lib = load()
    cap = fmap.shape[1] if fmap is not None else 0
    with torch.cuda.device(idx.device):
        _check(lib, lib.gl_group_feature_map(_ptr(idx), _ptr(counts), D, NB, g0, g1, cap, _ptr(nf), _ptr(fmap),
                                             _ptr(lidx), _stream(idx.device)), "gl_group_feature_map")


def fwd_octet(x, idx, w, b, counts, pre, NB: int, g0: int, g1: int, pool: int, act: int, groups_per_cta: int = 0,
              wabsmax=None):
    """Lane-per-neuron forward (gl_fwd_octet_f32): pre[:, :g1-g0] of the mean / sum pool; optionally
    wabsmax[g-g0] = max |w|.  For octet-arranged storage (group_octets); correct on any order."""
    _require_cuda(x, idx, w, b, counts, pre, wabsmax)
    lib = load()
    a = GlFwdArgs(_ptr(x), _ptr(idx), _ptr(w), _ptr(b), _ptr(counts), _ptr(pre), x.shape[0], x.shape[1], NB,
                  g0, g1, x.stride(0), pre.stride(0), pool, act, 0, groups_per_cta, _ptr(wabsmax), None, None, None,
                  None, 0, None, 0, None, 0, 0.0, 0, _wdtype(w), 0)
    with torch.cuda.device(x.device):
        _check(lib, lib.gl_fwd_octet_f32(ctypes.byref(a), _stream(x.device)), "gl_fwd_octet_f32")


def group_feature_prefix(idx, counts, D: int, NB: int, g0: int, g1: int, out):
    """out [(g1-g0+1) * D] int32: record inputs per feature, cumulated over the groups (gl_group_feature_prefix)."""
    _require_cuda(idx, counts, out)
    if out.dtype != torch.int32 or not out.is_contiguous() or out.numel() != (g1 - g0 + 1) * D:
        raise ValueError("out must be a contiguous int32 tensor of (g1-g0+1)*D elements")
    lib = load()
    with torch.cuda.device(idx.device):
        _check(lib, lib.gl_group_feature_prefix(_ptr(idx), _ptr(counts), D, NB, g0, g1, _ptr(out),
                                                _stream(idx.device)), "gl_group_feature_prefix")


def bwd_octet(x, idx, w, b, counts, gpre, dx, dw, db, NB: int, g0: int, g1: int, pool: int, act: int, wabsmax,
              rowmax, groups_per_cta: int = 0, feat_prefix=None):
    """Lane-per-neuron backward (gl_bwd_octet_f32): dx, dw, db += the mean / sum gradients, int32
    fixed-point dX tile from the per-group bounds ``wabsmax`` / ``rowmax``; with ``feat_prefix`` (from
    group_feature_prefix over g0 .. g1) gl_bwd_octet_prefix_f32, the same results with one instruction
    fewer per shared atomic."""
    _require_cuda(x, idx, w, b, counts, gpre, dx, dw, db, wabsmax, rowmax, feat_prefix)
    lib = load()
    a = GlBwdArgs(_ptr(x), _ptr(idx), _ptr(w), _ptr(b), _ptr(counts), _ptr(gpre), _ptr(dx), _ptr(dw), _ptr(db),
                  x.shape[0], x.shape[1], NB, g0, g1, x.stride(0), gpre.stride(0), dx.stride(0), pool, act, 0,
                  groups_per_cta, _ptr(wabsmax), _ptr(rowmax), None, None, None, None, 0, None, None, 0.0,
                  _wdtype(w))
    with torch.cuda.device(x.device):
        if feat_prefix is None:
            _check(lib, lib.gl_bwd_octet_f32(ctypes.byref(a), _stream(x.device)), "gl_bwd_octet_f32")
        else:
            _check(lib, lib.gl_bwd_octet_prefix_f32(ctypes.byref(a), _ptr(feat_prefix), _stream(x.device)),
                   "gl_bwd_octet_prefix_f32")


def group_octets(idx, counts, D: int, NB: int, g0: int, g1: int, order, kperm):
    """order, kperm [g1-g0, NB*8] int32: the octet arrangement of each group (gl_group_octets)."""
    _require_cuda(idx, counts, order, kperm)
    for t in (order, kperm):
        if t.dtype != torch.int32 or not t.is_contiguous() or tuple(t.shape) != (g1 - g0, NB * 8):
            raise ValueError("order and kperm must be contiguous int32 [g1-g0, NB*8]")
    lib = load()
    with torch.cuda.device(idx.device):
        _check(lib, lib.gl_group_octets(_ptr(idx), _ptr(counts), D, NB, g0, g1, _ptr(order), _ptr(kperm),
                                        _stream(idx.device)), "gl_group_octets")


def group_order(idx, counts, D: int, NB: int, g0: int, g1: int, unit: int, out):
    """out [g1-g0, NB*8] int32 = bank-aware processing order of each group (gl_group_order)."""
    _require_cuda(idx, counts, out)
    lib = load()
    with torch.cuda.device(idx.device):
        _check(lib, lib.gl_group_order(_ptr(idx), _ptr(counts), D, NB, g0, g1, unit, _ptr(out),
                                       _stream(idx.device)), "gl_group_order")


def adam(p, g, m, v, lr, beta1, beta2, eps, weight_decay, bc1, bc2, zero_grad=True, master=None,
         stochastic=False, seed=0):
    """One fused Adam(W) step (gl_adam_f32): fp32 gradient ``g`` (zeroed when ``zero_grad``), parameter
    ``p`` fp32 or bf16, moments ``m``/``v`` fp32 or bf16, optional fp32 ``master`` of a bf16 ``p``,
    stochastic rounding of a bf16 ``p`` without master from stream ``seed``."""
    _require_cuda(p, g, m, v, master)
    if g.dtype != torch.float32 or m.dtype != v.dtype or (master is not None and master.dtype != torch.float32):
        raise ValueError("adam: fp32 gradient and master, moments of one dtype")
    for t in (g, m, v) + ((master,) if master is not None else ()):
        if t.numel() != p.numel() or not t.is_contiguous():
            raise ValueError("adam: contiguous tensors of the parameter's size")
    lib = load()
    a = GlAdamArgs(_ptr(p), _ptr(g), _ptr(m), _ptr(v), p.numel(), lr, beta1, beta2, eps, weight_decay, bc1, bc2,
                   int(bool(zero_grad)), _ptr(master), _wdtype(p), _wdtype(m), int(bool(stochastic)),
                   int(seed) & 0xFFFFFFFF)
    with torch.cuda.device(p.device):
        _check(lib, lib.gl_adam_f32(ctypes.byref(a), _stream(p.device)), "gl_adam_f32")


def _k16_args(x, sched, w, b, counts, NB16: int, act: int, tokens: int):
    feat = sched["feat"]
    return GlK16Args(_ptr(x), _ptr(sched["env"]), _ptr(feat), _ptr(sched["buckets"]), _ptr(sched["q_off"]),
                     _ptr(sched["rec_off"]), _ptr(w), _ptr(b), _ptr(counts), 0, 0, 0, 0, 0,
                     x.shape[0], x.shape[1], counts.shape[0], NB16, feat.shape[0], feat.shape[1],
                     sched["buckets"].shape[0], x.stride(0), 0, 0, 0, act, tokens)


def _k16_entry(w, tensor_cores: bool, bwd: bool) -> str:
    """bf16 parameters: the tensor-core entry; fp32 ones: the tensor-core entry on three-term bf16 splits
    when ``tensor_cores``, else the SIMT one."""
    kind = "bwd" if bwd else "fwd"
    if w.dtype == torch.bfloat16:
        return f"gl_k16_{kind}_tc"
    return f"gl_k16_{kind}_tc_f32" if tensor_cores else f"gl_k16_{kind}_f32"


def k16_fwd(x, sched: dict, w, b, counts, pre, NB16: int, act: int = 1, tokens: int = 0,
            tensor_cores: bool = False) -> str:
    """pre[t, g] += Mean-pooled act(z) of the K16/C16 layer (GlK16Args); ``sched`` holds env, feat,
    buckets (sorted by set), q_off and rec_off.  bf16 parameters run the tensor-core entry
    (gl_k16_fwd_tc, x rounded to bf16); fp32 ones gl_k16_fwd_tc_f32 with ``tensor_cores``, else
    gl_k16_fwd_f32.  Returns the entry's name."""
    _require_cuda(x, w, b, counts, pre, *sched.values())
    lib = load()
    a = _k16_args(x, sched, w, b, counts, NB16, act, tokens)
    a.pre, a.ldp = _ptr(pre), pre.stride(0)
    name = _k16_entry(w, tensor_cores, False)
    with torch.cuda.device(x.device):
        _check(lib, getattr(lib, name)(ctypes.byref(a), _stream(x.device)), name)
    return name


def k16_bwd(x, sched: dict, w, b, counts, c1t, dx, dw, db, NB16: int, act: int = 1, tokens: int = 0,
            wabsmax=None, rowmax=None, tensor_cores: bool = False) -> str:
    """dx, dw, db += the K16/C16 layer's gradients for coefficients c1t [G, B] (GlK16Args).  The tensor-core
    entries (bf16 parameters; fp32 ones with ``tensor_cores``) take the optional fixed-point dX bounds
    wabsmax [G] / rowmax [nb]; the fp32 SIMT entry takes none.  Returns the entry's name."""
    _require_cuda(x, w, b, counts, c1t, dx, dw, db, *sched.values())
    lib = load()
    a = _k16_args(x, sched, w, b, counts, NB16, act, tokens)
    a.c1t, a.dx, a.dw, a.db = _ptr(c1t), _ptr(dx), _ptr(dw), _ptr(db)
    a.ldc, a.lddx = c1t.stride(0), dx.stride(0)
    name = _k16_entry(w, tensor_cores, True)
    with torch.cuda.device(x.device):
        if name == "gl_k16_bwd_f32":
            if wabsmax is not None or rowmax is not None:
                raise ValueError("gl_k16_bwd_f32 takes no fixed-point dX bounds")
            _check(lib, lib.gl_k16_bwd_f32(ctypes.byref(a), _stream(x.device)), name)
        else:
            if wabsmax is not None or rowmax is not None:
                _require_cuda(wabsmax, rowmax)
            _check(lib, getattr(lib, name)(ctypes.byref(a), _ptr(wabsmax), _ptr(rowmax), _stream(x.device)), name)
    return name


def k16_fwd_t5(x, sched: dict, w, b, counts, pre, NB16: int, act: int = 1, status=None) -> str:
    """pre[t, g] += Mean-pooled act(z) of the K16/C16 layer on the tcgen05 tensor cores (gl_k16_fwd_t5 for
    bf16 parameters, gl_k16_fwd_t5_f32 for fp32 ones, three-term splits); ``status`` (int32 [1], device,
    optional) receives 1 if a wait for the tensor cores ran out.  Returns the entry's name."""
    _require_cuda(x, w, b, counts, pre, status, *sched.values())
    lib = load()
    a = _k16_args(x, sched, w, b, counts, NB16, act, 0)
    a.pre, a.ldp = _ptr(pre), pre.stride(0)
    name = "gl_k16_fwd_t5" if w.dtype == torch.bfloat16 else "gl_k16_fwd_t5_f32"
    with torch.cuda.device(x.device):
        _check(lib, getattr(lib, name)(ctypes.byref(a), _ptr(status), _stream(x.device)), name)
    return name


def k16_bwd_t5(x, sched: dict, w, b, counts, c1t, dx, dw, db, NB16: int, act: int = 1, status=None) -> str:
    """dx, dw, db += the K16/C16 layer's gradients for coefficients c1t [G, B] on the tcgen05 tensor cores
    (gl_k16_bwd_t5 for bf16 parameters, gl_k16_bwd_t5_f32 for fp32 ones, three-term splits); dX is summed in
    fp32 in the tensor memory (no fixed-point bounds).  ``status`` as k16_fwd_t5.  Returns the entry's name."""
    _require_cuda(x, w, b, counts, c1t, dx, dw, db, status, *sched.values())
    lib = load()
    a = _k16_args(x, sched, w, b, counts, NB16, act, 0)
    a.c1t, a.dx, a.dw, a.db = _ptr(c1t), _ptr(dx), _ptr(dw), _ptr(db)
    a.ldc, a.lddx = c1t.stride(0), dx.stride(0)
    name = "gl_k16_bwd_t5" if w.dtype == torch.bfloat16 else "gl_k16_bwd_t5_f32"
    with torch.cuda.device(x.device):
        _check(lib, getattr(lib, name)(ctypes.byref(a), _ptr(status), _stream(x.device)), name)
    return name


def k16_auto_tokens(B: int, S: int, backward: bool) -> int:
    return int(load().gl_k16_auto_tokens(B, S, int(bool(backward))))

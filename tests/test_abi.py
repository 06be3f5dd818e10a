"""The C-ABI library loads on a CPU-only host, exports every entry point
include/granule_b200.h declares, and rejects bad arguments before touching a
device (no compute calls here)."""
import ctypes
import re

import pytest

from conftest import ROOT
from granulelayer_b200 import _native


def _declared():
    text = (ROOT / "include" / "granule_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|const char\*)\s+(gl_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    lib = _native.load()
    names = _declared()
    assert names, "no entry points parsed from the header"
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/granule_b200.h but not exported"
    assert set(names) == set(_native.EXPORTS)


def test_abi_version_and_status_strings():
    lib = _native.load()
    assert lib.gl_abi_version() == _native.ABI_VERSION
    assert lib.gl_status_string(0) == b"ok"
    for rc in range(-1, -8, -1):
        assert lib.gl_status_string(rc) != b"unknown status"


def test_argument_validation_needs_no_device():
    lib = _native.load()
    assert lib.gl_fwd_f32(None, None) == -1
    assert lib.gl_bwd_f32(None, None) == -1
    assert lib.gl_adam_f32(None, None) == -1
    a = _native.GlFwdArgs()
    a.B, a.D, a.NB, a.g0, a.g1 = 4, 0, 1, 0, 1           # D < 1
    assert lib.gl_fwd_f32(ctypes.byref(a), None) == -2
    a.D = 40000                                           # beyond int16 indices
    assert lib.gl_fwd_f32(ctypes.byref(a), None) == -2
    a.D, a.g0, a.g1 = 64, 3, 2                            # empty-reversed group range
    assert lib.gl_fwd_f32(ctypes.byref(a), None) == -2
    a.g0, a.g1, a.B = 0, 4, 0                             # empty batch: a no-op
    assert lib.gl_fwd_f32(ctypes.byref(a), None) == 0
    a.B = 4                                               # null pointers
    assert lib.gl_fwd_f32(ctypes.byref(a), None) == -1
    b = _native.GlBwdArgs()
    b.B, b.D, b.NB, b.g0, b.g1 = 4, 64, 1, 0, 0           # empty group range: a no-op
    assert lib.gl_bwd_f32(ctypes.byref(b), None) == 0
    ad = _native.GlAdamArgs()
    ad.n = -1
    assert lib.gl_adam_f32(ctypes.byref(ad), None) == -2
    ad.n = 0
    assert lib.gl_adam_f32(ctypes.byref(ad), None) == 0
    assert lib.gl_fwd_shared_f32(None, None) == -1
    sa = _native.GlSharedArgs()
    sa.B, sa.D, sa.NB, sa.C, sa.g0, sa.g1 = 4, 64, 4, 12, 0, 1   # C must be 8, 16, 32 or 64
    assert lib.gl_fwd_shared_f32(ctypes.byref(sa), None) == -2
    sa.C = 8
    assert lib.gl_bwd_shared_f32(ctypes.byref(sa), None) == -1  # null pointers
    sa.B = 0
    assert lib.gl_fwd_shared_f32(ctypes.byref(sa), None) == 0   # empty batch: a no-op
    assert lib.gl_k16_fwd_f32(None, None) == -1
    assert lib.gl_k16_bwd_f32(None, None) == -1
    k = _native.GlK16Args()
    k.B, k.D, k.G, k.NB16, k.Q, k.S = 4, 64, 2, 3, 1, 300   # S beyond uint8 local positions
    assert lib.gl_k16_fwd_f32(ctypes.byref(k), None) == -2
    k.S = 64
    assert lib.gl_k16_fwd_f32(ctypes.byref(k), None) == -1  # null pointers
    k.B = 0                                                  # empty batch: a no-op
    assert lib.gl_k16_bwd_f32(ctypes.byref(k), None) == 0
    assert lib.gl_k16_auto_tokens(0, 64, 0) == -2


def test_tensor_core_entry_points_validate_before_the_device():
    """The bf16 tensor-core entry points (Mode B generic and input-set, K16) reject bad arguments and
    run empty problems as no-ops without touching a device."""
    lib = _native.load()
    for fn in (lib.gl_fwd_shared_tc,):
        assert fn(None, None) == -1
    assert lib.gl_bwd_shared_tc(None, None, None, None) == -1
    sa = _native.GlSharedArgs()
    sa.B, sa.D, sa.NB, sa.C, sa.g0, sa.g1, sa.packed, sa.wdtype = 4, 64, 4, 8, 0, 1, 1, _native.DTYPE_BF16
    sa.pool, sa.act = _native.POOL_MEAN, _native.ACT_IDS["relu"]
    assert lib.gl_fwd_shared_tc(ctypes.byref(sa), None) == -1          # null pointers
    sa.packed = 0                                                       # canonical storage: not this path
    assert lib.gl_fwd_shared_tc(ctypes.byref(sa), None) == -4
    sa.packed, sa.wdtype = 1, _native.DTYPE_F32                         # fp32 storage: not this path
    assert lib.gl_fwd_shared_tc(ctypes.byref(sa), None) == -4
    sa.wdtype, sa.pool = _native.DTYPE_BF16, _native.POOL_MAX           # no max backward here
    assert lib.gl_bwd_shared_tc(ctypes.byref(sa), None, None, None) == -4
    sa.pool, sa.C = _native.POOL_MEAN, 12
    assert lib.gl_fwd_shared_tc(ctypes.byref(sa), None) == -2
    sa.C, sa.B = 8, 0                                                   # empty batch: a no-op
    assert lib.gl_fwd_shared_tc(ctypes.byref(sa), None) == 0
    assert lib.gl_bwd_shared_tc_sets(None, None, None) == -1
    assert lib.gl_fwd_shared_tc_sets(None, None, None) == -1
    st = _native.GlSetArgs()
    sa.B = 4
    assert lib.gl_bwd_shared_tc_sets(ctypes.byref(sa), ctypes.byref(st), None) == -1   # null pointers
    sa.pool = _native.POOL_MAX
    assert lib.gl_fwd_shared_tc_sets(ctypes.byref(sa), ctypes.byref(st), None) == -4   # mean / sum only
    assert lib.gl_k16_fwd_tc(None, None) == -1
    assert lib.gl_k16_bwd_tc(None, None, None, None) == -1
    k = _native.GlK16Args()
    k.B, k.D, k.G, k.NB16, k.Q, k.S, k.nbuckets, k.act = 4, 64, 2, 3, 1, 300, 1, _native.ACT_IDS["relu"]
    assert lib.gl_k16_fwd_tc(ctypes.byref(k), None) == -2                # S beyond uint8 local positions
    k.S = 64
    assert lib.gl_k16_fwd_tc(ctypes.byref(k), None) == -1                # null pointers
    k.act = _native.ACT_IDS["gelu"]
    assert lib.gl_k16_bwd_tc(ctypes.byref(k), None, None, None) == -4    # ReLU / identity only
    k.act, k.B = _native.ACT_IDS["relu"], 0                              # empty batch: a no-op
    assert lib.gl_k16_bwd_tc(ctypes.byref(k), None, None, None) == 0
    # the fp32 split entries validate the same way
    assert lib.gl_k16_fwd_tc_f32(None, None) == -1
    assert lib.gl_k16_bwd_tc_f32(None, None, None, None) == -1
    k.B, k.S = 4, 300
    assert lib.gl_k16_fwd_tc_f32(ctypes.byref(k), None) == -2
    k.S = 64
    assert lib.gl_k16_fwd_tc_f32(ctypes.byref(k), None) == -1
    k.act = _native.ACT_IDS["gelu"]
    assert lib.gl_k16_bwd_tc_f32(ctypes.byref(k), None, None, None) == -4
    k.act, k.B = _native.ACT_IDS["relu"], 0
    assert lib.gl_k16_bwd_tc_f32(ctypes.byref(k), None, None, None) == 0


def test_struct_layout_matches_header():
    # field order and sizes of the ctypes mirrors (pointers 8 B, int64 8 B, int32/float 4 B)
    assert ctypes.sizeof(_native.GlFwdArgs) == 6 * 8 + 7 * 8 + 4 * 4 + 2 * 8 + 4 * 8 + 2 * 8 + 2 * 8 + 4 * 4
    assert ctypes.sizeof(_native.GlBwdArgs) == 9 * 8 + 8 * 8 + 4 * 4 + 3 * 8 + 4 * 8 + 2 * 8 + 2 * 4
    assert ctypes.sizeof(_native.GlAdamArgs) == 4 * 8 + 8 + 8 * 4 + 8 + 4 * 4
    assert ctypes.sizeof(_native.GlK16Args) == 14 * 8 + 11 * 8 + 2 * 4
    assert ctypes.sizeof(_native.GlSharedArgs) == 10 * 8 + 10 * 8 + 6 * 4 + 2 * 8 + 4 * 8 + 2 * 4
    assert ctypes.sizeof(_native.GlEventArgs) == 9 * 8 + 10 * 8 + 6 * 4
    assert ctypes.sizeof(_native.GlSetArgs) == 5 * 8 + 3 * 8


def test_library_struct_layouts_match_ctypes_declarations():
    """gl_struct_layout / gl_struct_fields agree with every ctypes mirror: sizeof, offsets and names
    (the load-time check of the reference's bridge, backends/cuda/runtime.py:103-121)."""
    lib = _native.load()
    _native.check_struct_layouts(lib)          # raises on any difference
    buf = (ctypes.c_int64 * 64)()
    assert lib.gl_struct_layout(len(_native.STRUCTS), buf, 64) == -4      # unknown id
    assert lib.gl_struct_fields(len(_native.STRUCTS)) is None
    assert lib.gl_struct_layout(0, buf, 3) == -2                          # buffer too small
    header = (ROOT / "include" / "granule_b200.h").read_text()
    assert f"#define GL_STRUCT_COUNT {len(_native.STRUCTS)}" in header


def test_struct_layout_check_catches_a_drifted_binding():
    """A binding that dropped the trailing wdtype / reserved3 fields of GlFwdArgs (the drift the check
    exists for) is refused."""
    lib = _native.load()

    class Short(ctypes.Structure):
        _fields_ = [f for f in _native.GlFwdArgs._fields_ if f[0] not in ("wdtype", "reserved3")]

    saved = _native.STRUCTS
    try:
        _native.STRUCTS = (Short,) + saved[1:]
        with pytest.raises(_native.NativeLibraryError, match="layout mismatch"):
            _native.check_struct_layouts(lib)
    finally:
        _native.STRUCTS = saved


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(_native.NativeLibraryError):
        _native.load(tmp_path / "nope.so")


def test_reference_backend_module_is_the_integration_stub_and_loads():
    """INTEGRATION.md section 2 reproduces granulelayer_b200/reference_backend.py verbatim, and the module's
    own loader accepts this library (ABI version and struct layouts; no device needed)."""
    from granulelayer_b200 import reference_backend

    src = (ROOT / "granulelayer_b200" / "reference_backend.py").read_text()
    doc = (ROOT / "INTEGRATION.md").read_text()
    assert "```python\n" + src + "```" in doc
    assert "granulelayer_b200" not in src.split('"""', 2)[2]       # no imports from this package
    lib = reference_backend.load_library(_native.library_path())
    assert lib.gl_abi_version() == reference_backend.ABI_VERSION == _native.ABI_VERSION
    for st, which in reference_backend.STRUCT_IDS.items():
        assert [f for f, _ in st._fields_] == [f for f, _ in _native.STRUCTS[which]._fields_]

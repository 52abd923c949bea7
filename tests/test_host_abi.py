"""The C ABI library loads, exports every declared entry point, and its host
half (registry, sizes, host codecs, error paths) agrees with the oracle.
No GPU is needed: nothing here launches a kernel."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "autdot.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(aut_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(autlib):
    names = declared_functions()
    assert len(names) >= 20
    for name in names:
        assert hasattr(autlib, name), name


def test_python_binding_covers_the_header(autlib):
    from accessor_universal_test_b200 import _lib
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_registry_matches_the_reference_names(autlib, orc):
    from accessor_universal_test_b200 import DOT_FORMATS, _lib
    assert autlib.aut_abi_version() == 1
    for k, name in enumerate(DOT_FORMATS):
        assert _lib.format_id(name) == k
    count = autlib.aut_format_count()
    assert count == 106 + 2  # the reference's 106 named layouts + raw fp32/fp64
    names = [autlib.aut_format_name(k).decode() for k in range(count)]
    assert len(set(names)) == count
    assert autlib.aut_format_id(b"no_such_format") == -1
    import pyoracle
    r = pyoracle.reference()
    if r is not None:
        assert set(r.formats) <= set(names)
        for name, (_, desc) in r.formats.items():
            assert _lib.format_info(_lib.format_id(name)) == desc, name


def test_storage_bytes_follow_the_dense_word_count(autlib):
    from accessor_universal_test_b200 import _lib
    for name, bits in [("e2m3", 6), ("e8m0", 9), ("e8m15", 24), ("lns16_r11", 16)]:
        f = _lib.format_id(name)
        for n in [0, 1, 31, 32, 1000, (1 << 27) + 5]:
            assert _lib.storage_bytes(f, _lib.DENSE, n) == 4 * ((n * bits + 31) // 32 + 1)
    assert _lib.storage_bytes(_lib.format_id("e8m0"), _lib.PADDED, 10) == 20
    assert _lib.storage_bytes(_lib.format_id("e8m15"), _lib.PADDED, 10) == 40
    assert _lib.storage_bytes(_lib.format_id("e2m3"), _lib.PADDED, 10) == 10
    assert _lib.storage_bytes(_lib.format_id("fp32"), _lib.DENSE, 10) == 40
    assert _lib.storage_bytes(_lib.format_id("fp64"), _lib.DENSE, 10) == 80
    assert autlib.aut_packed_bytes(_lib.format_id("e2m3"), 4) == 3.0


def test_dot_support_matrix(autlib):
    from accessor_universal_test_b200 import DOT_FORMATS, _lib
    for name in DOT_FORMATS:
        f = _lib.format_id(name)
        for layout in (_lib.DENSE, _lib.PADDED):
            assert autlib.aut_dot_supported(f, layout, _lib.ACC_FP64) == 1, name
            want = 0 if name == "fp64" else 1
            assert autlib.aut_dot_supported(f, layout, _lib.ACC_FP32) == want, name
    # the generic DOT: FP32 where every value is an FP32 value (E <= 8,
    # M <= 23), FP64 for every bit format, LNS up to 16 bits
    expect = {("e3m4", 0): 1, ("e3m4", 1): 1, ("e9m22", 0): 0, ("e9m22", 1): 1,
              ("e0m31", 0): 0, ("e0m31", 1): 1, ("e0m23", 0): 1, ("e1m14", 0): 1,
              ("e11m4", 0): 0, ("e11m4", 1): 1, ("lns16_r4", 0): 1, ("lns16_r4", 1): 1,
              ("lns32_r20", 0): 0, ("lns32_r20", 1): 0}
    for (name, acc), want in expect.items():
        for layout in (_lib.DENSE, _lib.PADDED):
            got = autlib.aut_dot_supported(_lib.format_id(name), layout, acc)
            assert got == want, (name, acc, layout)
    assert autlib.aut_dot_supported(0, 7, 0) == 0


def _host_encode(fid, vals):
    from accessor_universal_test_b200 import _lib
    v = np.ascontiguousarray(vals, np.float64)
    out = np.empty(v.size, np.uint32)
    _lib.check(_lib.load().aut_encode_host(fid, v.ctypes.data, v.size, out.ctypes.data))
    return out


def _host_decode(fid, codes):
    from accessor_universal_test_b200 import _lib
    c = np.ascontiguousarray(codes, np.uint32)
    out = np.empty(c.size, np.float64)
    _lib.check(_lib.load().aut_decode_host(fid, c.ctypes.data, c.size, out.ctypes.data))
    return out


def test_host_codecs_match_oracle_on_every_format(autlib, orc):
    from accessor_universal_test_b200 import _lib
    rng = np.random.default_rng(11)
    for fid in range(autlib.aut_format_count()):
        desc = _lib.format_info(fid)
        if desc[0] == _lib.FAMILY_RAW_FP64:
            continue
        bits = desc[1]
        codes = (np.arange(1 << bits, dtype=np.uint32) if bits <= 16 else
                 rng.integers(0, 1 << bits, 50_000, dtype=np.uint64).astype(np.uint32))
        a = _host_decode(fid, codes)
        b = orc.decode_f64(desc, codes)
        assert np.array_equal(a.view(np.uint64), b.view(np.uint64)), desc
        vals = np.concatenate([b[np.isfinite(b)], rng.standard_normal(5000) * 4.0,
                               [0.0, -0.0, np.inf, -np.inf, np.nan, 1e-310]])
        assert np.array_equal(_host_encode(fid, vals), orc.encode(desc, vals)), desc


@pytest.mark.parametrize("name", ["e2m3", "e8m0", "e8m1", "e8m3", "e8m5", "bf16_e8m7",
                                  "e8m15", "lns8_r3", "lns16_r11", "e3m4"])
def test_host_pack_matches_oracle(autlib, orc, name):
    from accessor_universal_test_b200 import _lib
    fid = _lib.format_id(name)
    bits = _lib.format_info(fid)[1]
    for n in [1, 5, 129, 1000]:
        codes = np.random.default_rng(n).integers(0, 1 << bits, n, dtype=np.uint64).astype(np.uint32)
        out = np.zeros(_lib.storage_bytes(fid, _lib.DENSE, n), np.uint8)
        _lib.check(autlib.aut_pack_host(fid, _lib.DENSE, codes.ctypes.data, n, out.ctypes.data))
        assert np.array_equal(out.view(np.uint32), orc.pack_dense(bits, codes))
        back = np.empty(n, np.uint32)
        _lib.check(autlib.aut_unpack_host(fid, _lib.DENSE, out.ctypes.data, n, back.ctypes.data))
        assert np.array_equal(back, codes)
        pad = np.zeros(_lib.storage_bytes(fid, _lib.PADDED, n), np.uint8)
        _lib.check(autlib.aut_pack_host(fid, _lib.PADDED, codes.ctypes.data, n, pad.ctypes.data))
        _lib.check(autlib.aut_unpack_host(fid, _lib.PADDED, pad.ctypes.data, n, back.ctypes.data))
        assert np.array_equal(back, codes)


def test_errors_are_reported_not_raised(autlib):
    from accessor_universal_test_b200 import _lib
    assert autlib.aut_format_info(10_000, None, None, None, None) == _lib.AUT_ERR_INVALID_ARGUMENT
    assert b"unknown format" in autlib.aut_last_error()
    h = C.c_void_p()
    st = autlib.aut_workspace_create(0, C.byref(h))
    from conftest import HAS_GPU
    if not HAS_GPU:
        assert st == _lib.AUT_ERR_NO_DEVICE and not h.value
    else:
        assert st == _lib.AUT_OK
        autlib.aut_workspace_destroy(h)
    res = C.c_double()
    assert autlib.aut_dot(None, 3, 0, 0, None, None, 0, C.byref(res), None) == \
        _lib.AUT_ERR_INVALID_ARGUMENT


def test_collective_entry_points_check_their_arguments(autlib):
    """aut_comm_* / aut_dot_sharded refuse bad arguments before touching NCCL
    or a GPU."""
    from accessor_universal_test_b200 import _lib
    res = C.c_double()
    assert autlib.aut_dot_sharded(None, None, 3, 0, 0, None, None, 0, C.byref(res), None) == \
        _lib.AUT_ERR_INVALID_ARGUMENT
    assert b"communicator" in autlib.aut_last_error()
    h = C.c_void_p()
    ident = C.create_string_buffer(_lib.COMM_ID_BYTES)
    assert autlib.aut_comm_create(ident, 2, 2, 0, C.byref(h)) == _lib.AUT_ERR_INVALID_ARGUMENT
    assert autlib.aut_comm_create(None, 2, 0, 0, C.byref(h)) == _lib.AUT_ERR_INVALID_ARGUMENT
    assert autlib.aut_comm_unique_id(None) == _lib.AUT_ERR_INVALID_ARGUMENT
    assert autlib.aut_comm_allreduce(None, None, 1, None) == _lib.AUT_ERR_INVALID_ARGUMENT
    assert autlib.aut_comm_destroy(None) == _lib.AUT_OK

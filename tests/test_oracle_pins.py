"""Pin the oracle before trusting it.

The oracle (oracle/oracle.c) is checked against
  * the reference's own unit tests, compiled with asserts on (oracle/_ref),
  * the reference's own codecs / packer / dataset / compensated DOT, bit for
    bit (oracle/_ref/libautref.so), when the reference tree is present;
  * the committed golden fixtures in tests/golden/ (made by the reference's
    code, see tests/golden/make_golden.py), always.
"""
import csv
import json
import os
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN, ROOT

BINARY, PREFIX, LNS = 0, 1, 2


def _fmt(d):
    return (d["family"], d["total_bits"], d["exponent_bits"], d["finite"])


# ---- against the reference's own code (needs the reference tree) -------------

REF_TESTS = ["storage_formats_test", "decoder_strategy_core_test",
             "bitwidth_benchmark_core_test", "lns_benchmark_core_test",
             "memory_accessor_test"]


@pytest.mark.parametrize("name", REF_TESTS)
def test_reference_unit_tests_pass_with_asserts(ref, name):
    exe = os.path.join(ROOT, "oracle", "_ref", name)
    assert os.path.exists(exe)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr


def test_oracle_codecs_match_reference_all_formats(ref, orc):
    rng = np.random.default_rng(7)
    for name, (_, desc) in ref.formats.items():
        bits = desc[1]
        if bits <= 16:
            codes = np.arange(1 << bits, dtype=np.uint32)
        else:
            codes = rng.integers(0, 1 << bits, size=100_000, dtype=np.uint64).astype(np.uint32)
        a = ref.decode_f64(name, codes)
        b = orc.decode_f64(desc, codes)
        assert np.array_equal(a.view(np.uint64), b.view(np.uint64)), name
        a = ref.decode_f32(name, codes)
        b = orc.decode_f32(desc, codes)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), name
        finite = np.sort(ref.decode_f64(name, codes))
        finite = finite[np.isfinite(finite)]
        mids = (finite[:-1] + finite[1:]) / 2
        vals = np.concatenate([
            finite, mids, np.nextafter(mids, np.inf), np.nextafter(mids, -np.inf),
            rng.standard_normal(20_000) * rng.choice([1e-30, 1e-5, 1, 1e5, 1e30], 20_000),
            [0.0, -0.0, np.inf, -np.inf, np.nan, 5e-324, -5e-324, 1.7e308]])
        assert np.array_equal(ref.encode(name, vals), orc.encode(desc, vals)), name


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 7, 8, 9, 10, 12, 14, 16, 17, 24, 28, 32])
def test_oracle_dense_pack_matches_reference(ref, orc, bits):
    rng = np.random.default_rng(bits)
    codes = rng.integers(0, 1 << bits, size=1031, dtype=np.uint64).astype(np.uint32)
    assert np.array_equal(ref.pack_dense(bits, codes), orc.pack_dense(bits, codes))


def test_oracle_dot_v1_matches_reference(ref, orc):
    for case, cid in enumerate(ref.dot_v1_cases()):
        for vec in (0, 1):
            a = ref.dot_v1(case, vec, 4099)
            spec = _DOT_V1[cid]
            b = orc.dot_v1(spec[0], spec[1], spec[2], vec, 4099)
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), cid


def test_oracle_reference_dot_matches_reference(ref, orc):
    rng = np.random.default_rng(3)
    for name in ["e2m3", "e8m0", "e8m15", "lns8_r3", "lns16_r11"]:
        desc = ref.desc(name)
        bits = desc[1]
        codes_x = rng.integers(0, 1 << bits, 5000, dtype=np.uint64).astype(np.uint32)
        codes_y = rng.integers(0, 1 << bits, 5000, dtype=np.uint64).astype(np.uint32)
        xw, yw = ref.pack_dense(bits, codes_x), ref.pack_dense(bits, codes_y)
        with np.errstate(invalid="ignore"):
            r = ref.dot_dense(name, bits, xw, yw, 5000, threads=1)
            o = orc.dot_dense(desc, bits, xw, yw, 5000, threads=1)
        assert np.array_equal(np.array(r, dtype=np.float64).view(np.uint64),
                              np.array(o, dtype=np.float64).view(np.uint64)) or \
            (np.isnan(r[0][0]) and np.isnan(o[0][0])), name


# ---- against the committed golden fixtures (no reference needed) -----------------

# dot_v1 case id -> (family enum, seed, parameter), dot_dataset.hpp:106-134
_DOT_V1 = {
    "positive_uniform": (0, 0x123456789ABCDEF0, 0),
    "signed_uniform_seed0": (1, 0x123456789ABCDEF0, 0),
    "signed_uniform_seed1": (1, 0x8C3C010CB4754C9D, 0),
    "signed_uniform_seed2": (1, 0xD2B74407B1CE6E93, 0),
    "cancellation_1e2": (2, 0x123456789ABCDEF0, 6),
    "cancellation_1e4": (2, 0x123456789ABCDEF0, 13),
    "cancellation_1e6": (2, 0x123456789ABCDEF0, 19),
    "near_orthogonal": (2, 0x123456789ABCDEF0, 22),
    "dynamic_range_40": (3, 0xA4093822299F31D0, 20),
}


def _ld(hi, lo):
    return np.longdouble(hi) + np.longdouble(lo)


def test_oracle_dot_v1_fingerprints_and_reference_dots(orc):
    with open(os.path.join(GOLDEN, "dot_v1_inspect.csv")) as f:
        rows = list(csv.DictReader(f))
    assert len(rows) == 27
    for row in rows:
        kind, seed, param = _DOT_V1[row["dataset"]]
        n = int(row["n"])
        x = orc.dot_v1(kind, seed, param, 0, n)
        y = orc.dot_v1(kind, seed, param, 1, n)
        assert f"0x{orc.fnv1a(x):x}" == row["x_fingerprint"]
        assert f"0x{orc.fnv1a(y):x}" == row["y_fingerprint"]
        (dh, dl), (sh, sl) = orc.dot_reference(x, y)
        dot = _ld(dh, dl)
        want = np.longdouble(row["dot_reference"])
        # the CSV prints 21 significant digits of an 80-bit long double
        assert abs(dot - want) <= abs(want) * np.longdouble(1e-19) + np.longdouble(1e-30)
        assert abs(_ld(sh, sl) - np.longdouble(row["sum_abs"])) <= \
            np.longdouble(row["sum_abs"]) * np.longdouble(1e-19)


def test_published_signed_uniform_golden_value(orc):
    """datasets/dot_v1/validation_n1048576.csv: signed_uniform_seed0."""
    kind, seed, param = _DOT_V1["signed_uniform_seed0"]
    n = 1 << 20
    x = orc.dot_v1(kind, seed, param, 0, n)
    y = orc.dot_v1(kind, seed, param, 1, n)
    assert orc.fnv1a(x) == 0x6CA4178C4DF686DF
    assert orc.fnv1a(y) == 0x6A841D6C56C138D3
    (dh, dl), _ = orc.dot_reference(x, y)
    assert abs(_ld(dh, dl) - np.longdouble("-317.36476790556554306")) < 1e-16


def test_oracle_codecs_match_golden_vectors(orc):
    with open(os.path.join(GOLDEN, "codec_vectors.json")) as f:
        golden = json.load(f)
    for name, g in golden.items():
        desc = _fmt(g)
        codes = np.array(g["codes"], dtype=np.uint32)
        d64 = orc.decode_f64(desc, codes).view(np.uint64)
        assert [f"0x{b:016x}" for b in d64.tolist()] == g["decode_f64_bits"], name
        d32 = orc.decode_f32(desc, codes).view(np.uint32)
        assert [f"0x{b:08x}" for b in d32.tolist()] == g["decode_f32_bits"], name
        vals = np.array([int(b, 16) for b in g["encode_inputs_bits"]], dtype=np.uint64).view(np.float64)
        assert orc.encode(desc, vals).tolist() == g["encode_codes"], name


def _fnv_words(words):
    h = 1469598103934665603
    for w in words.astype(np.uint64).tolist():
        h ^= w
        h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return f"0x{h:016x}"


def test_oracle_synthetic_dots_match_golden(orc):
    with open(os.path.join(GOLDEN, "dot_vectors.json")) as f:
        golden = json.load(f)
    codec = json.load(open(os.path.join(GOLDEN, "codec_vectors.json")))
    seed = golden["seed"]
    for case in golden["cases"]:
        n, kind, name = case["n"], case["kind"], case["format"]
        if name in ("fp32", "fp64"):
            x = orc.synthetic(kind, seed, 0, n)
            y = orc.synthetic(kind, seed, 1, n)
            if name == "fp32":
                x, y = x.astype(np.float32), y.astype(np.float32)
            d, s = orc.dot_reference(x, y)
        else:
            desc = _fmt(codec[name])
            bits = desc[1]
            xw = orc.pack_dense(bits, orc.encode(desc, orc.synthetic(kind, seed, 0, n)))
            yw = orc.pack_dense(bits, orc.encode(desc, orc.synthetic(kind, seed, 1, n)))
            assert _fnv_words(xw) == case["x_words_fnv"], (name, n)
            assert _fnv_words(yw) == case["y_words_fnv"], (name, n)
            d, s = orc.dot_dense(desc, bits, xw, yw, n)
        assert (d[0], d[1]) == (case["dot_hi"], case["dot_lo"]), (name, n)
        assert (s[0], s[1]) == (case["sum_abs_hi"], case["sum_abs_lo"]), (name, n)


# ---- known answers of the reference's unit tests, restated -------------------------

def test_known_answers_storage_formats(orc):
    """tests/storage_formats_test.cpp:68-139 of the reference."""
    def rt(desc, v):
        return orc.decode_f64(desc, orc.encode(desc, [v]))[0]
    e1m6, e0m1, e0m3 = (BINARY, 8, 1, 1), (BINARY, 2, 0, 1), (BINARY, 4, 0, 1)
    fp4, e3m0, e2m5, e3m4 = (BINARY, 4, 2, 1), (BINARY, 4, 3, 0), (BINARY, 8, 2, 0), (BINARY, 8, 3, 0)
    e11m4, e11m20 = (PREFIX, 16, 11, 0), (PREFIX, 32, 11, 0)
    for desc, v in [(e1m6, 1.0), (e0m1, 0.5), (e0m3, 0.375), (fp4, 6.0), (e3m0, 1.0),
                    (e1m6, -1.0), (e2m5, 0.5), (e3m4, 0.25), (e11m4, 1.0), (e11m20, -0.0)]:
        got = rt(desc, v)
        assert got == v and np.signbit(got) == np.signbit(v)
    assert rt(e2m5, 1.0 + 2.0 ** -6) == 1.0
    assert rt(e2m5, 1.0 + 3.0 * 2.0 ** -6) == 1.0 + 2.0 ** -4
    assert rt(e11m4, 1.0 + 2.0 ** -5) == 1.0
    assert np.isinf(rt(e2m5, np.inf))
    sat = rt(e1m6, 100.0)
    assert np.isfinite(sat) and sat < 4.0


def test_known_answers_lns(orc):
    """tests/lns_benchmark_core_test.cpp:13-54,145-157 of the reference."""
    for bits, r in [(8, 3), (16, 11), (4, 0), (6, 2), (12, 6), (16, 4)]:
        desc = (LNS, bits, r, 0)
        codes = np.arange(1 << bits, dtype=np.uint32)
        v = orc.decode_f64(desc, codes)
        special = (codes & ((1 << (bits - 1)) - 1)) == (1 << (bits - 2))
        zeros = special & (codes < (1 << (bits - 1)))
        assert zeros.sum() == 1 and (v[zeros] == 0).all()
        assert np.isnan(v[special & ~zeros]).all() and (special & ~zeros).sum() == 1
        assert np.isfinite(v[~special]).all() and (v[~special] != 0).all()
        assert np.array_equal(orc.encode(desc, v[~special]), codes[~special])
        scale = float(1 << r)
        minimum = -(1 << (bits - 2)) + 1
        below = 2.0 ** ((minimum - 0.5001) / scale)
        above = 2.0 ** ((minimum - 0.4999) / scale)
        assert orc.encode(desc, [below])[0] == (1 << (bits - 2))
        assert orc.encode(desc, [above])[0] == (minimum & ((1 << (bits - 1)) - 1))
        inf_code = orc.encode(desc, [np.inf])[0]
        assert inf_code == (1 << (bits - 2)) - 1


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 7, 9, 14, 17, 28, 32])
def test_known_answers_dense_storage(orc, bits):
    """tests/bitwidth_benchmark_core_test.cpp:69-83 of the reference."""
    n = 257
    mask = (1 << bits) - 1
    codes = np.array([(i * 29 + 7) & mask for i in range(n)], dtype=np.uint32)
    words = orc.pack_dense(bits, codes)
    assert words.size == (n * bits + 31) // 32 + 1 and words[-1] == 0
    assert np.array_equal(orc.unpack_dense(bits, words, n), codes)

"""The fused DOT through the C ABI against the compensated long-double oracle."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN
from gpu_util import (DOT_FORMATS, SEED, STRATEGIES, TOL, device_pair, gpu_dot,
                      kind_of, normalized_error, oracle_codes, oracle_dot)

pytestmark = pytest.mark.gpu

SIZES = [1, 7, 100, 4099, 65536 + 13, (1 << 20) + 37]


def _accums(name):
    return [1] if name == "fp64" else [0, 1]


@pytest.mark.parametrize("name", DOT_FORMATS)
@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("strategy", STRATEGIES)
def test_dot_matches_oracle(ws, orc, name, layout, strategy):
    for n in SIZES:
        x, y = device_pair(ws, name, layout, n)
        ref_dot, ref_abs = oracle_dot(orc, name, n)
        for accum in _accums(name):
            got = gpu_dot(ws, name, layout, accum, x, y, n, strategy=strategy)
            err = normalized_error(got, ref_dot, ref_abs)
            assert err <= TOL[accum], (name, layout, accum, n, got, float(ref_dot), float(err))
            if name == "e2m3":
                # products k_a k_b / 64 and their partial sums are exact:
                # the DOT is the exact sum rounded once
                assert got == float(ref_dot), (name, n, got, float(ref_dot))


# (format, accumulator, decoder) triples with a kernel; every other explicit
# decoder is AUT_ERR_UNSUPPORTED.
DECODER_CASES = [("lns8_r3", 0, 2), ("lns8_r3", 1, 2), ("lns8_r3", 0, 5), ("lns8_r3", 1, 5),
                 ("lns16_r11", 0, 2),
                 ("lns16_r11", 0, 3), ("lns16_r11", 1, 3), ("lns16_r11", 0, 4),
                 ("lns16_r11", 1, 4), ("e8m5", 0, 1), ("e2m3", 1, 1), ("fp32", 0, 1),
                 ("e2m3", 0, 2), ("e2m3", 1, 2), ("e8m0", 0, 2), ("e8m0", 1, 2),
                 ("e8m1", 0, 2), ("e8m3", 1, 2), ("e8m5", 0, 2), ("e8m5", 1, 2),
                 ("e8m1", 0, 7), ("e8m1", 1, 7), ("e8m3", 0, 7), ("e8m5", 1, 7),
                 ("e8m1", 0, 8), ("e8m3", 1, 8), ("e8m5", 0, 8), ("e8m5", 1, 8)]


@pytest.mark.parametrize("name,accum,decoder", DECODER_CASES)
@pytest.mark.parametrize("strategy", STRATEGIES)
def test_every_decoder_matches_oracle(ws, orc, name, accum, decoder, strategy):
    for n in (3, 4099, (1 << 20) + 37):
        x, y = device_pair(ws, name, 0, n)
        ref_dot, ref_abs = oracle_dot(orc, name, n)
        got = gpu_dot(ws, name, 0, accum, x, y, n, strategy=strategy, decoder=decoder)
        err = normalized_error(got, ref_dot, ref_abs)
        assert err <= TOL[accum], (name, accum, decoder, n, got, float(ref_dot), float(err))


@pytest.mark.parametrize("name", ["e2m3", "e8m0", "e8m1", "e8m3", "e8m5"])
@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("strategy", [1, 2])
def test_full_table_decoder_equals_direct_decode(ws, orc, name, layout, strategy):
    """FULL_LUT (decode_with_table, one table word per code) against the
    oracle in both layouts; the e2m3 DOT is exact up to its final rounding
    with either decoder, so the two decoders agree bit for bit there."""
    for n in (5, 4099, (1 << 20) + 37):
        x, y = device_pair(ws, name, layout, n)
        ref_dot, ref_abs = oracle_dot(orc, name, n)
        for accum in (0, 1):
            got = gpu_dot(ws, name, layout, accum, x, y, n, strategy=strategy, decoder=2)
            err = normalized_error(got, ref_dot, ref_abs)
            assert err <= TOL[accum], (name, layout, accum, n, got, float(ref_dot), float(err))
            if name == "e2m3":
                assert got == float(ref_dot), (name, layout, accum, n, got, float(ref_dot))


def test_decoders_without_a_kernel_are_refused(ws):
    import torch
    from accessor_universal_test_b200 import _lib
    x = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    res = torch.zeros(1, dtype=torch.float64, device="cuda")
    refused = [("lns16_r11", 1, 2), ("lns16_r11", 0, 1), ("lns8_r3", 0, 3),
               ("lns8_r3", 0, 4), ("lns8_r3", 0, 1), ("e8m15", 0, 2), ("bf16_e8m7", 1, 2),
               ("fp32", 0, 2), ("e8m0", 0, 3), ("fp32", 0, 3),
               ("e8m15", 1, 4), ("lns16_r11", 0, 5), ("e8m0", 0, 5), ("fp64", 1, 5),
               ("e8m0", 0, 6), ("e2m3", 1, 6), ("fp32", 1, 6),
               ("e8m0", 0, 7), ("e8m15", 0, 7), ("lns8_r3", 0, 7), ("e8m0", 1, 8),
               ("bf16_e8m7", 0, 8), ("e2m3", 0, 8)]
    for name, accum, decoder in refused:
        with pytest.raises(_lib.AutError) as info:
            ws.dot(_lib.format_id(name), 0, accum, x.data_ptr(), x.data_ptr(), 64,
                   res.data_ptr(), decoder=decoder)
        assert info.value.status == _lib.AUT_ERR_UNSUPPORTED, (name, accum, decoder)
    with pytest.raises(_lib.AutError) as info:
        ws.dot(_lib.format_id("e8m0"), 0, 0, x.data_ptr(), x.data_ptr(), 64,
               res.data_ptr(), decoder=9)
    assert info.value.status == _lib.AUT_ERR_INVALID_ARGUMENT


def _fnv_words(words):
    h = 1469598103934665603
    for w in words.astype(np.uint64).tolist():
        h ^= w
        h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return f"0x{h:016x}"


def test_dot_matches_reference_golden_vectors(ws):
    """The reference's own CPU DOT of the same workloads (tests/golden)."""
    from accessor_universal_test_b200 import _lib
    golden = json.load(open(os.path.join(GOLDEN, "dot_vectors.json")))
    assert golden["seed"] == SEED
    for case in golden["cases"]:
        name, n = case["format"], case["n"]
        x, y = device_pair(ws, name, 0, n)
        if "x_words_fnv" in case:
            words = _lib.storage_bytes(_lib.format_id(name), 0, n) // 4
            xw = x[: 4 * words].cpu().numpy().view(np.uint32)
            yw = y[: 4 * words].cpu().numpy().view(np.uint32)
            assert _fnv_words(xw) == case["x_words_fnv"], (name, n)
            assert _fnv_words(yw) == case["y_words_fnv"], (name, n)
        ref_dot = np.longdouble(case["dot_hi"]) + np.longdouble(case["dot_lo"])
        ref_abs = np.longdouble(case["sum_abs_hi"]) + np.longdouble(case["sum_abs_lo"])
        for accum in _accums(name):
            got = gpu_dot(ws, name, 0, accum, x, y, n)
            assert normalized_error(got, ref_dot, ref_abs) <= TOL[accum], (name, n, accum)


def test_empty_dot_writes_zero(ws):
    import torch
    from accessor_universal_test_b200 import _lib
    res = torch.full((1,), 7.0, dtype=torch.float64, device="cuda")
    ws.dot(_lib.format_id("e8m0"), 0, 0, 0, 0, 0, res.data_ptr())
    torch.cuda.synchronize()
    assert res.item() == 0.0


@pytest.mark.parametrize("name", ["e2m3", "e8m0", "e8m15", "bf16_e8m7", "lns16_r11", "fp32"])
def test_unaligned_streams_take_the_scalar_path(ws, orc, name):
    import torch
    n = 50_003
    x, y = device_pair(ws, name, 0, n)
    ref_dot, ref_abs = oracle_dot(orc, name, n)
    xs = torch.zeros(x.numel() + 16, dtype=torch.uint8, device="cuda")
    ys = torch.zeros(y.numel() + 16, dtype=torch.uint8, device="cuda")
    xs[4:4 + x.numel()] = x
    ys[8:8 + y.numel()] = y
    for accum in (0, 1):
        got = gpu_dot(ws, name, 0, accum, xs, ys, n, x_off=4, y_off=8)
        assert normalized_error(got, ref_dot, ref_abs) <= TOL[accum]


@pytest.mark.parametrize("name", ["e8m0", "e8m5", "e8m15", "lns8_r3", "lns16_r11", "e2m3"])
@pytest.mark.parametrize("strategy", STRATEGIES)
def test_dot_is_deterministic_and_symmetric(ws, name, strategy):
    n = (1 << 22) + 5
    x, y = device_pair(ws, name, 0, n)
    for accum in (0, 1):
        a = gpu_dot(ws, name, 0, accum, x, y, n, strategy=strategy)
        b = gpu_dot(ws, name, 0, accum, x, y, n, strategy=strategy)
        c = gpu_dot(ws, name, 0, accum, y, x, n, strategy=strategy)
        assert a == b == c, (name, accum, a, b, c)


@pytest.mark.parametrize("name", ["e8m1", "bf16_e8m7", "e8m15", "lns8_r3", "lns16_r11"])
def test_special_codes_propagate_like_the_oracle(ws, orc, name):
    import torch
    from accessor_universal_test_b200 import _lib
    fid = _lib.format_id(name)
    desc = _lib.format_info(fid)
    n = 20_000
    _, _, cx = oracle_codes(orc, name, n, 0)
    _, _, cy = oracle_codes(orc, name, n, 1)
    cases = {"inf": orc.encode(desc, [np.inf])[0], "nan": orc.encode(desc, [np.nan])[0]}
    for label, code in cases.items():
        for pos in (0, 12_345, n - 1):
            xx = cx.copy()
            xx[pos] = code
            # The compensated reference turns +-inf into NaN (its correction
            # term computes inf - inf), so classify specials from the plain
            # sum of oracle-decoded products and use the compensated sum for
            # finite results only.
            with np.errstate(invalid="ignore", over="ignore"):
                prods = orc.decode_f64(desc, xx) * orc.decode_f64(desc, cy)
                plain = prods.sum()
                (d, s) = orc.dot_codes(desc, xx, cy, threads=1)
            want = plain if not np.isfinite(plain) else d[0]
            xb = np.zeros(_lib.storage_bytes(fid, 0, n), np.uint8)
            yb = np.zeros(_lib.storage_bytes(fid, 0, n), np.uint8)
            _lib.check(_lib.load().aut_pack_host(fid, 0, xx.ctypes.data, n, xb.ctypes.data))
            _lib.check(_lib.load().aut_pack_host(fid, 0, cy.ctypes.data, n, yb.ctypes.data))
            xt, yt = torch.from_numpy(xb).cuda(), torch.from_numpy(yb).cuda()
            for accum in (0, 1):
                got = gpu_dot(ws, name, 0, accum, xt, yt, n)
                if np.isnan(want):
                    assert np.isnan(got), (name, label, pos)
                elif np.isinf(want):
                    assert got == want, (name, label, pos, got, want)
                else:
                    assert abs(got - want) <= TOL[accum] * s[0], (name, label, pos, got, want)


LNS_DECODERS = [("lns8_r3", 0, 2), ("lns8_r3", 1, 2), ("lns8_r3", 0, 5), ("lns8_r3", 1, 5),
                ("lns16_r11", 0, 2),
                ("lns16_r11", 0, 3), ("lns16_r11", 1, 3), ("lns16_r11", 0, 4),
                ("lns16_r11", 1, 4)]


@pytest.mark.parametrize("name,accum,decoder", LNS_DECODERS)
@pytest.mark.parametrize("strategy", STRATEGIES)
def test_lns_reserved_codes_in_every_decoder(ws, orc, name, accum, decoder, strategy):
    """Zero and NaN codes (the reserved log code with either sign), sparse
    and dense, in one or both operands: zero products vanish and any NaN
    operand makes the DOT NaN (lns::multiply_codes)."""
    import torch
    from accessor_universal_test_b200 import _lib
    fid = _lib.format_id(name)
    desc = _lib.format_info(fid)
    n = 70_001
    _, _, cx = oracle_codes(orc, name, n, 0)
    _, _, cy = oracle_codes(orc, name, n, 1)
    zero = orc.encode(desc, [0.0])[0]
    nan = orc.encode(desc, [np.nan])[0]
    rng = np.random.default_rng(7)
    cases = {
        "sparse zeros in x": (rng.random(n) < 0.001, None, zero),
        "dense zeros in x and y": (rng.random(n) < 0.3, rng.random(n) < 0.3, zero),
        "one nan in y": (None, np.arange(n) == 40_000, nan),
    }
    for label, (mx, my, code) in cases.items():
        xx, yy = cx.copy(), cy.copy()
        if mx is not None:
            xx[mx] = code
        if my is not None:
            yy[my] = code
        with np.errstate(invalid="ignore"):
            plain = (orc.decode_f64(desc, xx) * orc.decode_f64(desc, yy)).sum()
        (d, s) = orc.dot_codes(desc, xx, yy, threads=4)
        bufs = []
        for codes in (xx, yy):
            b = np.zeros(_lib.storage_bytes(fid, 0, n), np.uint8)
            _lib.check(_lib.load().aut_pack_host(fid, 0, codes.ctypes.data, n, b.ctypes.data))
            bufs.append(torch.from_numpy(b).cuda())
        got = gpu_dot(ws, name, 0, accum, bufs[0], bufs[1], n, strategy=strategy,
                      decoder=decoder)
        if np.isnan(plain):
            assert np.isnan(got), label
        else:
            assert abs(got - d[0]) <= TOL[accum] * s[0], (label, got, d[0])


@pytest.mark.parametrize("name", ["e8m0", "e2m3", "lns16_r11", "fp32"])
def test_batched_dots_match_single_dots(ws, orc, name):
    import torch
    from accessor_universal_test_b200 import _lib
    fid = _lib.format_id(name)
    n, batch = 300_007, 5
    stride = (_lib.storage_bytes(fid, 0, n) + 255) // 256 * 256
    xb = torch.zeros(stride * batch, dtype=torch.uint8, device="cuda")
    yb = torch.zeros(stride * batch, dtype=torch.uint8, device="cuda")
    singles = []
    for b in range(batch):
        x, y = device_pair(ws, name, 0, n, seed=SEED + b)
        xb[b * stride: b * stride + x.numel()] = x[: min(x.numel(), stride)]
        yb[b * stride: b * stride + y.numel()] = y[: min(y.numel(), stride)]
        singles.append((gpu_dot(ws, name, 0, 1, x, y, n), x, y))
    res = torch.full((batch,), float("nan"), dtype=torch.float64, device="cuda")
    ws.dot_batched(fid, 0, 1, xb.data_ptr(), yb.data_ptr(), n, batch, stride, res.data_ptr())
    torch.cuda.synchronize()
    got = res.cpu().numpy()
    for b in range(batch):
        ref_dot, ref_abs = oracle_dot(orc, name, n, seed=SEED + b)
        assert normalized_error(got[b], ref_dot, ref_abs) <= TOL[1], (b, got[b], singles[b][0])
        assert abs(got[b] - singles[b][0]) <= 2 * TOL[1] * float(ref_abs)


@pytest.mark.parametrize("name", ["e8m1", "e8m3", "e8m5"])
@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("decoder", [7, 8])
def test_partial_table_decoders_in_both_layouts(ws, orc, name, layout, decoder):
    """prefix_lut / subnormal_lut: exact decodes, so the DOT is within the
    accumulator's bound in both layouts; inputs with subnormal and special
    codes run through tests/test_gpu_codec.py's decode checks."""
    for n in (5, 4099, (1 << 20) + 37):
        x, y = device_pair(ws, name, layout, n)
        ref_dot, ref_abs = oracle_dot(orc, name, n)
        for accum in (0, 1):
            for strategy in (1, 2):
                got = gpu_dot(ws, name, layout, accum, x, y, n, strategy=strategy,
                              decoder=decoder)
                err = normalized_error(got, ref_dot, ref_abs)
                assert err <= TOL[accum], (name, layout, decoder, accum, n, got, float(err))


COOP_FORMATS = ["e2m3", "e8m0", "e8m1", "e8m3", "e8m5", "bf16_e8m7", "e8m15"]


@pytest.mark.parametrize("name", COOP_FORMATS)
def test_cooperative_shuffle_loader_matches_oracle(ws, orc, name):
    """AUT_STRATEGY_COOPERATIVE (cooperative_shuffle): dense streams, whole
    chunks through the shuffles and the rest value by value, unaligned
    streams entirely value by value."""
    from accessor_universal_test_b200 import _lib
    for n in SIZES:
        x, y = device_pair(ws, name, 0, n)
        ref_dot, ref_abs = oracle_dot(orc, name, n)
        for accum in (0, 1):
            got = gpu_dot(ws, name, 0, accum, x, y, n, strategy=_lib.STRATEGY_COOPERATIVE)
            err = normalized_error(got, ref_dot, ref_abs)
            assert err <= TOL[accum], (name, accum, n, got, float(ref_dot), float(err))
            if name == "e2m3":
                assert got == float(ref_dot), (name, n, got)


def test_cooperative_loader_is_refused_where_it_does_not_apply(ws):
    import torch
    from accessor_universal_test_b200 import _lib
    x = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    res = torch.zeros(1, dtype=torch.float64, device="cuda")
    for name, layout, decoder in (("lns16_r11", 0, 0), ("fp32", 0, 0), ("e8m0", 1, 0),
                                  ("e8m0", 0, 2), ("lns8_r3", 0, 0)):
        with pytest.raises(_lib.AutError) as info:
            ws.dot(_lib.format_id(name), layout, 0, x.data_ptr(), x.data_ptr(), 64,
                   res.data_ptr(), strategy=_lib.STRATEGY_COOPERATIVE, decoder=decoder)
        assert info.value.status == _lib.AUT_ERR_UNSUPPORTED, (name, layout, decoder)

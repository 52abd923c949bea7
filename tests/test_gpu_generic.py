"""The generic DOT (every registered format without a fused kernel) against
the oracle: the runtime switch over the reference's format registries
(src/bitwidth_strategy_bench.cu:955-1211, lns_benchmark_core.hpp:44-61)."""
import numpy as np
import pytest

from gpu_util import SEED, TOL, normalized_error

pytestmark = pytest.mark.gpu

FUSED = {"fp32", "fp64", "e2m3", "e8m0", "e8m1", "e8m3", "e8m5", "bf16_e8m7", "e8m15",
         "lns8_r3", "lns16_r11"}


def _generic_formats():
    from accessor_universal_test_b200 import _lib
    lib = _lib.load()
    names = []
    for fid in range(lib.aut_format_count()):
        name = lib.aut_format_name(fid).decode()
        if name not in FUSED:
            names.append(name)
    return names


def _pair(ws, orc, name, layout, n, seed=SEED):
    import torch
    from accessor_universal_test_b200 import _lib
    fid = _lib.format_id(name)
    desc = _lib.format_info(fid)
    kind = 3 if desc[0] == _lib.FAMILY_LNS else 0
    codes = [orc.encode(desc, orc.synthetic(kind, seed, v, n)) for v in (0, 1)]
    bufs = []
    for c in codes:
        b = np.zeros(_lib.storage_bytes(fid, layout, n), np.uint8)
        _lib.check(_lib.load().aut_pack_host(fid, layout, c.ctypes.data, n, b.ctypes.data))
        bufs.append(torch.from_numpy(b).cuda())
    return fid, desc, codes, bufs


def test_every_registered_format_has_a_dot(autlib):
    from accessor_universal_test_b200 import _lib
    names = _generic_formats()
    assert len(names) == autlib.aut_format_count() - len(FUSED)
    for name in names:
        fid = _lib.format_id(name)
        fam, bits, _, _ = _lib.format_info(fid)
        want64 = 0 if (fam == _lib.FAMILY_LNS and bits > 16) else 1
        assert autlib.aut_dot_supported(fid, 0, 1) == want64, name


@pytest.mark.parametrize("layout", [0, 1])
# AUTO (table decode up to 8 bits, runtime-decoder TMA kernels above), SCALAR,
# and the runtime decoder forced on every bit format (DIRECT)
@pytest.mark.parametrize("strategy,decoder", [(0, 0), (3, 0), (0, 1)])
def test_generic_dot_matches_oracle_on_every_format(ws, orc, autlib, layout, strategy,
                                                    decoder):
    import torch
    from accessor_universal_test_b200 import _lib
    checked = 0
    for name in _generic_formats():
        fid = _lib.format_id(name)
        for n in (1, 4099, 65536 + 13):
            accs = [a for a in (0, 1) if autlib.aut_dot_supported(fid, layout, a)]
            if not accs or (decoder == 1 and _lib.format_info(fid)[0] == _lib.FAMILY_LNS):
                continue
            _, desc, codes, (x, y) = _pair(ws, orc, name, layout, n)
            (d, s) = orc.dot_codes(desc, codes[0], codes[1], threads=4)
            ref = np.longdouble(d[0]) + np.longdouble(d[1])
            sabs = np.longdouble(s[0]) + np.longdouble(s[1])
            for acc in accs:
                res = torch.full((1,), float("nan"), dtype=torch.float64, device="cuda")
                ws.dot(fid, layout, acc, x.data_ptr(), y.data_ptr(), n, res.data_ptr(),
                       strategy=strategy, decoder=decoder)
                torch.cuda.synchronize()
                got = res.item()
                if not np.isfinite(float(ref)):
                    assert np.isnan(got) or got == float(ref), (name, n, acc, got)
                    continue
                err = normalized_error(got, ref, sabs)
                assert err <= TOL[acc], (name, layout, n, acc, got, float(ref), float(err))
                checked += 1
    assert checked > 300


@pytest.mark.parametrize("name", ["e3m4", "e5m11", "e11m20", "lns16_r4", "lns6_r2", "e0m31"])
def test_generic_gemv_and_batched(ws, orc, name):
    """Rows of a generic-format matrix, 16-byte aligned or not, and batches."""
    import torch
    from accessor_universal_test_b200 import _lib
    fid = _lib.format_id(name)
    desc = _lib.format_info(fid)
    for rows, cols in ((40, 2048), (33, 999)):
        _, _, mcodes, (m, _) = _pair(ws, orc, name, 0, rows * cols)
        _, _, vcodes, (v, _) = _pair(ws, orc, name, 0, cols, seed=SEED + 1)
        out = torch.full((rows,), float("nan"), dtype=torch.float64, device="cuda")
        ws.gemv(fid, 0, 1, m.data_ptr(), v.data_ptr(), rows, cols, out.data_ptr())
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        for r in range(rows):
            d, s = orc.dot_codes(desc, mcodes[0][r * cols:(r + 1) * cols], vcodes[0], threads=1)
            ref = np.longdouble(d[0]) + np.longdouble(d[1])
            sabs = np.longdouble(s[0]) + np.longdouble(s[1])
            assert normalized_error(got[r], ref, sabs) <= TOL[1], (name, rows, cols, r)


EXHAUSTIVE = ["e1m0", "e2m0", "e3m0", "e7m0", "fp4_e2m1", "e0m7", "e2m5", "e3m4", "e5m3",
              "e1m14", "e5m11", "e8m8", "e9m6", "e10m5", "e11m4", "e4m23", "e9m22", "e0m31"]


@pytest.mark.parametrize("name", EXHAUSTIVE)
@pytest.mark.parametrize("layout", [0, 1])
def test_runtime_decoder_on_every_code(ws, orc, autlib, name, layout):
    """Every code (2^16 random codes above 16 bits) times the code nearest
    1.0, as a one-column GEMV (row r = code r times the vector's one code):
    zeros, subnormals, the largest values, inf and NaN of every exponent
    width against the oracle's decode, bit for bit, through the table decoder
    (codes of up to 8 bits) and the runtime-shift decoder."""
    import torch
    from accessor_universal_test_b200 import _lib
    fid = _lib.format_id(name)
    desc = _lib.format_info(fid)
    bits = desc[1]
    if bits <= 16:
        codes = np.arange(1 << bits, dtype=np.uint32)
    else:
        codes = np.random.default_rng(9).integers(0, 1 << bits, 1 << 16,
                                                  dtype=np.uint64).astype(np.uint32)
    one = np.array(orc.encode(desc, [1.0]), np.uint32)
    mat = np.zeros(_lib.storage_bytes(fid, layout, codes.size), np.uint8)
    vec = np.zeros(_lib.storage_bytes(fid, layout, 1), np.uint8)
    _lib.check(_lib.load().aut_pack_host(fid, layout, codes.ctypes.data, codes.size,
                                         mat.ctypes.data))
    _lib.check(_lib.load().aut_pack_host(fid, layout, one.ctypes.data, 1, vec.ctypes.data))
    mt, vt = torch.from_numpy(mat).cuda(), torch.from_numpy(vec).cuda()
    decoders = [0, 1] if bits <= 8 else [0]
    for acc in (0, 1):
        if not autlib.aut_dot_supported(fid, layout, acc):
            continue
        dec = orc.decode_f32 if acc == 0 else orc.decode_f64
        # the one-value DOT is the product of the two decoded values, formed
        # in FP64 (exact for FP32 values; one rounding for the widest codes);
        # formats without 1.0 (e1m0 rounds it to inf) still check every code
        with np.errstate(invalid="ignore", over="ignore"):
            want = dec(desc, codes).astype(np.float64) * np.float64(dec(desc, one)[0])
        nan = np.isnan(want)
        for decoder in decoders:
            out = torch.full((codes.size,), 7.0, dtype=torch.float64, device="cuda")
            ws.gemv(fid, layout, acc, mt.data_ptr(), vt.data_ptr(), codes.size, 1,
                    out.data_ptr(), decoder=decoder)
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            assert np.array_equal(np.isnan(got), nan), (name, acc, decoder)
            ok = got[~nan] == want[~nan]  # +-0 compare equal: the sum starts at +0
            assert ok.all(), (name, acc, decoder, codes[~nan][~ok][:5], got[~nan][~ok][:5],
                              want[~nan][~ok][:5])

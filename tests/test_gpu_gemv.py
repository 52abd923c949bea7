"""aut_gemv (matrix-vector product over compact storage) against the oracle:
every row is checked as a compensated long-double DOT of the same codes."""
import numpy as np
import pytest

from gpu_util import DOT_FORMATS, SEED, STRATEGIES, TOL, kind_of, normalized_error

pytestmark = pytest.mark.gpu


def _accums(name):
    return [1] if name == "fp64" else [0, 1]


def _operands(ws, orc, name, layout, rows, columns):
    """Device matrix (rows * columns values, vector id 0) and vector (columns
    values, vector id 1), plus the oracle's per-row reference function."""
    from accessor_universal_test_b200 import _lib, vectors
    kind = kind_of(name)
    m = vectors.encoded(ws, name, layout, kind, SEED, 0, rows * columns)
    v = vectors.encoded(ws, name, layout, kind, SEED, 1, columns)
    if name in ("fp32", "fp64"):
        mv = orc.synthetic(kind, SEED, 0, rows * columns)
        vv = orc.synthetic(kind, SEED, 1, columns)
        if name == "fp32":
            mv, vv = mv.astype(np.float32), vv.astype(np.float32)

        def ref(r):
            d, s = orc.dot_reference(mv[r * columns:(r + 1) * columns], vv)
            return d, s
    else:
        desc = _lib.format_info(_lib.format_id(name))
        mc = orc.encode(desc, orc.synthetic(kind, SEED, 0, rows * columns))
        vc = orc.encode(desc, orc.synthetic(kind, SEED, 1, columns))

        def ref(r):
            return orc.dot_codes(desc, mc[r * columns:(r + 1) * columns], vc, threads=1)
    return m, v, ref


def _gemv(ws, name, layout, accum, m, v, rows, columns, strategy=0, decoder=0):
    import torch
    from accessor_universal_test_b200 import _lib
    out = torch.full((max(rows, 1),), float("nan"), dtype=torch.float64, device="cuda")
    ws.gemv(_lib.format_id(name), layout, accum, m.data_ptr(), v.data_ptr(), rows, columns,
            out.data_ptr(), strategy=strategy, decoder=decoder)
    torch.cuda.synchronize()
    assert ws.status() == 0
    return out.cpu().numpy()[:rows]


def _check_rows(got, ref, accum, rows, label):
    for r in range(rows):
        d, s = ref(r)
        want = np.longdouble(d[0]) + np.longdouble(d[1])
        sabs = np.longdouble(s[0]) + np.longdouble(s[1])
        err = normalized_error(got[r], want, sabs)
        assert err <= TOL[accum], (label, r, got[r], float(want), float(err))


@pytest.mark.parametrize("name", DOT_FORMATS)
@pytest.mark.parametrize("layout", [0, 1])
def test_gemv_rows_match_oracle(ws, orc, name, layout):
    # 4096 columns: every row starts on a 16-byte boundary (vector paths);
    # 1000 columns: dense rows of 9/10/12/14/24/6-bit codes start inside a
    # word and are read by value index
    for rows, columns in ((37, 4096), (29, 1000)):
        m, v, ref = _operands(ws, orc, name, layout, rows, columns)
        for accum in _accums(name):
            got = _gemv(ws, name, layout, accum, m, v, rows, columns)
            _check_rows(got, ref, accum, rows, (name, layout, accum, columns))


@pytest.mark.parametrize("name", ["e8m0", "e2m3", "lns16_r11", "bf16_e8m7"])
@pytest.mark.parametrize("strategy", STRATEGIES)
def test_gemv_strategies_and_many_rows(ws, orc, name, strategy):
    # more rows than one launch carries (1024), both alignments
    for rows, columns in ((1100, 512), (1030, 333)):
        m, v, ref = _operands(ws, orc, name, 0, rows, columns)
        got = _gemv(ws, name, 0, 1, m, v, rows, columns, strategy=strategy)
        _check_rows(got, ref, 1, rows, (name, strategy, columns))


@pytest.mark.parametrize("decoder", [2, 3, 4])
def test_gemv_lns16_decoders(ws, orc, decoder):
    rows, columns = 64, 8192
    m, v, ref = _operands(ws, orc, "lns16_r11", 0, rows, columns)
    for accum in ((0, 1) if decoder != 2 else (0,)):
        got = _gemv(ws, "lns16_r11", 0, accum, m, v, rows, columns, decoder=decoder)
        _check_rows(got, ref, accum, rows, ("lns16_r11", decoder, accum))


def test_gemv_rows_equal_single_dots(ws, orc):
    """The e2m3 DOT is exact up to its final rounding, so row r of the GEMV
    equals aut_dot of that row bit for bit whatever grid either launch used."""
    import torch
    from accessor_universal_test_b200 import _lib
    rows, columns = 8, 1 << 14
    m, v, _ = _operands(ws, orc, "e2m3", 0, rows, columns)
    got = _gemv(ws, "e2m3", 0, 0, m, v, rows, columns)
    row_bytes = columns * 6 // 8
    for r in range(rows):
        res = torch.zeros(1, dtype=torch.float64, device="cuda")
        ws.dot(_lib.format_id("e2m3"), 0, 0, m.data_ptr() + r * row_bytes, v.data_ptr(),
               columns, res.data_ptr())
        torch.cuda.synchronize()
        assert got[r] == res.item(), r


def test_gemv_degenerate_shapes(ws):
    import torch
    from accessor_universal_test_b200 import _lib
    fid = _lib.format_id("e8m5")
    buf = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    out = torch.full((5,), 7.0, dtype=torch.float64, device="cuda")
    ws.gemv(fid, 0, 0, buf.data_ptr(), buf.data_ptr(), 5, 0, out.data_ptr())
    torch.cuda.synchronize()
    assert out.cpu().tolist() == [0.0] * 5
    ws.gemv(fid, 0, 0, 0, 0, 0, 100, out.data_ptr())  # no rows: nothing to do
    with pytest.raises(_lib.AutError) as info:
        ws.gemv(fid, 0, 0, buf.data_ptr(), buf.data_ptr(), 1 << 33, 4, out.data_ptr())
    assert info.value.status == _lib.AUT_ERR_TOO_LARGE


# The FP32 GEMV of the E8 codes, raw FP32 and lns8_r3 decodes the vector once
# per block when the columns are whole segments (one bulk-copy tile per row:
# 16384 values for 9- and 8-bit codes, 8192 for the others).
VECTOR_ONCE = ["e8m0", "e8m1", "e8m3", "e8m5", "bf16_e8m7", "e8m15", "fp32", "e2m3", "lns8_r3"]


# FP64 rows decode the vector once for the E8 codes, raw FP32, e2m3 and
# lns8_r3 (its FP64 table; 8192 values per tile)
VECTOR_ONCE_F64 = ["e8m0", "e8m1", "e8m3", "e8m5", "bf16_e8m7", "e8m15", "fp32", "e2m3",
                   "lns8_r3"]


@pytest.mark.parametrize("name", VECTOR_ONCE)
@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("accum", [0, 1])
def test_gemv_vector_once_rows_match_oracle(ws, orc, name, layout, accum):
    if accum == 1 and name not in VECTOR_ONCE_F64:
        pytest.skip("FP64 rows of this format take the batch path")
    # 1 row; 37 rows (a ragged group of 5); 1030 rows (two launches)
    for rows, columns in ((1, 16384), (37, 32768), (1030, 16384)):
        if name == "fp32" and layout == 1:
            continue
        m, v, ref = _operands(ws, orc, name, layout, rows, columns)
        got = _gemv(ws, name, layout, accum, m, v, rows, columns)
        _check_rows(got, ref, accum, rows, (name, layout, accum, rows, columns))


@pytest.mark.parametrize("layout", [0, 1])
def test_gemv_fp64_rows_with_tiny_and_huge_products(ws, orc, layout):
    """FP64 rows of e8m5 whose products fall below 2^-126 or overflow FP32:
    those row tiles are summed again from widened operands, so every row is
    the FP64 sum of exact products (compared with the long-double oracle)."""
    import torch
    from accessor_universal_test_b200 import _lib
    rows, columns = 12, 16384
    desc = _lib.format_info(_lib.format_id("e8m5"))
    vals = orc.synthetic(0, 11, 0, rows * columns).reshape(rows, columns)
    vec = orc.synthetic(0, 11, 1, columns)
    vals[2, 10:40] *= 2.0 ** -120      # times the vector values below: under 2^-126
    vec[10:40] *= 2.0 ** -10
    vals[6, 3000] = 2.0 ** 100         # times a vector value of 2^60: over FP32
    vec[3000] = 2.0 ** 60
    vals[9, :] = 0.0                   # a row of zero products
    mc = orc.encode(desc, vals.ravel())
    vc = orc.encode(desc, vec)
    fid = _lib.format_id("e8m5")
    bufs = []
    for codes in (mc, vc):
        if layout == 0:
            words = orc.pack_dense(desc[1], codes)
            data = words.view(np.uint8).copy()
        else:
            data = codes.astype(np.uint16).view(np.uint8).copy()
        bufs.append(torch.from_numpy(data).cuda())
    got = _gemv(ws, "e8m5", layout, 1, bufs[0], bufs[1], rows, columns)
    for r in range(rows):
        d, s = orc.dot_codes(desc, mc[r * columns:(r + 1) * columns], vc, threads=1)
        want = np.longdouble(d[0]) + np.longdouble(d[1])
        sabs = np.longdouble(s[0]) + np.longdouble(s[1])
        if sabs == 0:
            assert got[r] == 0.0, (r, got[r])
        else:
            assert normalized_error(got[r], want, sabs) <= TOL[1], (r, got[r], float(want))


def test_gemv_vector_once_is_deterministic(ws, orc):
    rows, columns = 300, 1 << 16
    m, v, _ = _operands(ws, orc, "e8m3", 0, rows, columns)
    a = _gemv(ws, "e8m3", 0, 0, m, v, rows, columns)
    for _ in range(3):
        b = _gemv(ws, "e8m3", 0, 0, m, v, rows, columns)
        assert a.tobytes() == b.tobytes()


def test_gemv_vector_once_special_values(ws, orc):
    """Inf and NaN codes in the matrix and the vector reach the rows they
    touch, and only those."""
    import torch
    from accessor_universal_test_b200 import _lib
    rows, columns = 24, 16384
    desc = _lib.format_info(_lib.format_id("e8m5"))
    vals = orc.synthetic(0, 5, 0, rows * columns).reshape(rows, columns)
    vec = orc.synthetic(0, 5, 1, columns)
    vals[3, 100] = np.inf
    vals[7, 9000] = np.nan
    vals[11, 5] = np.inf
    vals[11, 6] = -np.inf
    mc = orc.encode(desc, vals.ravel())
    vc = orc.encode(desc, vec)
    fid = _lib.format_id("e8m5")
    bufs = []
    for codes in (mc, vc):
        words = orc.pack_dense(desc[1], codes)
        assert words.size * 4 == _lib.storage_bytes(fid, 0, codes.size)
        bufs.append(torch.from_numpy(words.view(np.uint8).copy()).cuda())
    got = _gemv(ws, "e8m5", 0, 0, bufs[0], bufs[1], rows, columns)
    dec_m = orc.decode_f64(desc, mc).reshape(rows, columns)
    dec_v = orc.decode_f64(desc, vc)
    for r in range(rows):
        with np.errstate(invalid="ignore", over="ignore"):
            want = float((dec_m[r] * dec_v).sum())
        if np.isnan(want):
            assert np.isnan(got[r]), r
        elif np.isinf(want):
            assert got[r] == want, (r, got[r], want)
        else:
            assert np.isfinite(got[r]), r


@pytest.mark.parametrize("name", ["e8m0", "e8m5", "e8m15"])
def test_gemv_whole_segments_on_the_batch_path(ws, orc, name):
    """Whole-segment shapes that the vector-once kernel does not take: the
    LDG strategy and a matrix that does not start on a 16-byte boundary
    (value-index rows on the per-value path); and the FP64 rows beside
    them."""
    import torch
    from accessor_universal_test_b200 import _lib
    rows, columns = 19, 16384
    m, v, ref = _operands(ws, orc, name, 0, rows, columns)
    got = _gemv(ws, name, 0, 1, m, v, rows, columns)
    _check_rows(got, ref, 1, rows, (name, "fp64"))
    got = _gemv(ws, name, 0, 0, m, v, rows, columns, strategy=1)
    _check_rows(got, ref, 0, rows, (name, "ldg"))
    # the same matrix copied 4 bytes into a larger buffer
    shifted = torch.zeros(m.numel() + 16, dtype=torch.uint8, device="cuda")
    shifted[4:4 + m.numel()] = m
    out = torch.full((rows,), float("nan"), dtype=torch.float64, device="cuda")
    ws.gemv(_lib.format_id(name), 0, 0, shifted.data_ptr() + 4, v.data_ptr(), rows, columns,
            out.data_ptr())
    torch.cuda.synchronize()
    assert ws.status() == 0
    _check_rows(out.cpu().numpy(), ref, 0, rows, (name, "unaligned"))


@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("accum", [0, 1])
def test_gemv_e2m3_rows_are_exact(ws, orc, layout, accum):
    """e2m3 products and their partial sums are exact, so every row of the
    vector-once GEMV is the exact row sum rounded once, with either
    accumulator."""
    rows, columns = 21, 32768
    m, v, ref = _operands(ws, orc, "e2m3", layout, rows, columns)
    got = _gemv(ws, "e2m3", layout, accum, m, v, rows, columns)
    for r in range(rows):
        d, _ = ref(r)
        assert got[r] == float(np.longdouble(d[0]) + np.longdouble(d[1])), (layout, accum, r)


@pytest.mark.parametrize("accum", [0, 1])
def test_gemv_lns8_reserved_codes(ws, orc, accum):
    """lns8_r3 rows on the vector-once kernel (the FP32 and the FP64 table):
    the reserved code decodes to zero with its sign bit clear and to NaN with
    it set, in the matrix and in the vector; a NaN reaches only its row."""
    import torch
    from accessor_universal_test_b200 import _lib
    rows, columns = 24, 16384
    fid = _lib.format_id("lns8_r3")
    desc = _lib.format_info(fid)
    mc = orc.encode(desc, orc.synthetic(3, SEED, 0, rows * columns))
    vc = orc.encode(desc, orc.synthetic(3, SEED, 1, columns))
    mc[2 * columns + 17] = 0x40    # zero
    mc[2 * columns + 18] = 0x40
    mc[5 * columns + 4000] = 0xc0  # NaN
    mc[9 * columns:10 * columns] = 0x40  # a row of zeros
    vc[123] = 0x40                 # a zero in the vector touches every row
    bufs = [torch.from_numpy(orc.pack_dense(8, c).view(np.uint8).copy()).cuda() for c in (mc, vc)]
    got = _gemv(ws, "lns8_r3", 0, accum, bufs[0], bufs[1], rows, columns)
    for r in range(rows):
        if r == 5:
            assert np.isnan(got[r]), got[r]
            continue
        d, s = orc.dot_codes(desc, mc[r * columns:(r + 1) * columns], vc, threads=1)
        want = np.longdouble(d[0]) + np.longdouble(d[1])
        sabs = np.longdouble(s[0]) + np.longdouble(s[1])
        if r == 9:
            assert got[r] == 0.0, got[r]
            continue
        assert normalized_error(got[r], want, sabs) <= TOL[accum], (r, got[r], float(want))

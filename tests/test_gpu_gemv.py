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

"""The approximate LNS decoder (AUT_DECODER_EX2_APPROX: logs added, one
hardware ex2.approx.f32 per pair -- the reference's ex2_approx decoder with
the fused multiply) through the C ABI.

Stated bounds, written here:
  * every product's magnitude 2^((cx + cy) / 2^R) within a relative 2^-21 of
    the exact power of two -- checked for every log sum the format can form;
  * the DOT's normalised error within the exact decoders' bound plus 2^-21
    (FP32 accumulator 2e-6 + 2^-21, FP64 accumulator 1e-14 + 2^-21).
"""
import numpy as np
import pytest

from gpu_util import TOL, device_pair, gpu_dot, normalized_error, oracle_dot

pytestmark = pytest.mark.gpu

EX2 = 6
REL = 2.0 ** -21
TOL_EX2 = {0: TOL[0] + REL, 1: TOL[1] + REL}
FORMATS = {"lns8_r3": (8, 3), "lns16_r11": (16, 11)}


def _code(bits, log):
    """LNS code of +2^(log / 2^R): positive sign, two's-complement log."""
    return log & ((1 << (bits - 1)) - 1)


@pytest.mark.parametrize("name", sorted(FORMATS))
@pytest.mark.parametrize("accum", [0, 1])
def test_every_log_sum_within_the_stated_relative_error(ws, name, accum):
    """GEMVs with one column read each row by value index, so row r is the
    single product m_r * v: with m_r running over every finite log code and
    v over three logs (-max, 0, +max), the products cover every log sum."""
    import torch
    from accessor_universal_test_b200 import _lib
    bits, r = FORMATS[name]
    fid = _lib.format_id(name)
    top = (1 << (bits - 2)) - 1  # largest finite log code
    logs = np.arange(-top, top + 1, dtype=np.int64)
    # padded = dense for 8- and 16-bit codes: one container per code
    dt = np.uint8 if bits == 8 else np.uint16
    m = torch.from_numpy(np.array([_code(bits, int(c)) for c in logs], dtype=dt)).cuda()
    worst = 0.0
    for v_log in (-top, 0, top):
        v = torch.from_numpy(np.array([_code(bits, v_log)] * 8, dtype=dt)).cuda()
        out = torch.full((logs.size,), float("nan"), dtype=torch.float64, device="cuda")
        ws.gemv(fid, _lib.DENSE, accum, m.data_ptr(), v.data_ptr(), logs.size, 1,
                out.data_ptr(), decoder=EX2)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        want = np.exp2((logs + v_log).astype(np.float64) / (1 << r))
        rel = np.abs(got - want) / want
        worst = max(worst, float(rel.max()))
        assert rel.max() <= REL, (name, accum, v_log, float(rel.max()),
                                  int(logs[int(rel.argmax())]))
    print(f"{name} acc={'fp64' if accum else 'fp32'}: worst relative error of ex2.approx "
          f"products {worst:.3e} (bound {REL:.3e})")


@pytest.mark.parametrize("name", sorted(FORMATS))
@pytest.mark.parametrize("strategy", [1, 2, 3])
def test_ex2_dot_within_its_bound(ws, orc, name, strategy):
    for n in (3, 4099, (1 << 20) + 37):
        x, y = device_pair(ws, name, 0, n)
        ref_dot, ref_abs = oracle_dot(orc, name, n)
        for accum in (0, 1):
            got = gpu_dot(ws, name, 0, accum, x, y, n, strategy=strategy, decoder=EX2)
            err = normalized_error(got, ref_dot, ref_abs)
            assert err <= TOL_EX2[accum], (name, accum, strategy, n, got, float(err))


def test_ex2_is_refused_for_other_formats(ws):
    import torch
    from accessor_universal_test_b200 import _lib
    x = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    res = torch.zeros(1, dtype=torch.float64, device="cuda")
    for name in ("e8m0", "e2m3", "fp32", "lns16_r4"):
        with pytest.raises(_lib.AutError):
            ws.dot(_lib.format_id(name), 0, 0, x.data_ptr(), x.data_ptr(), 64,
                   res.data_ptr(), decoder=EX2)


def test_auto_never_picks_ex2(ws, orc):
    """AUTO stays on the exact decoders: with the same access strategy it
    runs the fraction-table fused decoder and agrees with it bit for bit."""
    from accessor_universal_test_b200 import _lib
    n = (1 << 20) + 37
    x, y = device_pair(ws, "lns16_r11", 0, n)
    auto = gpu_dot(ws, "lns16_r11", 0, 1, x, y, n, strategy=2)
    table = gpu_dot(ws, "lns16_r11", 0, 1, x, y, n, strategy=2,
                    decoder=_lib.DECODER_FRACTION_LUT_FUSED)
    assert auto == table

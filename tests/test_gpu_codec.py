"""Device decode / encode / generators against the oracle, bit for bit."""
import numpy as np
import pytest

from gpu_util import SEED

pytestmark = pytest.mark.gpu

DECODE_FORMATS = ["fp32", "e2m3", "e8m0", "e8m1", "e8m3", "e8m5", "bf16_e8m7", "e8m15",
                  "lns8_r3", "lns16_r11", "e3m4", "e0m7", "e11m4", "e11m20", "lns6_r2",
                  "fp4_e2m1", "e5m11", "e1m14", "e4m23"]


def _codes_for(bits, rng):
    if bits <= 16:
        codes = np.arange(1 << bits, dtype=np.uint32)
        # Repeat to at least 4099 (prime) codes so launches end in partial
        # warps and ragged blocks (src/lns_strategy_bench.cu:414-437).
        reps = max(1, -(-4099 // codes.size))
        codes = np.tile(codes, reps)
        if codes.size % 2 == 0:
            codes = codes[:-1]
        return codes
    return rng.integers(0, 1 << bits, 1 << 20 | 37, dtype=np.uint64).astype(np.uint32)


@pytest.mark.parametrize("name", DECODE_FORMATS)
@pytest.mark.parametrize("layout", [0, 1])
def test_device_decode_is_bit_exact(ws, orc, name, layout):
    import torch
    from accessor_universal_test_b200 import _lib
    fid = _lib.format_id(name)
    desc = _lib.format_info(fid)
    codes = _codes_for(desc[1], np.random.default_rng(5))
    n = codes.size
    packed = np.zeros(_lib.storage_bytes(fid, layout, n), np.uint8)
    _lib.check(_lib.load().aut_pack_host(fid, layout, codes.ctypes.data, n, packed.ctypes.data))
    dev = torch.from_numpy(packed).cuda()
    got64 = torch.empty(n, dtype=torch.float64, device="cuda")
    got32 = torch.empty(n, dtype=torch.float32, device="cuda")
    ws.decode(fid, layout, _lib.TARGET_FP64, dev.data_ptr(), n, got64.data_ptr())
    ws.decode(fid, layout, _lib.TARGET_FP32, dev.data_ptr(), n, got32.data_ptr())
    torch.cuda.synchronize()
    want64 = orc.decode_f64(desc, codes)
    want32 = orc.decode_f32(desc, codes)
    g64 = got64.cpu().numpy()
    g32 = got32.cpu().numpy()
    assert np.array_equal(g64.view(np.uint64), want64.view(np.uint64)), name
    nan = np.isnan(want32)
    # FP32 NaN payloads follow the hardware narrowing; every other value is
    # bit-identical.
    assert np.array_equal(np.isnan(g32), nan)
    assert np.array_equal(g32[~nan].view(np.uint32), want32[~nan].view(np.uint32)), name


def _encode_inputs(orc, desc, rng):
    codes = np.arange(1 << min(desc[1], 16), dtype=np.uint32)
    dec = orc.decode_f64(desc, codes)
    fin = np.unique(dec[np.isfinite(dec)])
    mids = (fin[:-1] + fin[1:]) / 2
    near = np.concatenate([mids, np.nextafter(mids, np.inf), np.nextafter(mids, -np.inf)])
    if desc[0] == 2:  # LNS: log-domain rounding boundaries
        r = desc[2]
        k = np.arange(-(1 << (desc[1] - 2)), 1 << (desc[1] - 2), dtype=np.float64)
        b = np.exp2((k + 0.5) / (1 << r))
        near = np.concatenate([near, b, np.nextafter(b, 0), np.nextafter(b, np.inf),
                               -b, np.nextafter(np.nextafter(b, 0), 0)])
    return np.concatenate([
        fin, near, orc.synthetic(0, SEED, 0, 50_000), orc.synthetic(2, SEED, 1, 50_000),
        rng.standard_normal(20_000) * rng.choice([1e-40, 1e-6, 1.0, 1e6, 1e40], 20_000),
        [0.0, -0.0, np.inf, -np.inf, np.nan, 5e-324, 1e308, -1e308]])


@pytest.mark.parametrize("name", ["fp32", "e2m3", "e8m0", "e8m1", "e8m3", "e8m5",
                                  "bf16_e8m7", "e8m15", "lns8_r3", "lns16_r11",
                                  "e3m4", "e0m7", "e11m4", "lns6_r2"])
@pytest.mark.parametrize("layout", [0, 1])
def test_device_encode_matches_host_encoder(ws, orc, name, layout):
    import torch
    from accessor_universal_test_b200 import _lib
    fid = _lib.format_id(name)
    desc = _lib.format_info(fid)
    vals = _encode_inputs(orc, desc, np.random.default_rng(9))
    n = vals.size
    want_codes = orc.encode(desc, vals)
    want = np.zeros(_lib.storage_bytes(fid, layout, n), np.uint8)
    _lib.check(_lib.load().aut_pack_host(fid, layout, want_codes.ctypes.data, n,
                                         want.ctypes.data))
    dv = torch.from_numpy(vals).cuda()
    out = torch.full((want.size,), 0xAB, dtype=torch.uint8, device="cuda")
    ws.encode(fid, layout, dv.data_ptr(), n, out.data_ptr())
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    if not np.array_equal(got, want):
        back = np.empty(n, np.uint32)
        _lib.check(_lib.load().aut_unpack_host(fid, layout, got.ctypes.data, n, back.ctypes.data))
        bad = np.nonzero(back != want_codes)[0][:5]
        raise AssertionError(f"{name}: {vals[bad]} -> {back[bad]} want {want_codes[bad]}")


@pytest.mark.parametrize("kind", [0, 1, 2, 3, 4])
def test_device_generators_match_oracle(orc, autlib, kind):
    import torch
    from accessor_universal_test_b200 import _lib
    for vec in (0, 1):
        for first, n in [(0, 1000), (123_456_789, 4099)]:
            out = torch.empty(n, dtype=torch.float64, device="cuda")
            _lib.generate(kind, SEED, vec, first, n, out.data_ptr())
            torch.cuda.synchronize()
            want = orc.synthetic(kind, SEED, vec, n, first)
            assert np.array_equal(out.cpu().numpy().view(np.uint64), want.view(np.uint64))

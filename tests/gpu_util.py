"""Shared helpers of the GPU parity tests (CUDA path via the C ABI, oracle as
the checker)."""
import numpy as np

SEED = 0x243F6A8885A308D3
DOT_FORMATS = ["fp32", "fp64", "e2m3", "e8m0", "e8m1", "e8m3", "e8m5",
               "bf16_e8m7", "e8m15", "lns8_r3", "lns16_r11"]
# generator kind per workload: 0 signed uniform double, 1 signed uniform
# float, 2 Irwin-Hall normal, 3 LNS cancellation pair
KIND = {"fp32": 1, "fp64": 0, "e2m3": 2, "lns8_r3": 3, "lns16_r11": 3}

# Normalised-error bounds |gpu - ref| / sum|x_i y_i| written into the tests:
#   FP64 accumulator: FP64 FMA chains + FP64 tree; bound 1e-14.
#   FP32 accumulator: FP32 FMA chains of at most 32 products between FP64
#   carries (4 chains x 128-value packets), so the worst case is 32 * 2^-24
#   = 1.9e-6; bound 2e-6.  The reference's FP32 kernel chains ~1024
#   products per thread at 2^27 (worst case ~6e-5).
TOL = {0: 2e-6, 1: 1e-14}


def kind_of(name):
    return KIND.get(name, 0)


def device_pair(ws, name, layout, n, seed=SEED):
    from accessor_universal_test_b200 import vectors
    kind = kind_of(name)
    x = vectors.encoded(ws, name, layout, kind, seed, 0, n)
    y = vectors.encoded(ws, name, layout, kind, seed, 1, n)
    return x, y


STRATEGIES = [1, 2, 3]  # LDG (registers), TMA (bulk copies into shared memory), SCALAR


def gpu_dot(ws, name, layout, accum, x, y, n, x_off=0, y_off=0, strategy=0, decoder=0):
    import torch
    from accessor_universal_test_b200 import _lib
    res = torch.full((1,), float("nan"), dtype=torch.float64, device=x.device)
    ws.dot(_lib.format_id(name), layout, accum, x.data_ptr() + x_off,
           y.data_ptr() + y_off, n, res.data_ptr(), strategy=strategy, decoder=decoder)
    torch.cuda.synchronize()
    assert ws.status() == 0, "a bounded device wait timed out"
    return float(res.item())


def oracle_codes(orc, name, n, vector_id, seed=SEED):
    from accessor_universal_test_b200 import _lib
    desc = _lib.format_info(_lib.format_id(name))
    vals = orc.synthetic(kind_of(name), seed, vector_id, n)
    return desc, vals, orc.encode(desc, vals)


def oracle_dot(orc, name, n, seed=SEED, threads=8):
    """(dot, sum_abs) as long doubles from the compensated reference."""
    if name in ("fp32", "fp64"):
        x = orc.synthetic(kind_of(name), seed, 0, n)
        y = orc.synthetic(kind_of(name), seed, 1, n)
        if name == "fp32":
            x, y = x.astype(np.float32), y.astype(np.float32)
        d, s = orc.dot_reference(x, y)
    else:
        desc, _, cx = oracle_codes(orc, name, n, 0, seed)
        _, _, cy = oracle_codes(orc, name, n, 1, seed)
        d, s = orc.dot_codes(desc, cx, cy, threads=threads)
    return (np.longdouble(d[0]) + np.longdouble(d[1]),
            np.longdouble(s[0]) + np.longdouble(s[1]))


def normalized_error(got, ref_dot, ref_abs):
    if ref_abs == 0:
        return abs(np.longdouble(got) - ref_dot)
    return abs(np.longdouble(got) - ref_dot) / ref_abs

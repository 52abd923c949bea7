"""aut_dot_noalloc: the fused DOT for callers that cannot allocate device
memory (their GPU memory belongs to another framework's pool, or a
cudaMalloc would stall a latency-critical path).  Its reduction scratch is a
fixed device array inside the library instead of a workspace.

Checked through the C ABI against the workspace entry point (aut_dot) and
the oracle's compensated long-double DOT, twice in a row so the second call
runs on the scratch the first one left behind; both layouts, pointers off
the 16-byte grid (the per-value path) and n = 0.  This file sorts last so
that a run stopping at its first failure has run every other test already.
"""
import ctypes as C

import numpy as np
import pytest

from gpu_util import TOL, device_pair, gpu_dot, oracle_dot

pytestmark = pytest.mark.gpu


def _noalloc(fid, layout, accum, x_ptr, y_ptr, n, batch, stride, res_ptr):
    from accessor_universal_test_b200 import _lib
    return _lib.load().aut_dot_noalloc(fid, layout, accum, x_ptr, y_ptr, n, batch,
                                       stride, res_ptr, None)


@pytest.mark.parametrize("name", ["e8m0", "e8m15", "e2m3", "bf16_e8m7", "fp32", "fp64",
                                  "e5m11", "e9m22"])
def test_noalloc_dot_matches_workspace_dot_twice_in_a_row(ws, orc, name):
    import torch
    from accessor_universal_test_b200 import _lib
    fid = _lib.format_id(name)
    n = (1 << 21) + 77
    for layout in (_lib.DENSE, _lib.PADDED):
        x, y = device_pair(ws, name, layout, n)
        ref_dot, ref_abs = oracle_dot(orc, name, n)
        accums = [a for a in (0, 1) if _lib.load().aut_dot_supported(fid, layout, a)]
        for accum in accums:
            want = gpu_dot(ws, name, layout, accum, x, y, n)
            for call in range(2):
                res = torch.full((1,), float("nan"), dtype=torch.float64, device="cuda")
                st = _noalloc(fid, layout, accum, x.data_ptr(), y.data_ptr(), n, 1, 0,
                              res.data_ptr())
                assert st == _lib.AUT_OK, _lib.load().aut_last_error()
                torch.cuda.synchronize()
                got = float(res.item())
                assert abs(got - want) <= TOL[accum] * float(ref_abs), (
                    name, layout, accum, call, got, want)
                err = abs(np.longdouble(got) - ref_dot) / ref_abs
                assert err <= TOL[accum], (name, layout, accum, call, got, float(ref_dot))


@pytest.mark.parametrize("name,layout", [("e8m1", 0), ("e2m3", 1), ("fp32", 0)])
def test_noalloc_off_grid_pointers_take_the_per_value_path(ws, orc, name, layout):
    """The same streams copied to start 4 bytes past a 16-byte boundary:
    both entry points read them value by value."""
    import torch
    from accessor_universal_test_b200 import _lib
    fid = _lib.format_id(name)
    n = 100_003
    x, y = device_pair(ws, name, layout, n)
    xs = torch.zeros(x.numel() + 16, dtype=torch.uint8, device="cuda")
    ys = torch.zeros(y.numel() + 16, dtype=torch.uint8, device="cuda")
    xs[4:4 + x.numel()] = x
    ys[4:4 + y.numel()] = y
    ref_dot, ref_abs = oracle_dot(orc, name, n)
    for accum in (0, 1):
        want = gpu_dot(ws, name, layout, accum, xs, ys, n, x_off=4, y_off=4)
        for call in range(2):
            res = torch.full((1,), float("nan"), dtype=torch.float64, device="cuda")
            assert _noalloc(fid, layout, accum, xs.data_ptr() + 4, ys.data_ptr() + 4, n, 1, 0,
                            res.data_ptr()) == _lib.AUT_OK, _lib.load().aut_last_error()
            torch.cuda.synchronize()
            got = float(res.item())
            assert abs(got - want) <= TOL[accum] * float(ref_abs), (name, accum, call, got, want)
            err = abs(np.longdouble(got) - ref_dot) / ref_abs
            assert err <= TOL[accum], (name, accum, call, got, float(ref_dot))


def test_noalloc_empty_vectors_give_zero(ws):
    import torch
    from accessor_universal_test_b200 import _lib
    fid = _lib.format_id("e8m0")
    buf = torch.zeros(64, dtype=torch.uint8, device="cuda")
    for call in range(2):
        res = torch.full((2,), float("nan"), dtype=torch.float64, device="cuda")
        assert _noalloc(fid, _lib.DENSE, 0, buf.data_ptr(), buf.data_ptr(), 0, 2, 16,
                        res.data_ptr()) == _lib.AUT_OK, _lib.load().aut_last_error()
        torch.cuda.synchronize()
        assert res.cpu().tolist() == [0.0, 0.0], call


def test_noalloc_batch_matches_single_dots(ws, orc):
    import torch
    from accessor_universal_test_b200 import _lib
    name = "e8m3"
    fid = _lib.format_id(name)
    n, batch = 300_001, 3
    stride = (_lib.storage_bytes(fid, _lib.DENSE, n) + 255) // 256 * 256
    xb = torch.zeros(stride * batch, dtype=torch.uint8, device="cuda")
    yb = torch.zeros(stride * batch, dtype=torch.uint8, device="cuda")
    singles, scale = [], []
    for b in range(batch):
        x, y = device_pair(ws, name, _lib.DENSE, n, seed=0x1234 + b)
        xb[b * stride: b * stride + x.numel()] = x
        yb[b * stride: b * stride + y.numel()] = y
        singles.append(gpu_dot(ws, name, _lib.DENSE, 1, x, y, n))
        scale.append(float(oracle_dot(orc, name, n, seed=0x1234 + b)[1]))
    for call in range(2):
        res = torch.full((batch,), float("nan"), dtype=torch.float64, device="cuda")
        assert _noalloc(fid, _lib.DENSE, 1, xb.data_ptr(), yb.data_ptr(), n, batch, stride,
                        res.data_ptr()) == _lib.AUT_OK
        torch.cuda.synchronize()
        got = res.cpu().numpy()
        for b in range(batch):
            assert abs(got[b] - singles[b]) <= TOL[1] * scale[b], (call, b)


def test_noalloc_refuses_what_it_cannot_hold(autlib):
    import torch
    from accessor_universal_test_b200 import _lib
    res = torch.zeros(65, dtype=torch.float64, device="cuda")
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    fid = _lib.format_id("e8m0")
    assert _noalloc(fid, 0, 0, buf.data_ptr(), buf.data_ptr(), 16, 65, 4096,
                    res.data_ptr()) == _lib.AUT_ERR_TOO_LARGE
    assert b"64" in autlib.aut_last_error()
    assert _noalloc(_lib.format_id("lns16_r11"), 0, 0, buf.data_ptr(), buf.data_ptr(), 16,
                    1, 0, res.data_ptr()) == _lib.AUT_ERR_UNSUPPORTED

"""Failure detection on the GPU without a fault: the bulk-copy kernels' bounded
barrier waits run out, the kernel reports it, and the context stays usable.

aut_workspace_inject_stall arms one tile's ring stage without issuing its
copies (so no copy is ever in flight for it) and shortens the wait bound to
about a millisecond; the wait for that tile gives up, the block lets its
other copies land, the workspace's sticky status gets
AUT_STATUS_WAIT_TIMEOUT and the DOT's result is NaN.  Afterwards the same
workspace computes correct DOTs again.
"""
import math

import pytest

from gpu_util import TOL, device_pair, gpu_dot, normalized_error, oracle_dot

pytestmark = pytest.mark.gpu

SHORT_WAIT = 2_000_000  # SM clock cycles, ~1 ms


@pytest.mark.parametrize("name,accum,stall_tile", [("e8m0", 0, 0), ("e8m15", 1, 1),
                                                   ("e2m3", 0, 3)])
def test_bounded_wait_runs_out_and_reports(ws, orc, name, accum, stall_tile):
    import torch
    from accessor_universal_test_b200 import _lib
    fid = _lib.format_id(name)
    n = 1 << 22
    x, y = device_pair(ws, name, _lib.DENSE, n)
    assert ws.status() == 0
    ws.inject_stall(stall_tile, SHORT_WAIT)
    try:
        res = torch.zeros(1, dtype=torch.float64, device="cuda")
        ws.dot(fid, _lib.DENSE, accum, x.data_ptr(), y.data_ptr(), n, res.data_ptr(),
               strategy=_lib.STRATEGY_TMA)
        torch.cuda.synchronize()
        assert math.isnan(float(res.item()))
        assert ws.status(clear=False) == _lib.STATUS_WAIT_TIMEOUT
        assert ws.status(clear=True) == _lib.STATUS_WAIT_TIMEOUT
        assert ws.status() == 0
    finally:
        ws.inject_stall()
    # the context and the workspace still work
    ref_dot, ref_abs = oracle_dot(orc, name, n)
    got = gpu_dot(ws, name, _lib.DENSE, accum, x, y, n, strategy=_lib.STRATEGY_TMA)
    assert normalized_error(got, ref_dot, ref_abs) <= TOL[accum]


def test_stall_hook_rejects_a_longer_bound(ws):
    from accessor_universal_test_b200 import _lib
    with pytest.raises(_lib.AutError):
        ws.inject_stall(0, 1 << 40)

"""Stream order under programmatic dependent launch, and the dynamic tail of
exact DOTs, through the C ABI.

The fused DOT kernels are launched with programmatic stream serialisation:
a DOT may be scheduled while the kernel before it on the stream is still
running, and reads nothing before that kernel has completed.  These tests
enqueue producer kernels (generate + encode) and DOTs back to back on one
stream, reusing the same input buffers, with no host synchronisation in
between, and check every result against the same DOT computed in isolation.

For the exact e2m3 DOT the last rounds of tiles are claimed dynamically by
whichever block is free; the sums are exact, so results must be
bit-identical from run to run, equal to the oracle's exactly rounded DOT,
and equal between the single and the batched entry points.
"""
import numpy as np
import pytest

from gpu_util import SEED, device_pair, gpu_dot, oracle_dot

pytestmark = pytest.mark.gpu


def _encode_into(ws, name, layout, out, seed, vector_id, n, stream):
    """Re-encode vector `vector_id` of `seed` into the existing buffer `out`
    (called inside `torch.cuda.stream(stream)`, so the temporaries belong to
    that stream and are reused only in its order)."""
    from accessor_universal_test_b200 import vectors
    from gpu_util import kind_of
    fresh = vectors.encoded(ws, name, layout, kind_of(name), seed, vector_id, n,
                            stream=stream.cuda_stream)
    out[: fresh.numel()].copy_(fresh)


@pytest.mark.parametrize("name,layout,accum", [("e2m3", 0, 0), ("e8m0", 0, 1),
                                               ("lns8_r3", 0, 0), ("e8m15", 0, 0)])
def test_back_to_back_producers_and_dots_on_one_stream(ws, name, layout, accum):
    import torch
    from accessor_universal_test_b200 import _lib
    fid = _lib.format_id(name)
    ws.prepare(fid)
    n = (1 << 24) + 13
    seeds = [SEED + 17 * r for r in range(4)]
    # each round's DOT in isolation (synchronised)
    expect = []
    for s in seeds:
        x, y = device_pair(ws, name, layout, n, seed=s)
        expect.append(gpu_dot(ws, name, layout, accum, x, y, n))
        del x, y
    torch.cuda.synchronize()
    # the same rounds back to back on one stream, into the same two buffers
    x, y = device_pair(ws, name, layout, n, seed=seeds[0])
    stream = torch.cuda.Stream()
    res = torch.full((len(seeds),), float("nan"), dtype=torch.float64, device="cuda")
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for r, s in enumerate(seeds):
            _encode_into(ws, name, layout, x, s, 0, n, stream)
            _encode_into(ws, name, layout, y, s, 1, n, stream)
            ws.dot(fid, layout, accum, x.data_ptr(), y.data_ptr(), n,
                   res.data_ptr() + 8 * r, stream.cuda_stream)
    stream.synchronize()
    assert ws.status() == 0
    got = res.cpu().numpy()
    assert np.array_equal(got, np.array(expect)), (got, expect)


@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("accum", [0, 1])
def test_exact_dot_with_claimed_tail_tiles_is_bit_identical(ws, orc, layout, accum):
    import torch
    n = (1 << 25) + 4097  # several rounds of tiles per block: the dynamic tail runs
    x, y = device_pair(ws, "e2m3", layout, n)
    runs = [gpu_dot(ws, "e2m3", layout, accum, x, y, n) for _ in range(4)]
    assert len(set(runs)) == 1, runs
    swapped = gpu_dot(ws, "e2m3", layout, accum, y, x, n)
    assert swapped == runs[0]
    ref_dot, _ = oracle_dot(orc, "e2m3", n)
    assert runs[0] == float(ref_dot), (runs[0], float(ref_dot))
    del x, y
    torch.cuda.empty_cache()


def test_batched_exact_dots_claim_tiles_per_pair(ws):
    import torch
    from accessor_universal_test_b200 import _lib
    fid = _lib.format_id("e2m3")
    n, batch = (1 << 23) + 5, 3
    stride = (_lib.storage_bytes(fid, 0, n) + 255) // 256 * 256
    xb = torch.zeros(stride * batch, dtype=torch.uint8, device="cuda")
    yb = torch.zeros(stride * batch, dtype=torch.uint8, device="cuda")
    singles = []
    for b in range(batch):
        x, y = device_pair(ws, "e2m3", 0, n, seed=SEED + b)
        xb[b * stride: b * stride + x.numel()] = x[: min(x.numel(), stride)]
        yb[b * stride: b * stride + y.numel()] = y[: min(y.numel(), stride)]
        singles.append(gpu_dot(ws, "e2m3", 0, 0, x, y, n))
    for _ in range(2):  # the second call finds the claim counters reset
        res = torch.full((batch,), float("nan"), dtype=torch.float64, device="cuda")
        ws.dot_batched(fid, 0, 0, xb.data_ptr(), yb.data_ptr(), n, batch, stride,
                       res.data_ptr())
        torch.cuda.synchronize()
        assert res.cpu().numpy().tolist() == singles


def test_dot_after_host_to_device_copies_on_one_stream(ws):
    """The e2e pattern: pinned host buffers copied into the same device
    buffers round after round, each round's DOT enqueued right after its
    copies (copies are not kernels: the DOT waits for them in full)."""
    import torch
    from accessor_universal_test_b200 import _lib
    name, layout, accum = "e8m3", 0, 0
    fid = _lib.format_id(name)
    n = (1 << 22) + 3
    rounds = []
    for r in range(3):
        x, y = device_pair(ws, name, layout, n, seed=SEED + 5 * r)
        rounds.append((x.cpu().pin_memory(), y.cpu().pin_memory(),
                       gpu_dot(ws, name, layout, accum, x, y, n)))
        del x, y
    dx = torch.empty_like(rounds[0][0], device="cuda")
    dy = torch.empty_like(rounds[0][1], device="cuda")
    res = torch.full((len(rounds),), float("nan"), dtype=torch.float64, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for r, (hx, hy, _) in enumerate(rounds):
            dx.copy_(hx, non_blocking=True)
            dy.copy_(hy, non_blocking=True)
            ws.dot(fid, layout, accum, dx.data_ptr(), dy.data_ptr(), n,
                   res.data_ptr() + 8 * r, stream.cuda_stream)
    stream.synchronize()
    assert res.cpu().numpy().tolist() == [expect for _, _, expect in rounds]

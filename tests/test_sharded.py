"""Sharding plan and the all-reduce composition, on CPU with gloo ranks.

The per-shard DOT here is the oracle (the GPU path is covered by
tests/test_gpu_*.py and bench.py under torchrun); what is tested is the host
logic: shard edges, alignment, one collective per DOT, the sum of partials
against the unsharded reference, and that a rank failure surfaces on the
other rank as an error within the process-group timeout.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from accessor_universal_test_b200.sharded import plan, shard_alignment

SEED = 0x243F6A8885A308D3


@pytest.mark.parametrize("bits", [6, 8, 9, 10, 12, 14, 16, 24, 32])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_plan_is_contiguous_and_aligned(bits, world):
    n = (1 << 20) + 12345
    shards = plan(n, world, bits)
    assert [s.rank for s in shards] == list(range(world))
    assert shards[0].first == 0
    assert sum(s.count for s in shards) == n
    for a, b in zip(shards, shards[1:]):
        assert b.first == a.first + a.count
    for s in shards:
        assert s.first % shard_alignment(bits) == 0
        assert (s.first * bits) % 128 == 0  # 16-byte aligned in a dense stream
        assert s.byte_offset(bits) % 16 == 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, name, n, q, fail_rank):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.dirname(here))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "oracle"))
    import pyoracle
    from accessor_universal_test_b200 import _lib
    from accessor_universal_test_b200.sharded import ShardedDot
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        orc = pyoracle.oracle()
        desc = _lib.format_info(_lib.format_id(name))

        def local_dot(shard, out):
            if rank == fail_rank:
                raise RuntimeError("injected rank failure before the collective")
            x = orc.synthetic(0, SEED, 0, shard.count, shard.first)
            y = orc.synthetic(0, SEED, 1, shard.count, shard.first)
            d, _ = orc.dot_codes(desc, orc.encode(desc, x), orc.encode(desc, y))
            out[0] = d[0] + d[1]

        out = torch.zeros(1, dtype=torch.float64)
        try:
            ShardedDot(n, desc[1], rank, world, local_dot)(out)
            q.put((rank, "ok", float(out[0])))
        except Exception as e:  # noqa: BLE001 - report any failure to the parent
            q.put((rank, "error", type(e).__name__))
    finally:
        dist.destroy_process_group()


def _run(world, name, n, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, name, n, q, fail_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return sorted(out)


@pytest.mark.parametrize("name", ["e8m0", "e8m15"])
def test_sharded_sum_matches_unsharded_reference(orc, name):
    from accessor_universal_test_b200 import _lib
    n = 200_003
    res = _run(2, name, n)
    assert [r[1] for r in res] == ["ok", "ok"]
    assert res[0][2] == res[1][2]  # every rank holds the same global result
    desc = _lib.format_info(_lib.format_id(name))
    x = orc.synthetic(0, SEED, 0, n)
    y = orc.synthetic(0, SEED, 1, n)
    (d, s) = orc.dot_codes(desc, orc.encode(desc, x), orc.encode(desc, y))
    assert abs(res[0][2] - (d[0] + d[1])) <= 1e-14 * (s[0] + s[1])


def test_a_failing_rank_surfaces_as_an_error_not_a_hang():
    res = _run(2, "e8m0", 10_000, fail_rank=1)
    assert res[1][1] == "error"          # the failing rank reports its exception
    assert res[0][1] == "error"          # the survivor's collective fails by timeout


def _async_worker(rank, world, port, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.dirname(here))
    from accessor_universal_test_b200.sharded import allreduce_partials_async
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        # two buffers in flight at once, as the benchmark's overlapped steps use them
        a = torch.tensor([1.0 + rank, 10.0 * rank], dtype=torch.float64)
        b = torch.tensor([0.5 * rank, -3.0], dtype=torch.float64)
        wa = allreduce_partials_async(a)
        wb = allreduce_partials_async(b)
        wa.wait()
        wb.wait()
        q.put((rank, a.tolist(), b.tolist()))
    finally:
        dist.destroy_process_group()


def test_async_allreduce_of_two_buffers_in_flight():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_async_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    for _, a, b in out:
        assert a == [3.0, 10.0] and b == [0.5, -6.0]
    from accessor_universal_test_b200.sharded import allreduce_partials_async
    assert allreduce_partials_async(torch.zeros(1)) is None  # one rank: nothing to do

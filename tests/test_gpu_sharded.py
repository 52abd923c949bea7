"""aut_dot_sharded on two GPUs: ONE dense 9-bit stream split into two
contiguous shards whose edges fall on whole 16-byte packets (sharded.plan),
each rank running the fused DOT on its byte range of the stream and one
NCCL all-reduce of the FP64 partial; every rank's result is checked against
the oracle's unsharded DOT.  One process per GPU; the communicator id
travels over a gloo process group.  Skipped with fewer than two GPUs.
"""
import os
import socket

import pytest

pytestmark = pytest.mark.gpu

SEED = 0x243F6A8885A308D3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, name, n, accum, out_path):
    import datetime

    import torch
    import torch.distributed as dist

    from accessor_universal_test_b200 import _lib, vectors
    from accessor_universal_test_b200.sharded import plan

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    torch.cuda.set_device(rank)
    ids = [_lib.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(ids, src=0)
    comm = _lib.Comm(ids[0], world, rank, rank)
    ws = _lib.Workspace(rank)
    fid = _lib.format_id(name)
    bits = _lib.format_info(fid)[1]
    # the whole stream on every GPU; each rank reads its shard in place
    x = vectors.encoded(ws, fid, _lib.DENSE, 0, SEED, 0, n)
    y = vectors.encoded(ws, fid, _lib.DENSE, 0, SEED, 1, n)
    shard = plan(n, world, bits)[rank]
    off = shard.byte_offset(bits)
    assert off % 16 == 0
    res = torch.full((1,), float("nan"), dtype=torch.float64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # twice: the second call reuses the communicator
        comm.dot(ws, fid, _lib.DENSE, accum, x.data_ptr() + off, y.data_ptr() + off,
                 shard.count, res.data_ptr(), stream)
    torch.cuda.synchronize()
    got = float(res.item())
    with open(f"{out_path}.{rank}", "w") as f:
        f.write(repr(got))
    ws.close()
    comm.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("accum", [0, 1])
def test_two_gpus_split_one_dense_stream(orc, accum, tmp_path):
    import numpy as np
    import torch
    import torch.multiprocessing as mp

    from gpu_util import TOL, normalized_error, oracle_dot
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    name, n, world = "e8m0", (1 << 22) + 4099, 2
    out = str(tmp_path / "result")
    mp.start_processes(_worker, args=(world, _free_port(), name, n, accum, out),
                       nprocs=world, join=True, start_method="spawn")
    ref_dot, ref_abs = oracle_dot(orc, name, n)
    results = [float(open(f"{out}.{r}").read()) for r in range(world)]
    assert results[0] == results[1]
    err = normalized_error(results[0], ref_dot, ref_abs)
    assert err <= TOL[accum], (accum, results, float(ref_dot), float(err))
    assert np.isfinite(results[0])

"""Contiguous sharding of long DOTs over the GPUs of one node.

Each rank owns the contiguous slice [first, first + count) of the global
vectors, reduces it to one FP64 partial with the fused DOT (aut_dot), and a
single all-reduce of the FP64 partials -- NCCL over NVLink in production,
gloo in the CPU tests -- gives every rank the global result.  For dense
bitstreams the shard edges fall on whole 16-byte packets
(128 / gcd(bits, 128) values), so every shard starts 16-byte aligned and the
vectorised kernels run on every shard.
"""
from __future__ import annotations

import math
from dataclasses import dataclass


def shard_alignment(bits: int) -> int:
    """Values per 16-byte packet of a B-bit dense stream."""
    return 128 // math.gcd(bits, 128)


@dataclass(frozen=True)
class Shard:
    rank: int
    first: int   # first global index of the shard
    count: int   # values in the shard

    def byte_offset(self, bits: int) -> int:
        """Offset of the shard's first value in a dense stream (whole words)."""
        return self.first * bits // 8


def plan(n_total: int, world: int, bits: int) -> list[Shard]:
    """Contiguous shards of near-equal size with packet-aligned edges; the
    last shard takes the remainder."""
    if world < 1:
        raise ValueError("world must be >= 1")
    align = shard_alignment(bits)
    per = (n_total // world) // align * align
    shards, first = [], 0
    for r in range(world):
        count = per if r < world - 1 else n_total - first
        shards.append(Shard(r, first, count))
        first += count
    return shards


def allreduce_partials(partials, group=None):
    """Sum the per-rank FP64 partials in place: one collective per call."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(partials, op=dist.ReduceOp.SUM, group=group)
    return partials


def allreduce_partials_async(partials, group=None):
    """Start the in-place sum of the per-rank partials and return its work
    handle (None on one rank).  With NCCL the collective runs on the
    library's own stream after the kernels that wrote `partials`, so work
    launched next on the caller's stream overlaps it; ``handle.wait()`` makes
    the caller's stream (not the host) wait for the sum, which must happen
    before `partials` is read or written again."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        return dist.all_reduce(partials, op=dist.ReduceOp.SUM, group=group, async_op=True)
    return None


class ShardedDot:
    """Runs one DOT per rank over its shard and all-reduces the partials.

    ``local_dot(shard, out)`` writes the shard's partial into ``out[0]``; in
    production it is ``Workspace.dot`` on device buffers, in tests any
    callable (e.g. the oracle on CPU tensors)."""

    def __init__(self, n_total: int, bits: int, rank: int, world: int, local_dot, group=None):
        self.shards = plan(n_total, world, bits)
        self.shard = self.shards[rank]
        self.local_dot = local_dot
        self.group = group

    def __call__(self, out):
        self.local_dot(self.shard, out)
        return allreduce_partials(out, self.group)

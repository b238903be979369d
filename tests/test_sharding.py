"""Sharding and verification gather across ranks, on CPU with gloo (no GPU).

A two-rank run checks the batch/unit partition and the checksum all-gather; a second
run makes one rank leave before the gather and checks that the other rank gets an
error from the short process-group timeout instead of hanging.
"""

import os
import socket
import sys
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from moda.sharding import (BatchShard, gather_checksums, output_checksum, shard_batches,
                           unit_ranges, unit_shard)


def test_weak_and_strong_batch_shards():
    assert shard_batches(4, 8, 3, weak=True) == BatchShard(12, 16, 32)
    assert shard_batches(16, 8, 3, weak=False) == BatchShard(6, 8, 16)
    assert shard_batches(16, 1, 0, weak=False) == BatchShard(0, 16, 16)
    with pytest.raises(ValueError):
        shard_batches(16, 3, 0, weak=False)
    with pytest.raises(ValueError):
        shard_batches(4, 2, 2, weak=True)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_units_partition_the_scaling_workload(world):
    # B=16 batches x H_k=8 KV heads = 128 units, each on exactly one rank
    ranges = unit_ranges(16, 8, world)
    covered = sorted(u for r in ranges for u in r)
    assert covered == list(range(128))
    assert len({len(r) for r in ranges}) == 1


@pytest.mark.parametrize("units,world", [(128, 3), (128, 5), (128, 7), (32, 6), (3, 8), (0, 2)])
def test_units_partition_any_world_size(units, world):
    ranges = [unit_shard(units, world, r) for r in range(world)]
    assert [u for r in ranges for u in r] == list(range(units))  # contiguous, in rank order
    assert max(map(len, ranges)) - min(map(len, ranges)) <= 1     # balanced


def test_unit_slice_is_the_same_memory_as_the_batch_head_view():
    """A unit range read as [U, G, T, d] is the same bytes as the [B, H, T, d] view."""
    B, Hk, G, T, d = 3, 4, 2, 5, 8
    Q = torch.randn(B, Hk * G, T, d)
    K = torch.randn(B, Hk, T, d)
    r = unit_shard(B * Hk, 5, 2)
    Qu = Q.view(B * Hk, G, T, d)[r.start:r.stop]
    Ku = K.view(B * Hk, 1, T, d)[r.start:r.stop]
    for i, u in enumerate(r):
        b, hk = divmod(u, Hk)
        assert torch.equal(Qu[i], Q[b, hk * G:(hk + 1) * G])
        assert torch.equal(Ku[i, 0], K[b, hk])
    with pytest.raises(ValueError):
        unit_shard(8, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    try:
        shard = shard_batches(4, world, rank, weak=True)
        g = torch.Generator().manual_seed(1000 + shard.b_lo)
        O = torch.randn(shard.batch, 2, 8, 4, generator=g)
        cs = output_checksum(O)
        if mode == "leave" and rank == 1:
            results[rank] = "left"
            return                       # leaves before the collective, no kernel in flight
        try:
            got = gather_checksums(cs)
            results[rank] = [tuple(float(v) for v in t) for t in got]
        except Exception as e:           # the short timeout ends the collective
            results[rank] = "error:" + type(e).__name__
    finally:
        if not (mode == "leave" and rank == 1):
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(world, mode):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    return dict(results)


def test_gather_checksums_two_ranks():
    res = _run(2, "ok")
    assert len(res[0]) == 2 and res[0] == res[1]
    # rank r's checksum is the checksum of its own shard
    for r in range(2):
        g = torch.Generator().manual_seed(1000 + 4 * r)
        ref = output_checksum(torch.randn(4, 2, 8, 4, generator=g))
        assert res[0][r] == tuple(float(v) for v in ref)


def test_rank_leaving_before_the_gather_times_out():
    res = _run(2, "leave")
    assert res[1] == "left"
    assert isinstance(res[0], str) and res[0].startswith("error:")

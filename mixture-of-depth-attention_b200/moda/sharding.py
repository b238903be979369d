"""Multi-GPU sharding of the fused forward by (batch x KV head) units.

Units u = b * H_k + h_k are independent: each owns its G query heads, KV head h_k and
depth rows [b, h_k, :T*L]. No data moves between GPUs during the forward; NCCL is
used only to gather small per-rank checksums of the outputs for verification.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class BatchShard:
    b_lo: int         # first batch index of this rank
    b_hi: int         # one past the last
    global_batch: int

    @property
    def batch(self) -> int:
        return self.b_hi - self.b_lo


def shard_batches(batch: int, world: int, rank: int, weak: bool) -> BatchShard:
    """Batch range of `rank`.

    weak=True: every rank runs its own `batch` (global batch = batch * world).
    weak=False: `batch` is split evenly; it must be divisible by `world` (whole
    batches keep every rank's tensors contiguous and its units complete).
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if weak:
        return BatchShard(rank * batch, (rank + 1) * batch, batch * world)
    if batch % world:
        raise ValueError(f"batch {batch} is not divisible by {world} ranks")
    per = batch // world
    return BatchShard(rank * per, (rank + 1) * per, batch)


def unit_shard(units: int, world: int, rank: int) -> range:
    """Contiguous range of (batch x KV head) units of `rank`, for any world size: the
    first ``units % world`` ranks get one unit more than the others.

    Unit u = b * H_k + h_k owns Q[b, h_k*G:(h_k+1)*G], K/V[b, h_k] and the depth rows
    [b, h_k, :T*L]. In the contiguous [B, H, rows, d] layouts these are consecutive
    memory, so a contiguous unit range is one slice of every tensor and can be run as a
    problem of ``len(range)`` batches with G query heads and one KV head.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if units < 0:
        raise ValueError(f"negative unit count {units}")
    return range(rank * units // world, (rank + 1) * units // world)


def unit_ranges(batch: int, kv_heads: int, world: int) -> list[range]:
    """(batch x KV head) unit ranges of all ranks (strong scaling over any world size)."""
    return [unit_shard(batch * kv_heads, world, r) for r in range(world)]


def output_checksum(O: torch.Tensor) -> torch.Tensor:
    """[sum, sum of |x|, all finite] of one rank's output, float64, on O's device."""
    Of = O.float()
    return torch.stack([Of.sum(), Of.abs().sum(), torch.isfinite(O).all().float()]).to(torch.float64)


def gather_checksums(cs: torch.Tensor) -> list[torch.Tensor]:
    """All ranks' checksums (verification only; outside any timed region)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return [cs]
    out = [torch.zeros_like(cs) for _ in range(dist.get_world_size())]
    dist.all_gather(out, cs)
    return out

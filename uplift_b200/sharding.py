"""Batch sharding across GPUs (one process per GPU).

The Local Attender and the upsampler are independent per image, so the only
parallelism is splitting the image batch into contiguous shards; nothing is
exchanged while computing.  `gather_to_rank0` is the optional final gather of
the per-rank outputs (torch.distributed: NCCL over NVLink on GPUs, gloo on
CPUs).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist


def shard_bounds(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [lo, hi) slice of n items for `rank`; the first n % world
    ranks get one extra item."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's slice of a batch-first tensor."""
    lo, hi = shard_bounds(t.shape[0], rank, world)
    return t[lo:hi]


def gather_to_rank0(local: torch.Tensor, n_total: int, group: Optional[dist.ProcessGroup] = None):
    """Concatenate every rank's batch slice on rank 0 in rank order.

    All ranks must call it (it is a collective).  Shards may differ by one
    item, so every rank pads to the largest shard for an equal-size
    all_gather_into_tensor, and rank 0 trims.  Returns the full batch on
    rank 0 and None elsewhere."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    sizes = [shard_bounds(n_total, r, world) for r in range(world)]
    biggest = max(hi - lo for lo, hi in sizes)
    if local.shape[0] != sizes[rank][1] - sizes[rank][0]:
        raise ValueError(f"rank {rank} holds {local.shape[0]} items, expected {sizes[rank][1] - sizes[rank][0]}")
    padded = local.new_zeros((biggest,) + tuple(local.shape[1:]))
    padded[:local.shape[0]] = local
    flat = padded.contiguous()
    out = flat.new_empty((world * biggest,) + tuple(local.shape[1:]))
    dist.all_gather_into_tensor(out, flat, group=group)
    if rank != 0:
        return None
    parts = [out[r * biggest:r * biggest + (hi - lo)] for r, (lo, hi) in enumerate(sizes)]
    return torch.cat(parts, dim=0)

"""Batch sharding across GPUs (one process per GPU).

The Local Attender and the upsampler are independent per image, so the only
parallelism is splitting the image batch into contiguous shards; nothing is
exchanged while computing.  `gather_to_rank0` is the optional final gather of
the per-rank outputs to rank 0 (torch.distributed gather: NCCL over NVLink
on GPUs, gloo on CPUs); the other ranks never receive or hold the full
batch.
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


def _dense_view(t: torch.Tensor) -> tuple[torch.Tensor, bool]:
    """A contiguous view of a dense tensor, without a copy: a channels_last
    4-D tensor is viewed as NHWC.  Returns (view, was_channels_last)."""
    if t.dim() == 4 and not t.is_contiguous() and t.is_contiguous(memory_format=torch.channels_last):
        return t.permute(0, 2, 3, 1), True
    return t.contiguous(), False


def gather_to_rank0(local: torch.Tensor, n_total: int, group: Optional[dist.ProcessGroup] = None):
    """Concatenate every rank's batch slice on rank 0 in rank order.

    All ranks must call it (it is a collective): a gather to rank 0
    (NCCL over NVLink on GPUs, gloo on CPUs), so only rank 0 receives and
    holds the full batch.  Shards may differ by one item: every rank pads to
    the largest shard for the equal-size gather and rank 0 trims.
    Channels_last tensors travel as their NHWC storage (no layout copy) and
    come back channels_last.  Returns the full batch on rank 0 and None
    elsewhere."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    sizes = [shard_bounds(n_total, r, world) for r in range(world)]
    biggest = max(hi - lo for lo, hi in sizes)
    if local.shape[0] != sizes[rank][1] - sizes[rank][0]:
        raise ValueError(f"rank {rank} holds {local.shape[0]} items, expected {sizes[rank][1] - sizes[rank][0]}")
    if local.shape[0] != biggest:
        padded = torch.zeros_like(local[:1]).expand((biggest,) + tuple(local.shape[1:])).clone(
            memory_format=torch.preserve_format)
        padded[:local.shape[0]] = local
        local = padded
    src, cl = _dense_view(local)
    dst = dist.get_global_rank(group, 0) if group is not None else 0
    if rank != 0:
        dist.gather(src, gather_list=None, dst=dst, group=group)
        return None
    out = torch.empty((world * biggest,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device,
                      memory_format=torch.channels_last if cl else torch.contiguous_format)
    parts = [_dense_view(out[r * biggest:(r + 1) * biggest])[0] for r in range(world)]
    dist.gather(src, gather_list=parts, dst=dst, group=group)
    keep = [out[r * biggest:r * biggest + (hi - lo)] for r, (lo, hi) in enumerate(sizes)]
    return keep[0] if world == 1 else torch.cat(keep, dim=0)

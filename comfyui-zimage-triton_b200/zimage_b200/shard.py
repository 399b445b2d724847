"""Multi-GPU image sharding for batched generation (data parallel over images).

A batch of independent images is split across ranks (one process per GPU);
each rank runs the full step for its images, the CFG pair of an image stays on
one rank, and the final latents are gathered with one collective at the end.
There is no exchange during the steps: weights are replicated.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(n_items: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, stop) of n_items for `rank`; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def image_seeds(n_images: int, base_seed: int = 0) -> list[int]:
    """Per-image seeds independent of the sharding, so any world size reproduces the 1-GPU latents."""
    return [base_seed + i for i in range(n_images)]


def gather_images(local: torch.Tensor, n_images: int, group=None) -> torch.Tensor:
    """All-gather per-rank image tensors [n_local, ...] into [n_images, ...] on every rank.

    Uneven shards are padded to the largest shard for the collective and trimmed after.
    """
    if not dist.is_available() or not dist.is_initialized():
        return local
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    s0, s1 = shard_range(n_images, world, rank)
    if local.shape[0] != s1 - s0:
        raise ValueError(f"rank {rank} holds {local.shape[0]} images, expected {s1 - s0}")
    biggest = max(shard_range(n_images, world, r)[1] - shard_range(n_images, world, r)[0] for r in range(world))
    pad = torch.zeros((biggest,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad, group=group)
    parts = []
    for r in range(world):
        a, b = shard_range(n_images, world, r)
        parts.append(bufs[r][: b - a])
    return torch.cat(parts, 0)

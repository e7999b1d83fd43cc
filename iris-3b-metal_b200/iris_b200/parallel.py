"""Data-parallel replicas across the GPUs of one node.

The denoiser has no exchange step at 1024^2: images (each with its CFG pair)
are independent, so every rank samples its own slice of the batch with no
collective in the timed loop. Results are gathered afterwards. One process per
GPU (``torchrun``); ranks read RANK / WORLD_SIZE / LOCAL_RANK from the
environment.
"""

from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def image_shard(images: int, rank: int, world: int) -> tuple[int, int]:
    """Rank ``rank`` of ``world`` takes images ``[lo, hi)``; contiguous, balanced
    to within one image, in rank order."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(images, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def env_world() -> tuple[int, int, int]:
    """(rank, world size, local rank) from the torchrun environment (1 rank if unset)."""
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def init_process_group(backend: str, timeout_s: float = 120.0) -> None:
    """Join the default group with a short timeout, so a rank that never joins
    (or dies) ends the others' next collective with an error instead of a hang."""
    if dist.is_initialized():
        return
    rank, world, _ = env_world()
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def gather_images(local: torch.Tensor, images: int) -> torch.Tensor:
    """All-gather each rank's ``[n_r, ...]`` slice into ``[images, ...]`` (outside
    any timed region); slices may differ in length by one."""
    world = dist.get_world_size()
    counts = [image_shard(images, r, world)[1] - image_shard(images, r, world)[0] for r in range(world)]
    width = max(counts)
    padded = local.new_zeros((width, *local.shape[1:]))
    padded[: local.shape[0]] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded)
    return torch.cat([p[:c] for p, c in zip(parts, counts)], dim=0)

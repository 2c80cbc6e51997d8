# SPDX-License-Identifier: MIT OR Apache-2.0
"""Batch sharding across GPUs (one process per GPU): each rank owns a contiguous range of whole
batches, i.e. whole (batch, head) slices, and runs the op on its shard with no exchange. The
kernels' results depend on nothing but each slice's data (key-block and query-tile sizes are
constants), so a sharded run is bit-identical to the single-GPU run; NCCL is used only to gather
results when that is checked."""

from __future__ import annotations


def shard_range(batch: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) of the batches rank `rank` of `world` owns: contiguous, sizes differing by <= 1."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    base, extra = divmod(batch, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def gather_batches(tensor, world: int, dist, pad_to: int):
    """All-gather [b_r, ...] shards of possibly different sizes (padded to `pad_to` batches) and
    return the [sum b_r, ...] concatenation on every rank."""
    import torch
    b = tensor.shape[0]
    buf = torch.zeros((pad_to,) + tuple(tensor.shape[1:]), dtype=tensor.dtype,
                      device=tensor.device)
    buf[:b] = tensor
    sizes = torch.tensor([b], device=tensor.device)
    all_sizes = [torch.zeros_like(sizes) for _ in range(world)]
    dist.all_gather(all_sizes, sizes)
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf)
    return torch.cat([p[: int(n.item())] for p, n in zip(parts, all_sizes)], dim=0)

"""Data-parallel sharding of the featurization across GPUs (one process per GPU, torch.distributed).

Rays are independent, so training shards a ray batch into contiguous ranges, one per rank; every rank featurizes its
range forward and backward, and the gradient buffers are then all-reduced (the only exchange of a training step).
Inference shards a frame's Morton-ordered pixels into contiguous tiles and needs no collective. A shard passes the
batch index of its first sample as the featurizer's sample offset, so the shards draw exactly the multisample
patterns of the whole batch and N ranks reproduce one GPU's gradients up to summation order.
"""
from __future__ import annotations

import torch


def shard_range(n_items: int, world: int, rank: int) -> tuple[int, int]:
    """(start, count) of rank's contiguous share of n_items; the first n_items % world ranks get one more."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f'rank {rank} outside a world of {world}')
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def sample_offset(ray_start: int, n_intervals: int) -> int:
    """Batch index of the first sample of a shard that starts at ray ray_start (samples are ray-major)."""
    return ray_start * n_intervals


def allreduce_gradients(buffers, group=None, average: bool = True) -> None:
    """Sums (or averages) gradient buffers over the ranks in place. fp16 buffers (the NeRF grid's fine levels, scaled
    by 2^20) are divided by the world size before the sum when averaging, so that the sum of large per-rank values
    cannot overflow fp16; fp32 buffers are summed, then divided."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    for buffer in buffers:
        if world == 1:
            continue
        if average and buffer.dtype == torch.float16:
            buffer.div_(world)
            dist.all_reduce(buffer, group=group)
        else:
            dist.all_reduce(buffer, group=group)
            if average:
                buffer.div_(world)

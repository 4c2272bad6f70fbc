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


def allreduce_gradients(buffers, group=None, average: bool = True, half_wire: str = 'fp16') -> None:
    """Sums (or averages) gradient buffers over the ranks in place; on the NCCL backend the buffers of one call and one
    dtype go out as one coalesced collective (a single NCCL group). fp32 buffers are summed, then divided. fp16 buffers (the NeRF
    grid's fine levels, scaled by 2^20) when averaging: half_wire 'fp16' divides them by the world size first and sums
    in fp16 (the sum of large per-rank values cannot overflow; the partial sums round to fp16, so at 8 ranks a value
    near 40,000 can come back one fp16 spacing low), 'fp32' sums fp32 copies (twice the bytes on the wire; exact to
    fp32 before the final rounding)."""
    import torch.distributed as dist
    if half_wire not in ('fp16', 'fp32'):
        raise ValueError(f'half_wire must be fp16 or fp32, not {half_wire}')
    world = dist.get_world_size(group)
    if world == 1 or not buffers:
        return
    wire, widened = [], []
    for buffer in buffers:
        if average and buffer.dtype == torch.float16:
            if half_wire == 'fp32':
                wide = buffer.float()
                widened.append((buffer, wide))
                wire.append(wide)
            else:
                buffer.div_(world)
                wire.append(buffer)
        else:
            wire.append(buffer)
    # one coalesced collective per dtype (a coalesced all-reduce takes tensors of one type), in order of appearance
    by_dtype: dict = {}
    for t in wire:
        by_dtype.setdefault(t.dtype, []).append(t)
    coalesce = dist.get_backend(group) == 'nccl'  # gloo has no coalesced collectives
    for tensors in by_dtype.values():
        if coalesce and len(tensors) > 1:
            with dist._coalescing_manager(group, device=tensors[0].device):
                for t in tensors:
                    dist.all_reduce(t, group=group)
        else:
            for t in tensors:
                dist.all_reduce(t, group=group)
    if average:
        for buffer in buffers:
            if buffer.dtype != torch.float16:
                buffer.div_(world)
        for buffer, wide in widened:
            buffer.copy_(wide.div_(world))

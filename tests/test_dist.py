"""Data-parallel host logic on two and eight gloo ranks (CPU): ray shards partition the batch, the gradient all-reduce averages
fp32 and fp16 buffers without fp16 overflow, and the featurization gradients of two ray shards (CPU oracle, one per
rank) sum to the gradients of the whole batch."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from zipnerf_b200 import sharding


def free_port() -> int:
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def test_shard_ranges_partition_the_batch():
    for n in [0, 1, 7, 65536, 65537]:
        for world in [1, 2, 3, 8]:
            covered = []
            for rank in range(world):
                start, count = sharding.shard_range(n, world, rank)
                covered.extend(range(start, start + count))
            assert covered == list(range(n))
    with pytest.raises(ValueError):
        sharding.shard_range(10, 2, 2)
    assert sharding.sample_offset(3, 64) == 192


def _worker(rank: int, world: int, port: int, queue) -> None:
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    import datetime
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        # averaging: fp16 values whose sum would overflow (world x 40000 > 65504)
        half = torch.full((4,), 40000.0, dtype=torch.float16)
        single = torch.full((3,), float(rank + 1))
        sharding.allreduce_gradients([half, single])
        # the fp32 wire for fp16 buffers: the average of equal values is exact; mixed with fp32 buffers, each dtype is
        # one coalesced collective
        half_wide = torch.full((4,), 40000.0 + 32.0 * rank, dtype=torch.float16)
        extra = [torch.full((5,), float(rank)), torch.full((2,), 2.0 * rank)]
        sharding.allreduce_gradients([extra[0], half_wide, extra[1]], half_wire='fp32')
        assert extra[0].tolist() == [(world - 1) / 2] * 5 and extra[1].tolist() == [float(world - 1)] * 2
        mixed = [torch.full((3,), float(rank)), torch.full((4,), 100.0, dtype=torch.float16), torch.full((6,), 1.0)]
        sharding.allreduce_gradients(mixed)
        assert mixed[0].tolist() == [(world - 1) / 2] * 3 and mixed[1].tolist() == [100.0] * 4 and mixed[2].tolist() == [1.0] * 6
        # featurization gradients of this rank's ray shard with the CPU oracle
        import zf_testdata as td
        from oracle.zf_oracle import GridSpec, Oracle
        case = td.grids_case(4, 33, 5, -1)
        grid = GridSpec(case['level'], case['sizes'], case['entries'], 4, 0)
        start, count = sharding.shard_range(33, world, rank)
        rays = [np.ascontiguousarray(case[k][start:start + count]) for k in ('origins', 'directions', 'radii', 'tdist')]
        n = case['tdist'].shape[1] - 1
        grad = np.ascontiguousarray(case['grad_features'][start * n:(start + count) * n])
        g32, g16 = Oracle().backward(grid, *rays, case['seed'], grad)
        g32 = torch.from_numpy(g32.copy())
        sharding.allreduce_gradients([g32], average=False)
        queue.put((rank, half.tolist(), single.tolist(), g32.numpy(), half_wide.tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('world', [2, 8])
def test_gradient_exchange(world):
    """world 8 is the largest run of the benchmark: there the fp16 pre-division matters most (8 x 40000)."""
    ctx = mp.get_context('spawn')
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(rank, world, port, queue)) for rank in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    import zf_testdata as td
    from oracle.zf_oracle import GridSpec, Oracle
    case = td.grids_case(4, 33, 5, -1)
    grid = GridSpec(case['level'], case['sizes'], case['entries'], 4, 0)
    full32, _ = Oracle().backward(grid, *(case[k] for k in ('origins', 'directions', 'radii', 'tdist')), case['seed'],
                                  np.ascontiguousarray(case['grad_features']))
    for rank, half, single, g32, half_wide in results:
        # mean of 40000 + 32 k over k < world, rounded once to fp16 (spacing 32 there)
        expected = float(torch.tensor(40000.0 + 32.0 * (world - 1) / 2).half())
        assert half_wide == [expected] * 4, half_wide
        # no overflow; the collective's fp16 partial sums round (spacing 32 above 32768): within one spacing per add
        assert all(abs(h - 40000.0) <= 32.0 * (world - 1) for h in half), f'fp16 average overflowed or drifted: {half}'
        if world == 2:
            assert half == [40000.0] * 4  # 20000 + 20000 is exact
        assert single == [(world + 1) / 2] * 3
        # the shards' summed gradients are the whole batch's, up to fp32 summation order
        np.testing.assert_allclose(g32, full32, rtol=0, atol=1e-5 * float(np.abs(full32).max()))

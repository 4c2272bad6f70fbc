"""Inference render of one config-3 frame (zipnerf_b200/render.py, the order of the reference's
Renderer.render_image / render_rays_inference, Renderer.py:86-118,140-165): the frame assembled from two Morton shards
(the sharding of a two-GPU render, run here one after the other on one GPU) equals the one-shard frame bit for bit,
as does a render with another ray-batch size; every pixel is written, finite, and a composite of the background and
the scene's colors."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def frame(cuda_device):
    from zipnerf_b200 import render
    one = render.FrameRenderer(cuda_device)
    one.render()
    torch.cuda.synchronize()
    return one.image().clone()


def test_render_writes_every_pixel(frame):
    assert torch.isfinite(frame).all()
    assert frame.min().item() >= 0.0 and frame.max().item() <= 1.0 + 1e-6  # sigmoid colors composited over a white background
    assert frame.std().item() > 0.0


@pytest.mark.parametrize('world', [2, 3])
def test_sharded_render_equals_one_gpu_bit_for_bit(cuda_device, frame, world):
    from zipnerf_b200 import render
    shards = [render.FrameRenderer(cuda_device, rank=k, world=world, batch_rays=100_000) for k in range(world)]
    assembled = torch.full_like(frame, float('nan'))
    covered = 0
    for s in shards:
        s.rgb.fill_(float('nan'))
        s.render()
        torch.cuda.synchronize()
        pixels = s.order[s.begin:s.end]
        assembled.view(-1, 3)[pixels] = s.rgb[pixels]
        covered += s.n_rays
    assert covered == frame.numel() // 3
    assert torch.equal(assembled.view(torch.int32), frame.view(torch.int32))

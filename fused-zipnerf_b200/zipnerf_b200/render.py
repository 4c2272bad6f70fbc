"""Inference render of one frame on this backend (config 3), in the order of the reference renderer
(Renderer.render_image / render_rays_inference, Renderer.py:86-118,140-165): the frame's pixels in Morton order
(Renderer.pixel_order, Renderer.py:120-130) are cut into ray batches; per batch the camera rays and first-level
intervals (view_rays), the two proposal levels' featurization with their fused density MLPs writing raw densities only
(deterministic multisample patterns, the 32-ray interleaved thread mapping), the deterministic resampling of the next
level's intervals (composite_and_resample, seed -1), the NeRF level's featurization into packed bf16 features and the
NeRF-input tail, the NeRF MLP's inference forward and the final compositing into the frame's pixels (composite_final).

Sharding (inference shards by Morton tile with no collective): rank k of `world` renders the contiguous range
[k P / world, (k + 1) P / world) of the P Morton-ordered pixels and writes only those pixels of its frame buffer; the
host assembles the frame from the ranks' ranges. Every kernel on the path computes each ray (and each of its samples)
independently of the other rays of its batch, so the pixels a shard writes equal, bit for bit, the same pixels of a
one-GPU render.

Model: config 3's grids (config 2's: two proposal grids of 10 levels x 1 feature, 16 -> 512, table 2^21, density MLPs
of width 64; the NeRF grid of 10 levels x 4 features, 16 -> 8192, table 2^21), the reference model's NeRF MLP widths
(nerf_mlp_parameters(50, 64, 256, 256, 4)), seeded random parameters (no trained scene is available). Camera: a
1296 x 840 pinhole with a focal length of 1100 pixels on a radius-4 sphere, looking at the origin.
"""
from __future__ import annotations

import math

import torch

from zipnerf_b200 import rows, sharding, workloads

N_SAMPLES = (64, 64, 32)
DEGREE = 4
MLP_WIDTH = 64
NEAR, FAR = 0.2, 1000.0


def look_at_camera(width: int, height: int, focal: float, seed: int, device) -> tuple[torch.Tensor, torch.Tensor, float]:
    """(local_directions [height * width, 3], c2w [3, 4], pixel radius) of a pinhole camera on a radius-4 sphere looking
    at the origin (camera looks along -z in its own frame; pixel centers at +0.5; the cone radius at unit distance is
    (1 / fx + 1 / fy) / sqrt(12), utils.pixel_radius)."""
    g = torch.Generator().manual_seed(seed)
    eye = torch.nn.functional.normalize(torch.randn(3, generator=g), dim=0) * 4.0
    forward = torch.nn.functional.normalize(-eye, dim=0)
    right = torch.nn.functional.normalize(torch.linalg.cross(forward, torch.tensor([0.0, 0.0, 1.0])), dim=0)
    up = torch.linalg.cross(right, forward)
    c2w = torch.stack([right, up, -forward, eye], dim=1).float().contiguous().to(device)
    y, x = torch.meshgrid(torch.arange(height, device=device), torch.arange(width, device=device), indexing='ij')
    local = torch.stack([(x + 0.5 - width / 2) / focal, -(y + 0.5 - height / 2) / focal, -torch.ones_like(x, dtype=torch.float32)], dim=-1)
    return local.reshape(-1, 3).float().contiguous(), c2w, (2.0 / focal) / math.sqrt(12.0)


class FrameRenderer:
    """One rank's model, camera and frame buffers. render() draws this rank's share of the frame."""

    def __init__(self, device, width: int = 1296, height: int = 840, focal: float = 1100.0, seed: int = 3, batch_rays: int = 1 << 18,
                 rank: int = 0, world: int = 1) -> None:
        import ZipNeRFCudaBackend as backend
        self.backend, self.device = backend, device
        self.width, self.height, self.batch_rays = width, height, batch_rays
        g = torch.Generator(device='cpu').manual_seed(seed)
        self.levels = []
        for level in range(3):
            proposal = level < 2
            sizes, entries = workloads.grid_layout(10, 21, 16, 512 if proposal else 8192)
            f = 1 if proposal else 4
            featurizer = backend.Featurizer(level, sizes, entries, f, MLP_WIDTH if proposal else 0)
            table = ((torch.rand(sum(entries), f, generator=g) * 2 - 1) * backend.grid_max_value).to(device)
            offsets = [0]
            for e in entries:
                offsets.append(offsets[-1] + e)
            mags = torch.stack([(backend.grid_max_value ** 2 + table[a:b].square().mean()).sqrt() for a, b in zip(offsets[:-1], offsets[1:])])
            entry = {'featurizer': featurizer, 'table': table, 'magnitudes': mags.float().contiguous()}
            if proposal:
                n_out = 10 * 2
                w0 = ((torch.rand(MLP_WIDTH, n_out, generator=g) * 2 - 1) * math.sqrt(6 / n_out)).to(device)
                w1 = ((torch.rand(1, MLP_WIDTH, generator=g) * 2 - 1) * math.sqrt(6 / MLP_WIDTH)).to(device)
                b0 = ((torch.rand(MLP_WIDTH, generator=g) * 2 - 1) * 0.1).to(device)
                b1 = torch.full((1,), -1.0, device=device)
                entry['mlp'] = (w0.contiguous(), b0, w1.contiguous(), b1)
            self.levels.append(entry)
        self.mlp = backend.NerfMlp(50, 64, 256, 256, DEGREE)
        layout = self.mlp.layout
        params = torch.zeros(layout.numel)
        layout.initialize(params, g)
        for name, _, fan_in in layout.parameters:
            if fan_in == 0:
                layout.view(params, name).uniform_(-0.1, 0.1, generator=g)
        self.mlp_params = params.to(device)
        self.packed = self.mlp.pack(self.mlp_params)
        self.local_directions, self.c2w, self.radius = look_at_camera(width, height, focal, seed, device)
        self.warp = rows.ray_warp(NEAR, FAR)
        self.background = torch.ones(3, device=device)
        self.order = workloads.morton_order(width, height).to(device)
        self.n_pixels = width * height
        start, count = sharding.shard_range(self.n_pixels, world, rank)
        self.begin, self.end = start, start + count
        self.rgb = torch.zeros(self.n_pixels, 3, device=device)
        self.empty = torch.empty(0, device=device)

    @property
    def n_rays(self) -> int:
        """rays (pixels) this rank renders"""
        return self.end - self.begin

    @property
    def n_intervals(self) -> int:
        return self.n_rays * sum(N_SAMPLES)

    def render(self) -> None:
        """This rank's pixels of the frame into self.rgb (the other pixels are left as they are)."""
        b, e = self.backend, self.empty
        for start in range(self.begin, self.end, self.batch_rays):
            pixel_indices = self.order[start:min(start + self.batch_rays, self.end)]
            origins, directions, radii, encoded, sdist, tdist = b.view_rays(pixel_indices, self.local_directions, self.c2w, self.radius, DEGREE,
                                                                            N_SAMPLES[0], self.warp)
            R = pixel_indices.numel()
            for level in range(2):
                lv = self.levels[level]
                raw = torch.empty(R, N_SAMPLES[level], device=self.device)
                lv['featurizer'].forward(origins, directions, radii, tdist, -1, True, lv['table'], lv['magnitudes'], *lv['mlp'], raw, e, e, e, e)
                _, sdist, tdist = b.composite_and_resample(raw, sdist, tdist, directions, 1.0, N_SAMPLES[level + 1], -1, level + 1, self.warp)
            n = R * N_SAMPLES[2]
            features = torch.empty(n, self.mlp.n_features, dtype=torch.bfloat16, device=self.device)
            inputs = torch.empty(n, self.mlp.n_inputs, dtype=torch.bfloat16, device=self.device)
            nerf = self.levels[2]
            nerf['featurizer'].forward(origins, directions, radii, tdist, -1, True, nerf['table'], nerf['magnitudes'], e, e, e, e, e, e, features,
                                       encoded, inputs)
            outputs, _ = self.mlp.forward(features, inputs, self.packed, False)
            b.composite_final(outputs, tdist, directions, self.background, pixel_indices, self.rgb, e, e, False)

    def image(self) -> torch.Tensor:
        """The frame buffer as [height, width, 3]."""
        return self.rgb.view(self.height, self.width, 3)

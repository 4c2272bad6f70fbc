"""Workloads of the per-step kernels around the featurization (the sampling steps, the final level's losses and the
Adam step), sized like a config-2 training step: 65,536 rays; proposal levels of 64 intervals feeding 64 and 32; the
final level's 32 intervals; a ray pool of 185 views of
1296 x 840 pixels (config 4's pool, synthetic uniform-noise colors, one pinhole camera, poses on a radius-4
hemisphere); and the optimizer buffers of the reference model's default grids (Model.py:65-78,100-105): proposal grids
of 6 and 8 levels x 1 feature, the NeRF grid of 10 levels x 4 features split at its fp32 / fp16 gradient levels, the
proposal and NeRF MLP parameter buffers.

Each kernel is timed alone with CUDA events on the current stream, with the L2 flushed (a 256 MB write) before every
launch. Algorithmic bytes count every array element the kernel must read or write once.
"""
from __future__ import annotations

import math

import numpy as np
import torch

N_RAYS = 65536
FLUSH_BYTES = 256 << 20  # > the 126 MB L2


def ray_warp(near: float, far: float, power: float = -1.5, premult: float = 2.0) -> list[float]:
    """The seven float32 ray-warp constants of utils.ray_warp (utils.py:19-27)."""
    def fn(x: float) -> np.float32:
        x = np.float32(x) * np.float32(premult)
        y = np.float32(abs(power - 1) / power) * ((np.abs(x) / np.float32(abs(power - 1)) + np.float32(1)) ** np.float32(power) - np.float32(1))
        return np.copysign(y, x)
    y_max = np.nextafter(np.float32((power - 1) / power), np.float32(0)) if power < 0 else np.float32(np.inf)
    return [near, far, float(fn(near)), float(fn(far)), power, premult, float(y_max)]


WARP = ray_warp(0.2, 1000.0)


def resample_inputs(n_rays: int, n: int, device, seed: int = 11) -> dict:
    """A proposal level's raw densities N(0, 2), sorted normalized edges from 0 to 1, their metric edges, directions."""
    g = torch.Generator(device=device).manual_seed(seed)
    s = torch.sort(torch.rand(n_rays, n + 1, generator=g, device=device), dim=1).values
    s[:, 0], s[:, -1] = 0.0, 1.0
    near, far, fn_near, fn_far, p, premult, y_max = WARP
    y = s * fn_far + (1 - s) * fn_near
    yp = y.abs().clamp(max=y_max)
    t = (torch.copysign(abs(p - 1) * (torch.pow(p / abs(p - 1) * yp + 1, 1 / p) - 1), y) / premult).clamp(near, far)
    d = torch.nn.functional.normalize(torch.randn(n_rays, 3, generator=g, device=device), dim=1)
    return {'raw_density': torch.randn(n_rays, n, generator=g, device=device) * 2.0, 'sdist': s.contiguous(), 'tdist': t.contiguous(),
            'directions': d.contiguous()}


def resample_bytes(n: int, m: int) -> int:
    """per ray: raw densities, edges s and t, direction; weights, new edges s and t"""
    return 4 * n + 8 * (n + 1) + 12 + 4 * n + 8 * (m + 1)


def ray_pool(device, n_views: int = 185, width: int = 1296, height: int = 840, focal: float = 1100.0, seed: int = 4) -> dict:
    g = torch.Generator(device=device).manual_seed(seed)
    y, x = torch.meshgrid(torch.arange(height, device=device), torch.arange(width, device=device), indexing='ij')
    local = torch.stack([(x + 0.5 - width / 2) / focal, -(y + 0.5 - height / 2) / focal, -torch.ones_like(x, dtype=torch.float32)], dim=-1)
    c2w = []
    for _ in range(n_views):
        eye = torch.nn.functional.normalize(torch.randn(3, generator=g, device=device), dim=0).abs() * 4.0
        forward = torch.nn.functional.normalize(-eye, dim=0)
        right = torch.nn.functional.normalize(torch.linalg.cross(forward, torch.tensor([0.0, 0.0, 1.0], device=device)), dim=0)
        up = torch.linalg.cross(right, forward)
        c2w.append(torch.stack([right, up, -forward, eye], dim=1))
    n_pixels = width * height
    return {'view_offsets': torch.arange(n_views + 1, device=device, dtype=torch.int64) * n_pixels,
            'view_cameras': torch.zeros(n_views, dtype=torch.int32, device=device),
            'camera_offsets': torch.tensor([0, n_pixels], dtype=torch.int64, device=device),
            'local_directions': local.reshape(-1, 3).float().contiguous(), 'c2w': torch.stack(c2w).float().contiguous(),
            'camera_radii': torch.tensor([(2.0 / focal) / math.sqrt(12.0)], device=device),
            'pool_rgb': torch.randint(0, 256, (n_views * n_pixels, 3), generator=g, device=device, dtype=torch.uint8)}


def new_rays_bytes(n_samples: int, width: int) -> int:
    """per ray: the pixel's color and camera direction read; origin, direction, radius, color, encoding, edges written"""
    return 3 + 12 + 12 + 12 + 4 + 12 + 2 * width + 8 * (n_samples + 1)


def final_inputs(device, n_rays: int = N_RAYS, seed: int = 13) -> dict:
    """A training step's final-level inputs: rays initialized and resampled through both proposal levels (64, 64, 32
    intervals) by the sampling kernels, raw proposal densities N(0, 2), NeRF outputs N(0, 2) in bf16, random targets."""
    from zipnerf_b200 import capi
    g = torch.Generator(device=device).manual_seed(seed)
    d = torch.nn.functional.normalize(torch.randn(n_rays, 3, generator=g, device=device), dim=1).contiguous()
    _, s, t = capi.initialize_rays(seed, d, 4, 64, WARP)
    proposals = []
    for level, (n_next, blur) in enumerate(((64, 0.03), (32, 0.003)), start=1):
        raw = torch.randn(n_rays, s.shape[1] - 1, generator=g, device=device) * 2.0
        w, s_next, t_next = capi.composite_and_resample(raw, s, t, d, 0.5, n_next, seed, level, WARP)
        proposals.append({'raw_density': raw, 'sdist': s, 'tdist': t, 'weights': w, 'interlevel_weight': 0.01, 'interlevel_blur': blur})
        s, t = s_next, t_next
    outputs = torch.randn(n_rays, 32, 8, generator=g, device=device) * 2.0
    outputs[..., 4:] = 0.0
    return {'nerf_outputs': outputs.to(torch.bfloat16).contiguous(), 'sdist': s, 'tdist': t, 'proposals': proposals, 'directions': d, 'seed': seed,
            'rgb_target': torch.rand(n_rays, 3, generator=g, device=device)}


def final_bytes(n: int = 32, proposal_intervals=(64, 64)) -> int:
    """per ray: the NeRF outputs read (4 of 8 values per interval), their gradient rows written (8 values), edges s and
    t, direction, target; per proposal level its raw densities, edges, weights read and its gradient written"""
    return 8 * n + 16 * n + 8 * (n + 1) + 12 + 12 + sum(4 * m + 8 * (m + 1) + 4 * m + 4 * m for m in proposal_intervals)


LOSS_ARGS = (0.001, 0.01, -0.25, 10000.0)  # charbonnier padding, distortion weight, power, premult (Trainer.py:24-33)


def adam_layout() -> list[dict]:
    """The optimizer buffers of the reference trainer (Trainer.py:44-57) for the model's default grids: numel, level
    offsets (elements), fp16 gradients, gradient scale."""
    def grid(n_levels: int, features: int):
        sizes = [16 * 2 ** level for level in range(n_levels)]
        entries = [min(s ** 3, 2 ** 21) for s in sizes]
        return entries, features
    buffers = []
    for n_levels in (6, 8):
        entries, f = grid(n_levels, 1)
        buffers.append({'numel': sum(entries) * f, 'offsets': [int(v) * f for v in np.cumsum([0] + entries)], 'half': False, 'scale': 1.0})
    entries, f = grid(10, 4)
    n_fp32 = sum(1 for e in entries if e < 2 ** 20)
    fp32, fp16 = entries[:n_fp32], entries[n_fp32:]
    buffers.append({'numel': sum(fp32) * f, 'offsets': [int(v) * f for v in np.cumsum([0] + fp32)], 'half': False, 'scale': 2.0 ** 20})
    buffers.append({'numel': sum(fp16) * f, 'offsets': [int(v) * f for v in np.cumsum([0] + fp16)], 'half': True, 'scale': 2.0 ** 20})
    # proposal MLPs (64 x (L (1 + 1)) + 64 + 64 + 1 each, padded to 4) and the NeRF MLP (nerf_mlp.cu:440-455)
    buffers.append({'numel': 2052, 'offsets': [], 'half': False, 'scale': 1.0})
    buffers.append({'numel': 227556, 'offsets': [], 'half': False, 'scale': 1.0})
    return buffers


def adam_inputs(device, seed: int = 5):
    g = torch.Generator(device=device).manual_seed(seed)
    layout = adam_layout()
    params = [(torch.rand(b['numel'], generator=g, device=device) * 2 - 1) * 1e-5 for b in layout]
    grads = [(torch.randn(b['numel'], generator=g, device=device) * 1e-6 * b['scale']).to(torch.float16 if b['half'] else torch.float32)
             for b in layout]
    n_levels = sum(max(len(b['offsets']) - 1, 0) for b in layout)
    return layout, params, grads, n_levels


def adam_bytes(layout) -> int:
    """per parameter: parameter, both moments read and written, gradient read and zeroed"""
    return sum(b['numel'] * (24 + (4 if b['half'] else 8)) for b in layout)


class LaunchTimer:
    """CUDA-event time of single launches on the current stream, each after an L2 flush."""

    def __init__(self, device) -> None:
        self.flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=device)
        self.start, self.end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def __call__(self, launch, iters: int = 10, warmup: int = 3) -> float:
        times = []
        for i in range(warmup + iters):
            self.flush.zero_()
            self.start.record()
            launch()
            self.end.record()
            self.end.synchronize()
            if i >= warmup:
                times.append(self.start.elapsed_time(self.end))
        return float(np.median(times))

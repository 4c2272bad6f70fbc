"""Seeded synthetic inputs of the featurization workloads (the Mip-NeRF 360 scenes the reference trains on are not
available, so these stand in for them with the reference's shapes, sizes and value ranges).

Each workload is a list of ``Level`` entries: the featurizer layout of one sampling level (as ``Model.HashGrid`` builds
it, Model.py:17-24) plus its rays and interval endpoints. All tensors are generated with ``torch.Generator`` on the
CPU (reproducible for a given seed) and moved to the requested device.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

GRID_MAX_VALUE = 1e-4 / 10.0  # hash_init_range / precondition_scaling (zipnerf_config.h:8-9, bindings.cu:14)
ENCODED_WIDTH = 32  # direction_block_width(4) (zipnerf_config.h:18)
NERF_INPUTS_WIDTH = 96  # NeRF MLP inputs: 64 hidden features + the encoded direction block


def grid_layout(n_levels: int, log2_hashmap_size: int, base_resolution: int, finest_resolution: int):
    """Level sizes and entries of a hash grid with geometric resolutions (Model.py:19-21)."""
    scale = (finest_resolution / base_resolution) ** (1.0 / (n_levels - 1)) if n_levels > 1 else 1.0
    sizes = [round(base_resolution * scale ** level) for level in range(n_levels)]
    entries = [min(size ** 3, 2 ** log2_hashmap_size) for size in sizes]
    return sizes, entries


def power_ladder_inverse_warp(s: torch.Tensor, near: float, far: float, p: float = -1.5, premult: float = 2.0) -> torch.Tensor:
    """Normalized ray distance s in [0, 1] -> metric distance t (utils.ray_warp, ray_ops.cuh:20-33), in float32."""
    def fn(x: float) -> float:
        x = x * premult
        y = abs(p - 1) / p * ((abs(x) / abs(p - 1) + 1) ** p - 1)
        return math.copysign(y, x)
    fn_near, fn_far = fn(near), fn(far)
    y_max = math.nextafter((p - 1) / p, 0.0) if p < 0 else math.inf
    y = s * fn_far + (1.0 - s) * fn_near
    yp = y.abs().clamp(max=y_max) if p < 0 else y.abs()
    x = torch.copysign(abs(p - 1) * (torch.pow(p / abs(p - 1) * yp + 1.0, 1.0 / p) - 1.0), y) / premult
    return x.clamp(near, far)


def resampled_tdist(n_rays: int, n_intervals: int, generator: torch.Generator, near: float = 0.2, far: float = 1000.0,
                    n_bins: int = 64) -> torch.Tensor:
    """Interval endpoints [n_rays, n_intervals + 1] drawn from a random piecewise-constant weight per ray over the
    normalized distance (stratified inverse-CDF resampling, as sample_intervals in ray_ops.cuh:41-88), warped to
    metric distances in [near, far]."""
    logits = torch.randn(n_rays, n_bins, generator=generator) * 2.0
    weights = torch.softmax(logits, dim=1)
    cdf = torch.cat([torch.zeros(n_rays, 1), torch.cumsum(weights, dim=1).clamp(max=1.0)], dim=1)
    cdf[:, -1] = 1.0
    jitter = torch.rand(n_rays, 1, generator=generator)
    u = (torch.arange(n_intervals + 1, dtype=torch.float32)[None] + jitter) / (n_intervals + 1)
    idx = torch.searchsorted(cdf, u.contiguous(), right=True).clamp(1, n_bins)
    c0, c1 = cdf.gather(1, idx - 1), cdf.gather(1, idx)
    s = ((idx - 1).float() + ((u - c0) / (c1 - c0).clamp(min=1e-12)).clamp(0, 1)) / n_bins
    s, _ = torch.sort(s, dim=1)
    return power_ladder_inverse_warp(s, near, far).contiguous()


def random_rays(n_rays: int, generator: torch.Generator, origin_range: float = 1.0, radius: float = 1e-3):
    origins = (torch.rand(n_rays, 3, generator=generator) * 2.0 - 1.0) * origin_range
    directions = torch.nn.functional.normalize(torch.randn(n_rays, 3, generator=generator), dim=1)
    radii = torch.full((n_rays,), radius)
    return origins.contiguous(), directions.contiguous(), radii.contiguous()


@dataclass
class Level:
    """One sampling level: featurizer layout, grid parameters and the level's intervals."""
    level: int
    sizes: list
    entries: list
    n_features: int
    mlp_width: int
    tdist: torch.Tensor
    table: torch.Tensor
    scale_magnitudes: torch.Tensor
    mlp: tuple | None = None  # (w0 [W, n_out], b0 [W], w1 [1, W], b1 [1])

    @property
    def n_levels(self) -> int:
        return len(self.sizes)

    @property
    def n_output_features(self) -> int:
        return self.n_levels * (self.n_features + 1)

    @property
    def n_intervals(self) -> int:
        return self.tdist.shape[1] - 1


@dataclass
class Workload:
    name: str
    origins: torch.Tensor
    directions: torch.Tensor
    radii: torch.Tensor
    encoded_directions: torch.Tensor
    levels: list = field(default_factory=list)
    pattern_seed: int = 0

    @property
    def n_rays(self) -> int:
        return self.origins.shape[0]

    @property
    def n_intervals_total(self) -> int:
        return self.n_rays * sum(level.n_intervals for level in self.levels)

    def to(self, device) -> 'Workload':
        def move(x):
            return x.to(device) if isinstance(x, torch.Tensor) else x
        levels = [Level(l.level, l.sizes, l.entries, l.n_features, l.mlp_width, move(l.tdist), move(l.table),
                        move(l.scale_magnitudes), tuple(move(t) for t in l.mlp) if l.mlp is not None else None)
                  for l in self.levels]
        return Workload(self.name, move(self.origins), move(self.directions), move(self.radii), move(self.encoded_directions),
                        levels, self.pattern_seed)


def _grid_params(sizes, entries, n_features, generator):
    table = (torch.rand(sum(entries), n_features, generator=generator) * 2.0 - 1.0) * GRID_MAX_VALUE
    # scale feature magnitudes of Model.HashGrid.scale_feature_magnitudes (Model.py:37-40)
    offsets = [0]
    for e in entries:
        offsets.append(offsets[-1] + e)
    magnitudes = torch.stack([(GRID_MAX_VALUE ** 2 + table[a:b].square().mean()).sqrt() for a, b in zip(offsets[:-1], offsets[1:])])
    return table.contiguous(), magnitudes.float().contiguous()


def _proposal_mlp(n_out: int, width: int, generator: torch.Generator):
    """He-uniform first layer and output weights (Model.py:59-62,107-109), zero biases."""
    w0 = (torch.rand(width, n_out, generator=generator) * 2 - 1) * math.sqrt(6 / n_out)
    w1 = (torch.rand(1, width, generator=generator) * 2 - 1) * math.sqrt(6 / width)
    return w0.contiguous(), torch.zeros(width), w1.contiguous(), torch.zeros(1)


def config1(n_rays: int = 4096, seed: int = 0) -> Workload:
    """CPU-runnable case: one NeRF-style level, 10 levels x 4 features, table 2^19, resolutions 16 -> 2048, 32 sorted
    intervals per ray with endpoints uniform in [0.2, 100]."""
    g = torch.Generator().manual_seed(seed)
    origins, directions, radii = random_rays(n_rays, g)
    tdist, _ = torch.sort(torch.rand(n_rays, 33, generator=g) * (100.0 - 0.2) + 0.2, dim=1)
    sizes, entries = grid_layout(10, 19, 16, 2048)
    table, mags = _grid_params(sizes, entries, 4, g)
    encoded = torch.randn(n_rays, ENCODED_WIDTH, generator=g).bfloat16()
    return Workload('config1', origins, directions, radii, encoded, [Level(2, sizes, entries, 4, 0, tdist.contiguous(), table, mags)],
                    pattern_seed=seed)


def config2(n_rays: int = 65536, seed: int = 1, samples=(64, 64, 32)) -> Workload:
    """Paper-shape training step: two proposal levels (10 x 1 features, table 2^21, 16 -> 512, fused MLP of width
    64) and the NeRF level (10 x 4 features, table 2^21, 16 -> 8192)."""
    g = torch.Generator().manual_seed(seed)
    origins, directions, radii = random_rays(n_rays, g)
    encoded = torch.randn(n_rays, ENCODED_WIDTH, generator=g).bfloat16()
    levels = []
    for level, n in enumerate(samples[:-1]):
        sizes, entries = grid_layout(10, 21, 16, 512)
        table, mags = _grid_params(sizes, entries, 1, g)
        tdist = resampled_tdist(n_rays, n, g)
        levels.append(Level(level, sizes, entries, 1, 64, tdist, table, mags, _proposal_mlp(len(sizes) * 2, 64, g)))
    sizes, entries = grid_layout(10, 21, 16, 8192)
    table, mags = _grid_params(sizes, entries, 4, g)
    levels.append(Level(len(samples) - 1, sizes, entries, 4, 0, resampled_tdist(n_rays, samples[-1], g), table, mags))
    return Workload('config2', origins, directions, radii, encoded, levels, pattern_seed=seed)


def morton_order(width: int, height: int) -> torch.Tensor:
    """Pixel indices of a width x height image in Morton (Z) order (Renderer.pixel_order, Renderer.py:120-130)."""
    def spread(v: torch.Tensor) -> torch.Tensor:
        for shift, mask in ((8, 0x00FF00FF), (4, 0x0F0F0F0F), (2, 0x33333333), (1, 0x55555555)):
            v = (v | (v << shift)) & mask
        return v
    y, x = torch.meshgrid(torch.arange(height), torch.arange(width), indexing='ij')
    return (spread(x) | (spread(y) << 1)).flatten().argsort()


def config3(n_rays: int | None = None, seed: int = 3, width: int = 1296, height: int = 840, focal: float = 1100.0,
            samples=(64, 64, 32)) -> Workload:
    """Inference render of one frame: a pinhole camera (focal length in pixels) on a radius-4 sphere looking at the
    origin, rays of the pixels in Morton order (the first n_rays of them, all by default), deterministic patterns
    (pattern seed -1), interval endpoints from the random piecewise-constant resampling as in config 2. Grids as in
    config 2."""
    g = torch.Generator().manual_seed(seed)
    eye = torch.nn.functional.normalize(torch.randn(3, generator=g), dim=0) * 4.0
    forward = torch.nn.functional.normalize(-eye, dim=0)
    up = torch.tensor([0.0, 0.0, 1.0])
    right = torch.nn.functional.normalize(torch.linalg.cross(forward, up), dim=0)
    true_up = torch.linalg.cross(right, forward)
    order = morton_order(width, height)
    if n_rays is not None:
        order = order[:n_rays]
    px, py = (order % width).float() + 0.5, (order // width).float() + 0.5
    local = torch.stack([(px - width / 2) / focal, -(py - height / 2) / focal, torch.ones_like(px)], dim=1)
    directions = local[:, 0:1] * right + local[:, 1:2] * true_up + local[:, 2:3] * forward
    R = order.numel()
    origins = eye.expand(R, 3).contiguous()
    radii = torch.full((R,), (2.0 / focal) / math.sqrt(12.0))  # pixel_radius: (1/fx + 1/fy) / sqrt(12) (utils.py:14-16)
    encoded = torch.randn(R, ENCODED_WIDTH, generator=g).bfloat16()
    levels = []
    for level, n in enumerate(samples[:-1]):
        sizes, entries = grid_layout(10, 21, 16, 512)
        table, mags = _grid_params(sizes, entries, 1, g)
        levels.append(Level(level, sizes, entries, 1, 64, resampled_tdist(R, n, g), table, mags, _proposal_mlp(len(sizes) * 2, 64, g)))
    sizes, entries = grid_layout(10, 21, 16, 8192)
    table, mags = _grid_params(sizes, entries, 4, g)
    levels.append(Level(len(samples) - 1, sizes, entries, 4, 0, resampled_tdist(R, samples[-1], g), table, mags))
    return Workload('config3', origins, directions.contiguous(), radii, encoded, levels, pattern_seed=-1)


def config5(n_rays: int = 65536, seed: int = 5, n_intervals: int = 160) -> Workload:
    """Atomic-contention stress: origins within a 0.05-radius ball, directions within a 5 degree cone, one NeRF level
    of 12 x 4 features, table 2^22, resolutions 16 -> 16384."""
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(n_rays, 3, generator=g)
    origins = torch.nn.functional.normalize(u, dim=1) * 0.05 * torch.rand(n_rays, 1, generator=g) ** (1 / 3)
    axis = torch.tensor([0.0, 0.0, 1.0])
    cos_max = math.cos(math.radians(5.0))
    cos_t = 1.0 - torch.rand(n_rays, generator=g) * (1.0 - cos_max)
    phi = torch.rand(n_rays, generator=g) * 2 * math.pi
    sin_t = (1 - cos_t ** 2).sqrt()
    directions = torch.stack([sin_t * phi.cos(), sin_t * phi.sin(), cos_t], dim=1) * axis[2]
    radii = torch.full((n_rays,), 1e-3)
    sizes, entries = grid_layout(12, 22, 16, 16384)
    table, mags = _grid_params(sizes, entries, 4, g)
    encoded = torch.randn(n_rays, ENCODED_WIDTH, generator=g).bfloat16()
    tdist = resampled_tdist(n_rays, n_intervals, g)
    return Workload('config5', origins.contiguous(), directions.contiguous(), radii, encoded,
                    [Level(2, sizes, entries, 4, 0, tdist, table, mags)], pattern_seed=seed)


def nerf_feature_width(n_output_features: int) -> int:
    """bf16 feature row width of the NeRF MLP: n_output_features padded to a multiple of 8."""
    return (n_output_features + 7) // 8 * 8

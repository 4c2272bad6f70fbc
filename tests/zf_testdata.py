"""Deterministic inputs of the parity cases (shared by the tests and tests/golden/make_golden.py).

Every value comes from a splitmix64 counter hash and IEEE-exact float32 arithmetic (products, sums, square roots), so
the same inputs are regenerated bit for bit on any machine; grid tables of millions of rows are therefore never
stored. The cases follow the reference's differential test (tests/compare_backends.py:77-155) and the benchmark
configurations (config 1 and config 2 of the north-star description), at sizes the CPU oracle finishes in seconds.
"""
from __future__ import annotations

import numpy as np

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def splitmix64(x: np.ndarray) -> np.ndarray:
    x = (x + np.uint64(0x9E3779B97F4A7C15)) & M64
    x = ((x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & M64
    x = ((x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & M64
    return x ^ (x >> np.uint64(31))


def hash_uniform(seed: int, n: int, offset: int = 0) -> np.ndarray:
    """n float32 values in [0, 1) with 24 random bits: uniform(seed, index) of the counter hash."""
    with np.errstate(over='ignore'):
        base = splitmix64(np.array([seed], dtype=np.uint64))[0]
        idx = np.arange(offset, offset + n, dtype=np.uint64)
        h = splitmix64(idx ^ base)
    return (h >> np.uint64(40)).astype(np.float32) * np.float32(1.0 / 16777216.0)


def symmetric(seed: int, n: int, scale: float) -> np.ndarray:
    """uniform in [-scale, scale) (float32)"""
    return ((hash_uniform(seed, n) * np.float32(2.0) - np.float32(1.0)) * np.float32(scale)).astype(np.float32)


def grid_layout(n_levels: int, log2_hashmap_size: int, base: int, finest: int):
    scale = (finest / base) ** (1.0 / (n_levels - 1)) if n_levels > 1 else 1.0
    sizes = [round(base * scale ** level) for level in range(n_levels)]
    entries = [min(size ** 3, 2 ** log2_hashmap_size) for size in sizes]
    return sizes, entries


def rays(seed: int, n_rays: int, origin_scale: float = 1.0, radius_max: float = 0.01, far_first: bool = False):
    """origins in [-s, s)^3, directions normalized from [-1, 1)^3 (float32 exact ops), radii in (0, radius_max)."""
    origins = symmetric(seed, 3 * n_rays, origin_scale).reshape(n_rays, 3)
    if far_first and n_rays > 0:
        origins[0] = np.array([-10000.0, 0.0, 0.0], np.float32)  # exercises far contraction (compare_backends.py:86)
    d = symmetric(seed + 1, 3 * n_rays, 1.0).reshape(n_rays, 3)
    d[np.abs(d).sum(1) == 0] = np.float32(1.0)
    norm = np.sqrt((d * d).sum(1, dtype=np.float32)).astype(np.float32)
    directions = (d / norm[:, None]).astype(np.float32)
    radii = ((hash_uniform(seed + 2, n_rays) + np.float32(1e-3)) * np.float32(radius_max)).astype(np.float32)
    return np.ascontiguousarray(origins), np.ascontiguousarray(directions), radii


def linspace_tdist(n_rays: int, n_intervals: int, near: float, far: float) -> np.ndarray:
    step = np.float32((far - near) / n_intervals)
    t = np.float32(near) + np.arange(n_intervals + 1, dtype=np.float32) * step
    return np.ascontiguousarray(np.repeat(t[None], n_rays, axis=0).astype(np.float32))


def sorted_tdist(seed: int, n_rays: int, n_intervals: int, near: float, far: float) -> np.ndarray:
    t = hash_uniform(seed, n_rays * (n_intervals + 1)).reshape(n_rays, n_intervals + 1) * np.float32(far - near) + np.float32(near)
    return np.ascontiguousarray(np.sort(t.astype(np.float32), axis=1))


def bf16_bits(values: np.ndarray) -> np.ndarray:
    """round-to-nearest-even bf16 bit patterns of float32 values"""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (bits + np.uint64(0x7FFF) + ((bits >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    return rounded.astype(np.uint16)


def bf16_to_float(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


class Case(dict):
    """Inputs of one parity case: grid layout, rays, tables, MLP weights and upstream gradients (numpy)."""

    @property
    def name(self) -> str:
        return self['name']


def grids_case(features: int, n_rays: int, n_intervals: int, seed: int) -> Case:
    """check_grids of compare_backends.py:77-123: levels [2, 4, 128] with entries [8, 64, 2^20] (level 2 hashed,
    fp32 gradients on the first two levels), far-contraction ray 0, bf16 gradients of magnitude ~1e-5."""
    sizes, entries = [2, 4, 128], [8, 64, 1 << 20]
    key = 1000 * features + 10 * n_rays + n_intervals
    origins, directions, radii = rays(key, n_rays, origin_scale=3.0, far_first=True)
    n_out = len(sizes) * (features + 1)
    count = n_rays * n_intervals
    grad = bf16_bits(symmetric(key + 7, count * (n_out + 3), 2e-5).reshape(count, n_out + 3))
    return Case(name=f'grids_F{features}_R{n_rays}_I{n_intervals}_S{seed}', level=2, sizes=sizes, entries=entries, n_features=features,
                mlp_width=0, origins=origins, directions=directions, radii=radii, tdist=linspace_tdist(n_rays, n_intervals, 0.1, 2.5),
                seed=seed, table_seed=features, table_scale=0.01, encoded=bf16_bits(symmetric(key + 9, n_rays * 32, 1.0).reshape(n_rays, 32)),
                grad_features=grad)


def proposals_case(n_levels: int, n_rays: int, n_intervals: int, seed: int) -> Case:
    """check_proposals of compare_backends.py:126-155: F = 1, dense levels 2^(i+1), fused MLP of width 64."""
    sizes = [2 ** (i + 1) for i in range(n_levels)]
    entries = [min(2 ** (3 * (i + 1)), 4096) for i in range(n_levels)]
    key = 100000 + 1000 * n_levels + 10 * n_rays + n_intervals
    origins, directions, radii = rays(key, n_rays, origin_scale=3.0)
    width = n_levels * 2
    mlp = (symmetric(key + 3, 64 * width, 0.3).reshape(64, width), symmetric(key + 4, 64, 0.01), symmetric(key + 5, 64, 0.3).reshape(1, 64),
           symmetric(key + 6, 1, 0.01))
    count = n_rays * n_intervals
    return Case(name=f'proposals_L{n_levels}_R{n_rays}_I{n_intervals}_S{seed}', level=0, sizes=sizes, entries=entries, n_features=1,
                mlp_width=64, origins=origins, directions=directions, radii=radii, tdist=linspace_tdist(n_rays, n_intervals, 0.1, 3.0),
                seed=seed, table_seed=50 + n_levels, table_scale=0.01, mlp=mlp,
                grad_raw_density=symmetric(key + 8, count, 1.0).reshape(n_rays, n_intervals))


def config1_case(n_rays: int = 48) -> Case:
    """A ray subset of config 1: 10 levels x 4 features, table 2^19, resolutions 16 -> 2048, 32 sorted intervals in
    [0.2, 100], pattern seed 0, fp32 gradients on every level."""
    sizes, entries = grid_layout(10, 19, 16, 2048)
    origins, directions, radii = rays(11, n_rays, origin_scale=1.0, radius_max=2e-3)
    count = n_rays * 32
    return Case(name=f'config1_R{n_rays}', level=2, sizes=sizes, entries=entries, n_features=4, mlp_width=0, origins=origins,
                directions=directions, radii=radii, tdist=sorted_tdist(12, n_rays, 32, 0.2, 100.0), seed=0, table_seed=13, table_scale=1e-5,
                encoded=bf16_bits(symmetric(14, n_rays * 32, 1.0).reshape(n_rays, 32)),
                grad_features=bf16_bits(symmetric(15, count * 56, 1.0).reshape(count, 56)))


def config2_nerf_case(n_rays: int = 24) -> Case:
    """A ray subset of config 2's NeRF level: 10 x 4 features, table 2^21, resolutions 16 -> 8192 (levels 4-9 hashed,
    fp16 gradients from level 3)."""
    sizes, entries = grid_layout(10, 21, 16, 8192)
    origins, directions, radii = rays(21, n_rays, origin_scale=1.0, radius_max=2e-3)
    count = n_rays * 32
    return Case(name=f'config2nerf_R{n_rays}', level=2, sizes=sizes, entries=entries, n_features=4, mlp_width=0, origins=origins,
                directions=directions, radii=radii, tdist=sorted_tdist(22, n_rays, 32, 0.2, 1000.0), seed=1, table_seed=23, table_scale=1e-5,
                encoded=bf16_bits(symmetric(24, n_rays * 32, 1.0).reshape(n_rays, 32)),
                grad_features=bf16_bits(symmetric(25, count * 56, 1e-5).reshape(count, 56)))


def config2_proposal_case(n_rays: int = 24, level: int = 1) -> Case:
    """A ray subset of config 2's proposal levels: 10 x 1 feature, table 2^21, resolutions 16 -> 512, MLP width 64."""
    sizes, entries = grid_layout(10, 21, 16, 512)
    origins, directions, radii = rays(31, n_rays, origin_scale=1.0, radius_max=2e-3)
    n_out = 20
    mlp = (symmetric(33, 64 * n_out, (6 / n_out) ** 0.5).reshape(64, n_out), symmetric(34, 64, 0.01),
           symmetric(35, 64, (6 / 64) ** 0.5).reshape(1, 64), symmetric(36, 1, 0.01))
    return Case(name=f'config2prop_R{n_rays}_P{level}', level=level, sizes=sizes, entries=entries, n_features=1, mlp_width=64,
                origins=origins, directions=directions, radii=radii, tdist=sorted_tdist(32, n_rays, 64, 0.2, 1000.0), seed=1, table_seed=37,
                table_scale=1e-5, mlp=mlp, grad_raw_density=symmetric(38, n_rays * 64, 1e-2).reshape(n_rays, 64))


def table(case: Case) -> np.ndarray:
    rows = sum(case['entries'])
    return symmetric(case['table_seed'], rows * case['n_features'], case['table_scale']).reshape(rows, case['n_features'])


def scale_magnitudes(case: Case) -> np.ndarray:
    return (np.float32(0.03) + np.float32(0.01) * np.arange(len(case['sizes']), dtype=np.float32)).astype(np.float32)


def golden_cases() -> list:
    cases = []
    for features in [1, 2, 3, 4]:
        for n_rays, n_intervals, seed in [(1, 1, -1), (33, 5, 37), (65, 3, -1)]:
            cases.append(grids_case(features, n_rays, n_intervals, seed))
    for n_levels in [6, 8]:
        for n_rays, n_intervals in [(1, 1), (33, 5), (65, 3), (129, 32)]:
            for seed in [-1, 37]:
                cases.append(proposals_case(n_levels, n_rays, n_intervals, seed))
    cases += [config1_case(), config2_nerf_case(), config2_proposal_case(level=0), config2_proposal_case(level=1)]
    return cases

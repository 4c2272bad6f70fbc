"""Seeded inputs of the sampling steps and the Adam step (numpy, reference layouts), shared by the CPU checks, the
golden fixtures (tests/golden/make_golden_sampling.py) and the GPU parity tests.

The value ranges follow the reference's training step (Renderer.py:55-77, Trainer.py:44-57): proposal raw densities
around the MLP's output scale with a few clipped (> 89) and non-finite entries, interval edges resampled in the
normalized distance with some empty bins, unnormalized ray directions, the ray warp of near 0.2 / far 1000 with the
power ladder (-1.5, 2) of Model.py:67-68, and grids / gradients of the optimizer buffers' shapes.
"""
from __future__ import annotations

import numpy as np

from oracle.zf_step_oracle import ray_warp

WARP = ray_warp(0.2, 1000.0)
DEGREE = 4  # Model.py:77


def directions(rng: np.random.Generator, n: int) -> np.ndarray:
    d = rng.normal(size=(n, 3)).astype(np.float32)
    return (d * rng.uniform(0.5, 2.0, size=(n, 1))).astype(np.float32)


def sorted_edges(rng: np.random.Generator, n_rays: int, n: int, empty_fraction: float = 0.05) -> np.ndarray:
    """[n_rays, n + 1] sorted edges in [0, 1] from 0 to 1 with some repeated (empty) bins."""
    s = np.sort(rng.uniform(0.0, 1.0, size=(n_rays, n + 1)).astype(np.float32), axis=1)
    s[:, 0], s[:, -1] = 0.0, 1.0
    repeat = rng.uniform(size=(n_rays, n)) < empty_fraction
    for r, i in zip(*np.nonzero(repeat)):
        s[r, i + 1] = s[r, i]
    return np.maximum.accumulate(s, axis=1)


def to_metric(s: np.ndarray, warp=WARP) -> np.ndarray:
    """The inverse power ladder in float32 (ray_ops.cuh:26-33), for consistent (s, t) input pairs."""
    near, far, fn_near, fn_far, p, premult, y_max = [np.float32(v) for v in warp]
    s = s.astype(np.float32)
    y = s * fn_far + (np.float32(1) - s) * fn_near
    yp = np.minimum(np.abs(y), y_max) if p < 0 else np.abs(y)
    q = np.float32(abs(p - 1))
    x = np.copysign(q * (np.power(p / q * yp + np.float32(1), np.float32(1) / p) - np.float32(1)), y) / premult
    return np.clip(x, near, far).astype(np.float32)


def resample_case(n_rays: int, n: int, n_out: int, seed: int) -> dict:
    """Inputs of composite_and_resample: raw densities N(0, 3) with ~2 % clipped (100) and ~0.5 % NaN entries."""
    rng = np.random.default_rng(seed)
    raw = (rng.normal(size=(n_rays, n)) * 3.0).astype(np.float32)
    raw[rng.uniform(size=raw.shape) < 0.02] = 100.0
    raw[rng.uniform(size=raw.shape) < 0.005] = np.nan
    sdist = sorted_edges(rng, n_rays, n)
    return {'raw_density': raw, 'sdist': sdist, 'tdist': to_metric(sdist), 'directions': directions(rng, n_rays), 'n_samples': n_out}


def ray_pool(seed: int, sizes=((12, 9), (7, 5)), views=(0, 1, 0)) -> dict:
    """A small training-ray pool: cameras of the given (width, height) with pinhole local directions, views of those
    cameras with random rotations and positions, random 8-bit colors (the argument layout of generate_rays,
    Trainer.py:64-84)."""
    rng = np.random.default_rng(seed)
    local = []
    for w, h in sizes:
        x, y = np.meshgrid(np.arange(w) + 0.5 - w / 2, np.arange(h) + 0.5 - h / 2)
        f = 1.2 * max(w, h)
        local.append(np.stack([x / f, -y / f, -np.ones_like(x)], axis=-1).reshape(-1, 3))
    camera_offsets = np.cumsum([0] + [len(l) for l in local]).astype(np.int64)
    view_pixels = [len(local[c]) for c in views]
    view_offsets = np.cumsum([0] + view_pixels).astype(np.int64)
    c2w = []
    for _ in views:
        q, _ = np.linalg.qr(rng.normal(size=(3, 3)))
        c2w.append(np.concatenate([q, rng.normal(size=(3, 1)) * 2.0], axis=1))
    return {
        'view_offsets': view_offsets, 'view_cameras': np.asarray(views, np.int32), 'camera_offsets': camera_offsets,
        'local_directions': np.concatenate(local).astype(np.float32), 'c2w': np.stack(c2w).astype(np.float32),
        'camera_radii': np.array([1.0 / (1.2 * max(w, h)) / np.sqrt(3.0) for w, h in sizes], np.float32),
        'pool_rgb': rng.integers(0, 256, size=(int(view_offsets[-1]), 3), dtype=np.uint8),
    }


def adam_case(seed: int, level_sizes=((64, 512, 4096), (1024, 2048)), mlp: int = 1412, half_buffer: int = 1) -> dict:
    """Buffers of an Adam object shaped like the trainer's (Trainer.py:44-57): grid buffers with level offsets (one of
    them with fp16 gradients scaled by 2^20) and an unregularized MLP buffer; parameters U(+-1e-4), gradients with a
    few non-finite entries."""
    rng = np.random.default_rng(seed)
    params, grads, scales, offsets = [], [], [], []
    for b, sizes in enumerate(list(level_sizes) + [None]):
        numel = sum(sizes) if sizes is not None else mlp
        params.append((rng.uniform(-1e-4, 1e-4, size=numel)).astype(np.float32))
        if b == half_buffer:
            g = (rng.normal(size=numel) * 1e-6 * 2.0 ** 20).astype(np.float16)
            g[rng.uniform(size=numel) < 0.002] = np.float16(np.inf)
            grads.append(g)
            scales.append(2.0 ** 20)
        else:
            g = (rng.normal(size=numel) * 1e-5).astype(np.float32)
            g[rng.uniform(size=numel) < 0.002] = np.nan
            g[rng.uniform(size=numel) < 0.002] = np.inf
            grads.append(g)
            scales.append(1.0)
        offsets.append([int(v) for v in np.cumsum([0] + list(sizes))] if sizes is not None else [])
    return {'params': params, 'grads': grads, 'grad_scales': scales, 'level_offsets': offsets, 'reg_weight': 0.1, 'max_value': 1e-5,
            'beta1': 0.9, 'beta2': 0.99, 'eps': 1e-15}


def final_case(oracle, n_rays: int, seed: int, n_final: int = 32) -> dict:
    """Inputs of the final level (train_final / composite_final): both proposal levels' raw densities N(0, 3), their
    edges and compositing weights from the CPU restatement's own resampling chain (64 -> 64 -> n_final intervals),
    NeRF outputs N(0, 2) as bf16 bit patterns with a few NaN and infinite entries (empty samples), random targets."""
    rng = np.random.default_rng(seed)
    d = directions(rng, n_rays)
    _, s, t = oracle.initialize_rays(seed, d, DEGREE, 64, WARP)
    proposals = []
    for level, n_next in ((1, 64), (2, n_final)):
        raw = (rng.normal(size=(n_rays, s.shape[1] - 1)) * 3.0).astype(np.float32)
        w, s_next, t_next = oracle.composite_and_resample(raw, s, t, d, 0.7, n_next, seed, level, WARP)
        proposals.append({'raw_density': raw, 'sdist': s, 'tdist': t, 'weights': w, 'interlevel_weight': 0.01,
                          'interlevel_blur': (0.03, 0.003)[level - 1]})
        s, t = s_next, t_next
    outputs = (rng.normal(size=(n_rays, n_final, 8)) * 2.0).astype(np.float32)
    outputs[..., 4:] = 0.0
    outputs[rng.uniform(size=outputs.shape) < 0.002] = np.nan
    outputs[rng.uniform(size=outputs.shape) < 0.002] = np.inf
    bits = ((outputs.view(np.uint32) + 0x7fff + ((outputs.view(np.uint32) >> 16) & 1)) >> 16).astype(np.uint16)  # round to nearest even
    bits[np.isnan(outputs)] = 0x7fc0
    return {'nerf_outputs': bits, 'sdist': s, 'tdist': t, 'proposals': proposals, 'directions': d, 'seed': seed + 1000,
            'rgb_target': rng.uniform(size=(n_rays, 3)).astype(np.float32)}


LOSS_ARGS = (0.001, 0.01, -0.25, 10000.0)  # charbonnier padding, distortion weight, power, premult (Trainer.py:24-33)

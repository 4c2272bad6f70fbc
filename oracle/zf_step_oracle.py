"""ctypes binding of the CPU checkers of the sampling steps, the final level and the Adam step (TEST INFRASTRUCTURE
ONLY).

``StepOracle`` wraps the C restatement (oracle/zf_step_oracle.c -> oracle/_build/libzf_step_oracle.so); ``RefSamplingCpu``
wraps the reference's own per-ray sampling functions built for the host (oracle/ref_cpu/ref_sampling.cpp ->
oracle/_ref/libzf_ref_sampling_cpu.so, built where the reference sources exist and shipped prebuilt). Both take and
return numpy arrays with the reference's layouts; only tests and the benchmark's checker legs use them.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / '_build' / 'libzf_step_oracle.so'
REF_LIB = HERE / '_ref' / 'libzf_ref_sampling_cpu.so'

_p, _i64, _i32, _f32, _f64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_double


def build() -> None:
    subprocess.run(['make', '-s', '-C', str(HERE), 'all'], check=True)


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(_p)


def _warp(values) -> np.ndarray:
    w = np.asarray(values, np.float32)
    assert w.shape == (7,)
    return w


def ray_warp(near: float, far: float, power: float = -1.5, premult: float = 2.0) -> list[float]:
    """The seven float32 constants of utils.ray_warp (utils.py:19-27): near, far, fn(near), fn(far), power, premult,
    y_max (one float32 ulp below the asymptote (p - 1) / p for p < 0)."""
    def fn(x: float) -> np.float32:
        x = np.float32(x) * np.float32(premult)
        y = np.float32(abs(power - 1) / power) * ((np.abs(x) / np.float32(abs(power - 1)) + np.float32(1)) ** np.float32(power) - np.float32(1))
        return np.copysign(y, x)
    y_max = np.nextafter(np.float32((power - 1) / power), np.float32(0)) if power < 0 else np.float32(np.inf)
    return [near, far, float(fn(near)), float(fn(far)), power, premult, float(y_max)]


class _Sampling:
    """The sampling and final-level entry points over one library whose functions carry the given prefix."""

    def __init__(self, lib: ctypes.CDLL, prefix: str) -> None:
        self.lib, self.prefix = lib, prefix
        f = self._f
        f('direction_block_width').argtypes = [_i32]
        f('direction_block_width').restype = _i32
        f('initialize_rays').argtypes = [_i64, _p, _i32, _i32, _i32, _p, _p, _p, _p]
        f('view_rays').argtypes = [_p, _i32, _p, _p, _f32, _i32, _i32, _p, _p, _p, _p, _p, _p, _p]
        f('generate_rays').argtypes = [_i64, _i32, _p, _i32, _p, _p, _p, _p, _p, _p, _i64, _i32, _i32, _p, _p, _p, _p, _p, _p, _p, _p]
        f('sample_uniforms').argtypes = [_i64, _i64, _i64, _p]
        f('composite_and_resample').argtypes = [_p, _p, _p, _p, _i32, _i32, _f32, _i32, _i64, _i32, _p, _p, _p, _p]
        f('train_final').argtypes = [_p, _p, _p, _i32, _i32, _i32, _p, _p, _p, _p, _p, _p, _p, _p, _p, ctypes.c_uint64, _p, _f32, _f32, _f32, _f32, _p, _p]
        f('composite_final').argtypes = [_p, _p, _p, _p, _p, _i32, _i32, _p, _p, _p, _i32]
        for name in ['initialize_rays', 'view_rays', 'generate_rays', 'sample_uniforms', 'composite_and_resample', 'train_final', 'composite_final']:
            f(name).restype = None

    def _f(self, name: str):
        return getattr(self.lib, self.prefix + name)

    def direction_block_width(self, degree: int) -> int:
        return self._f('direction_block_width')(degree)

    def initialize_rays(self, seed: int, directions: np.ndarray, degree: int, n_samples: int, warp):
        d = np.ascontiguousarray(directions, np.float32)
        n = d.shape[0]
        encoded = np.zeros((n, self.direction_block_width(degree)), np.uint16)
        sdist, tdist = np.zeros((n, n_samples + 1), np.float32), np.zeros((n, n_samples + 1), np.float32)
        self._f('initialize_rays')(seed, _ptr(d), n, degree, n_samples, _ptr(_warp(warp)), _ptr(encoded), _ptr(sdist), _ptr(tdist))
        return encoded, sdist, tdist

    def view_rays(self, pixel_indices: np.ndarray, local_directions: np.ndarray, c2w: np.ndarray, radius: float, degree: int, n_samples: int, warp):
        px = np.ascontiguousarray(pixel_indices, np.int64)
        local = np.ascontiguousarray(local_directions, np.float32)
        m = np.ascontiguousarray(c2w, np.float32)
        n = px.shape[0]
        origins, directions, radii = np.zeros((n, 3), np.float32), np.zeros((n, 3), np.float32), np.zeros(n, np.float32)
        encoded = np.zeros((n, self.direction_block_width(degree)), np.uint16)
        sdist, tdist = np.zeros((n, n_samples + 1), np.float32), np.zeros((n, n_samples + 1), np.float32)
        self._f('view_rays')(_ptr(px), n, _ptr(local), _ptr(m), radius, degree, n_samples, _ptr(_warp(warp)), _ptr(origins), _ptr(directions),
                             _ptr(radii), _ptr(encoded), _ptr(sdist), _ptr(tdist))
        return origins, directions, radii, encoded, sdist, tdist

    def generate_rays(self, seed: int, n_rays: int, view_offsets, view_cameras, camera_offsets, local_directions, c2w, camera_radii, pool_rgb,
                      degree: int, n_samples: int, warp):
        vo = np.ascontiguousarray(view_offsets, np.int64)
        vc = np.ascontiguousarray(view_cameras, np.int32)
        co = np.ascontiguousarray(camera_offsets, np.int64)
        local = np.ascontiguousarray(local_directions, np.float32)
        m = np.ascontiguousarray(c2w, np.float32)
        radii_in = np.ascontiguousarray(camera_radii, np.float32)
        rgb_pool = np.ascontiguousarray(pool_rgb, np.uint8)
        n = n_rays
        origins, directions, rgb = (np.zeros((n, 3), np.float32) for _ in range(3))
        radii = np.zeros(n, np.float32)
        encoded = np.zeros((n, self.direction_block_width(degree)), np.uint16)
        sdist, tdist = np.zeros((n, n_samples + 1), np.float32), np.zeros((n, n_samples + 1), np.float32)
        self._f('generate_rays')(seed, n, _ptr(vo), vc.shape[0], _ptr(vc), _ptr(co), _ptr(local), _ptr(m), _ptr(radii_in), _ptr(rgb_pool),
                                 rgb_pool.shape[0], degree, n_samples, _ptr(_warp(warp)), _ptr(origins), _ptr(directions), _ptr(radii), _ptr(rgb),
                                 _ptr(encoded), _ptr(sdist), _ptr(tdist))
        return origins, directions, radii, rgb, encoded, sdist, tdist

    def sample_uniforms(self, seed: int, stream: int, n: int) -> np.ndarray:
        values = np.zeros(n, np.float32)
        self._f('sample_uniforms')(seed, stream, n, _ptr(values))
        return values

    def composite_and_resample(self, raw_density, sdist, tdist, directions, anneal: float, n_samples: int, seed: int, next_level: int, warp):
        raw = np.ascontiguousarray(raw_density, np.float32)
        s = np.ascontiguousarray(sdist, np.float32)
        t = np.ascontiguousarray(tdist, np.float32)
        d = np.ascontiguousarray(directions, np.float32)
        n_rays, n = raw.shape
        weights = np.zeros((n_rays, n), np.float32)
        s_next, t_next = np.zeros((n_rays, n_samples + 1), np.float32), np.zeros((n_rays, n_samples + 1), np.float32)
        self._f('composite_and_resample')(_ptr(raw), _ptr(s), _ptr(t), _ptr(d), n_rays, n, anneal, n_samples, seed, next_level, _ptr(_warp(warp)),
                                          _ptr(weights), _ptr(s_next), _ptr(t_next))
        return weights, s_next, t_next

    def train_final(self, outputs, sdist, tdist, proposals, directions, seed: int, rgb_target, charbonnier_padding: float, distortion_weight: float,
                    distortion_power: float, distortion_premult: float):
        """outputs: bf16 bit patterns uint16 [R, n, 8]; proposals: dicts of raw_density, sdist, tdist, weights (numpy),
        interlevel_weight, interlevel_blur. Returns (gradient bits uint16 [R, n, 8], [proposal gradients], loss sums
        float64 [4])."""
        out = np.ascontiguousarray(outputs, np.uint16)
        s, t = np.ascontiguousarray(sdist, np.float32), np.ascontiguousarray(tdist, np.float32)
        d, target = np.ascontiguousarray(directions, np.float32), np.ascontiguousarray(rgb_target, np.float32)
        n_rays, n1 = t.shape
        k = len(proposals)
        arrays = [{key: np.ascontiguousarray(p[key], np.float32) for key in ('raw_density', 'sdist', 'tdist', 'weights')} for p in proposals]
        grads = [np.zeros_like(a['raw_density']) for a in arrays]
        ptrs = lambda key: (_p * max(k, 1))(*[a[key].ctypes.data for a in arrays])  # noqa: E731
        n_p = (_i32 * max(k, 1))(*[a['raw_density'].shape[1] for a in arrays])
        weights = np.array([p['interlevel_weight'] for p in proposals] or [0], np.float32)
        blurs = np.array([p['interlevel_blur'] for p in proposals] or [0], np.float32)
        grad_ptrs = (_p * max(k, 1))(*[g.ctypes.data for g in grads])
        out_grad = np.zeros_like(out)
        sums = np.zeros(4, np.float64)
        self._f('train_final')(_ptr(out), _ptr(s), _ptr(t), n_rays, n1 - 1, k, n_p, ptrs('raw_density'), ptrs('sdist'), ptrs('tdist'), ptrs('weights'),
                               grad_ptrs, _ptr(weights), _ptr(blurs), _ptr(d), seed, _ptr(target), charbonnier_padding, distortion_weight,
                               distortion_power, distortion_premult, _ptr(out_grad), _ptr(sums))
        return out_grad, grads, sums

    def composite_final(self, outputs, tdist, directions, background, pixel_indices, n_pixels: int, use_median_depth: bool):
        """Returns (rgb [pixels, 3], alpha [pixels], depth [pixels]); pixels that no ray writes stay -1."""
        out = np.ascontiguousarray(outputs, np.uint16)
        t = np.ascontiguousarray(tdist, np.float32)
        d = np.ascontiguousarray(directions, np.float32)
        bg = np.ascontiguousarray(background, np.float32)
        px = np.ascontiguousarray(pixel_indices, np.int64)
        rgb, alpha, depth = np.full((n_pixels, 3), -1, np.float32), np.full(n_pixels, -1, np.float32), np.full(n_pixels, -1, np.float32)
        self._f('composite_final')(_ptr(out), _ptr(t), _ptr(d), _ptr(bg), _ptr(px), t.shape[0], t.shape[1] - 1, _ptr(rgb), _ptr(alpha), _ptr(depth),
                                   int(use_median_depth))
        return rgb, alpha, depth


class StepOracle(_Sampling):
    """The C restatement: sampling steps and Adam."""

    def __init__(self) -> None:
        if not ORACLE_LIB.exists():
            build()
        lib = ctypes.CDLL(str(ORACLE_LIB))
        super().__init__(lib, 'oracle_')
        lib.oracle_adam_buffer.argtypes = [_p, _p, _i32, _p, _p, _i64, _f64, _p, _i32, _f64, _f64, _f64, _f64, _i64, _f64, _p]
        lib.oracle_adam_buffer.restype = None

    def adam_step(self, params: list, grads: list, exp_avgs: list, exp_avg_sqs: list, grad_scales, level_offsets, reg_weight: float,
                  max_value: float, beta1: float, beta2: float, eps: float, step: int, lr: float):
        """One Adam step in place over the buffers (numpy float32 params / moments; grads float32 or float16, zeroed);
        returns (magnitudes float32 [levels], regularization float32) of the updated parameters."""
        level_sums = []
        for b, (p, g, m, v) in enumerate(zip(params, grads, exp_avgs, exp_avg_sqs)):
            offsets = np.asarray(level_offsets[b], np.int64)
            sums = np.zeros(max(len(offsets) - 1, 1), np.float64)
            half = g.dtype == np.float16
            self.lib.oracle_adam_buffer(_ptr(p), _ptr(g), int(half), _ptr(m), _ptr(v), p.size, grad_scales[b], _ptr(offsets) if len(offsets) else None,
                                        len(offsets), reg_weight, beta1, beta2, eps, step, lr, _ptr(sums))
            for i in range(len(offsets) - 1):
                level_sums.append((sums[i], offsets[i + 1] - offsets[i]))
        magnitudes = np.array([np.sqrt(max_value ** 2 + s / size) for s, size in level_sums], np.float32)
        regularization = np.float32(sum(0.5 * np.float32(reg_weight / size) * s for s, size in level_sums))
        return magnitudes, regularization


class RefSamplingCpu(_Sampling):
    """The reference's own per-ray sampling functions on the host."""

    def __init__(self) -> None:
        if not REF_LIB.exists():
            raise FileNotFoundError(f'{REF_LIB} is not built (make -C oracle ref, where the reference sources exist)')
        super().__init__(ctypes.CDLL(str(REF_LIB)), 'ref_cpu_')

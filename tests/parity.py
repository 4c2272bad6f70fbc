"""Tolerances of the CUDA kernels against the CPU oracle, shared by the GPU tests.

The kernels use the GPU's fast-math intrinsics and fused multiply-adds, exactly as the reference's kernels do; the
oracle uses IEEE libm arithmetic. Sample positions x in [0, 1]^3 therefore differ by ~1e-7, and a level of resolution
``size`` turns that into trilinear weight differences of ~size * 1e-7 (at 8192 cells per axis, fp32 positions resolve a
cell to ~1e-3 either way). Features and gradients are continuous in the positions, so they are compared with a
per-level absolute term proportional to the level's resolution plus a relative term; corner rows are compared exactly
wherever no fractional coordinate lies within the position tolerance of a cell boundary.
"""
from __future__ import annotations

import numpy as np

FEATURE_SCALE = 10.0 / 6.0
X_ATOL = 2e-6          # contracted positions in [0, 1]
SCALE_RTOL = 2e-5      # multisample radii
FEATURE_RTOL = 1e-5    # relative to the largest feature magnitude of the level (north star: 1e-5 relative in fp32)
POSITION_NOISE = 4e-6  # per-level absolute term: FEATURE_SCALE * max|table| * size * POSITION_NOISE
GRAD_RTOL = 1e-3       # grid gradients relative to the largest gradient of the level (north star: 1e-3 given fp16 order)
HALF_EPS = 2.0 ** -10


def level_feature_tolerance(sizes, n_features, table_max, reference: np.ndarray) -> np.ndarray:
    """Absolute tolerance per output column of [n, L (F + 1)] features."""
    L = len(sizes)
    ref = np.abs(reference.reshape(-1, L, n_features + 1)).max(axis=0)  # [L, F + 1]
    tol = FEATURE_RTOL * ref + (FEATURE_SCALE * table_max * np.asarray(sizes, np.float64) * POSITION_NOISE)[:, None] + 1e-12
    return tol.reshape(-1)


def assert_features_close(actual: np.ndarray, expected: np.ndarray, sizes, n_features: int, table_max: float, what: str = 'features') -> float:
    """Returns the largest error as a fraction of the tolerance."""
    tol = level_feature_tolerance(sizes, n_features, table_max, expected)
    err = np.abs(actual.astype(np.float64) - expected.astype(np.float64))
    ratio = float((err / tol).max()) if err.size else 0.0
    if ratio > 1.0:
        idx = np.unravel_index(np.argmax(err / tol), err.shape)
        raise AssertionError(f'{what}: max error {err[idx]:.3e} at {idx} exceeds tolerance {tol[idx[-1]]:.3e} '
                             f'(actual {actual[idx]:.6e}, expected {expected[idx]:.6e})')
    return ratio


def bf16_to_float(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def half_to_float(bits: np.ndarray) -> np.ndarray:
    return bits.astype(np.uint16).view(np.float16).astype(np.float32)


def assert_grad_close(actual: np.ndarray, expected: np.ndarray, offsets, sizes, n_features: int, grad_abs_max: float, half: bool,
                      row_base: int = 0, what: str = 'grad') -> float:
    """Per-level comparison of a (fp32 or fp16) gradient table [rows * F] whose first row is table row row_base."""
    a = actual.reshape(-1, n_features).astype(np.float64)
    b = expected.reshape(-1, n_features).astype(np.float64)
    worst = 0.0
    for level, size in enumerate(sizes):
        lo, hi = offsets[level] - row_base, offsets[level + 1] - row_base
        if hi <= 0 or lo >= a.shape[0]:
            continue
        lo, hi = max(lo, 0), min(hi, a.shape[0])
        bl, al = b[lo:hi], a[lo:hi]
        scale = max(float(np.abs(bl).max()), 1e-30)
        tol = GRAD_RTOL * scale + grad_abs_max * size * POSITION_NOISE + (4 * HALF_EPS * scale if half else 0.0) + 1e-30
        err = float(np.abs(al - bl).max()) if bl.size else 0.0
        worst = max(worst, err / tol)
        if err > tol:
            raise AssertionError(f'{what}: level {level} (size {size}) max error {err:.3e} exceeds {tol:.3e} (max |ref| {scale:.3e})')
    return worst

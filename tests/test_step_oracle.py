"""The CPU checkers of the sampling steps, the final level and the Adam step: the C restatement
(oracle/zf_step_oracle.c) against the golden vectors of the reference's own sampling and final-level functions
(tests/golden/make_golden_sampling.py) and against those functions built for the host where they are present, the invariants of the resampled intervals, and the Adam
restatement against an independent vectorized numpy restatement of optimizer_api.cu:43-53."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import sampling_cases as sc
from golden.make_golden_sampling import RESAMPLE_CASES, cases as golden_cases
from oracle.zf_step_oracle import REF_LIB, RefSamplingCpu, StepOracle

GOLDEN = Path(__file__).resolve().parent / 'golden' / 'sampling.npz'


@pytest.fixture(scope='module')
def step_oracle():
    return StepOracle()


def test_restatement_matches_golden_vectors(step_oracle):
    golden = np.load(GOLDEN)
    produced = golden_cases(step_oracle)
    assert sorted(produced) == sorted(golden.files)
    for key in golden.files:
        expected, actual = golden[key], produced[key]
        assert expected.dtype == actual.dtype and expected.shape == actual.shape, key
        assert np.array_equal(expected.view(np.uint8), np.ascontiguousarray(actual).view(np.uint8)), f'{key} differs from the golden vector'


@pytest.mark.skipif(not REF_LIB.exists(), reason='the reference host build is not present (make -C oracle ref)')
@pytest.mark.parametrize('n_rays,n,m,seed,anneal,jitter_seed,level', RESAMPLE_CASES + [(300, 64, 64, 12, 1.0, 4, 1), (129, 48, 17, 13, 3.0, -1, 2)])
def test_restatement_matches_reference_host_build(step_oracle, n_rays, n, m, seed, anneal, jitter_seed, level):
    ref = RefSamplingCpu()
    c = sc.resample_case(n_rays, n, m, seed)
    args = (c['raw_density'], c['sdist'], c['tdist'], c['directions'], anneal, m, jitter_seed, level, sc.WARP)
    for a, b in zip(step_oracle.composite_and_resample(*args), ref.composite_and_resample(*args)):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    d = sc.directions(np.random.default_rng(seed), n_rays)
    for s in (seed, -1):
        for a, b in zip(step_oracle.initialize_rays(s, d, sc.DEGREE, m, sc.WARP), ref.initialize_rays(s, d, sc.DEGREE, m, sc.WARP)):
            assert np.array_equal(a, b)
    pool = sc.ray_pool(seed)
    args = (seed, n_rays, pool['view_offsets'], pool['view_cameras'], pool['camera_offsets'], pool['local_directions'], pool['c2w'],
            pool['camera_radii'], pool['pool_rgb'], sc.DEGREE, m, sc.WARP)
    for a, b in zip(step_oracle.generate_rays(*args), ref.generate_rays(*args)):
        assert np.array_equal(a, b)


@pytest.mark.skipif(not REF_LIB.exists(), reason='the reference host build is not present (make -C oracle ref)')
@pytest.mark.parametrize('n_rays,seed,n_final', [(1, 3, 32), (33, 4, 32), (129, 5, 64), (64, 6, 2)])
def test_final_level_restatement_matches_reference_host_build(step_oracle, n_rays, seed, n_final):
    ref = RefSamplingCpu()
    c = sc.final_case(step_oracle, n_rays, seed, n_final)
    args = (c['nerf_outputs'], c['sdist'], c['tdist'], c['proposals'], c['directions'], c['seed'], c['rgb_target'], *sc.LOSS_ARGS)
    (ga, pa, la), (gb, pb, lb) = step_oracle.train_final(*args), ref.train_final(*args)
    assert np.array_equal(ga, gb) and all(np.array_equal(x.view(np.uint32), y.view(np.uint32)) for x, y in zip(pa, pb)) and np.array_equal(la, lb)
    assert np.isfinite(la).all() and (la > 0).all()
    # no proposal levels: the same output gradients, no interlevel term
    g0, p0, l0 = step_oracle.train_final(*args[:3], [], *args[4:])
    assert np.array_equal(g0, ga) and p0 == [] and l0[2] == 0.0
    pixels = np.random.default_rng(seed).permutation(n_rays)
    for median in (False, True):
        a = step_oracle.composite_final(c['nerf_outputs'], c['tdist'], c['directions'], np.array([0.2, 0.5, 0.9], np.float32), pixels, n_rays, median)
        b = ref.composite_final(c['nerf_outputs'], c['tdist'], c['directions'], np.array([0.2, 0.5, 0.9], np.float32), pixels, n_rays, median)
        assert all(np.array_equal(x.view(np.uint32), y.view(np.uint32)) for x, y in zip(a, b))
        assert (a[1] >= 0).all() and (a[2] >= sc.WARP[0]).all()


@pytest.mark.parametrize('n,m,anneal,jitter_seed', [(64, 64, 1.0, 3), (64, 32, 10.0, -1), (2, 64, 0.0, 5), (64, 2, 1.0, -1)])
def test_resampled_intervals_are_sorted_and_bounded(step_oracle, n, m, anneal, jitter_seed):
    c = sc.resample_case(257, n, m, 40 + n + m)
    w, s, t = step_oracle.composite_and_resample(c['raw_density'], c['sdist'], c['tdist'], c['directions'], anneal, m, jitter_seed, 1, sc.WARP)
    assert np.isfinite(w).all() and (w >= 0).all() and (w.sum(axis=1) <= 1.0 + 1e-5).all()
    assert (np.diff(s, axis=1) >= 0).all() and s.min() >= 0.0 and s.max() <= 1.0
    assert (np.diff(t, axis=1) >= 0).all() and t.min() >= sc.WARP[0] and t.max() <= sc.WARP[1]


def test_centered_first_level_is_deterministic(step_oracle):
    d = sc.directions(np.random.default_rng(2), 8)
    _, s, _ = step_oracle.initialize_rays(-1, d, sc.DEGREE, 64, sc.WARP)
    assert (s == s[0]).all()  # every ray gets the same centered pattern
    enc, _, _ = step_oracle.initialize_rays(-1, d, 0, 8, sc.WARP)
    assert enc.shape == (8, 8)  # direction_block_width(0): 3 + 1 -> 8


def numpy_adam(p, g, m, v, inv, reg, beta1, beta2, eps, lr, step):
    """optimizer_api.cu:43-53 vectorized in float32 numpy (an independent restatement)."""
    f = np.float32
    b1, b2, e, l = f(beta1), f(beta2), f(eps), f(lr)
    bc1, bc2 = f(1.0 - float(b1) ** step), f(1.0 - float(b2) ** step)
    with np.errstate(invalid='ignore', over='ignore'):
        g = g * f(inv) + reg * p
        g = np.where(np.isnan(g), f(0), np.clip(g, -np.finfo(np.float32).max, np.finfo(np.float32).max)).astype(np.float32)
        m = b1 * m + (f(1) - b1) * g
        v = b2 * v + (f(1) - b2) * g * g
        p = p - l * (m / bc1) / (np.sqrt(v / bc2) + e)
    return p.astype(np.float32), m.astype(np.float32), v.astype(np.float32)


def test_adam_restatement_matches_numpy(step_oracle):
    case = sc.adam_case(3)
    params = [p.copy() for p in case['params']]
    grads = [g.copy() for g in case['grads']]
    ms = [np.zeros_like(p) for p in params]
    vs = [np.zeros_like(p) for p in params]
    expected = [(p.copy(), np.zeros_like(p), np.zeros_like(p)) for p in params]
    for step in (1, 2, 3):
        g_in = [g.copy() for g in case['grads']]
        grads = [g.copy() for g in g_in]
        mags, reg = step_oracle.adam_step(params, grads, ms, vs, case['grad_scales'], case['level_offsets'], case['reg_weight'], case['max_value'],
                                          case['beta1'], case['beta2'], case['eps'], step, 1e-2)
        for b, g in enumerate(g_in):
            p0, m0, v0 = expected[b]
            offsets = case['level_offsets'][b]
            reg_w = np.zeros_like(p0)
            for i in range(len(offsets) - 1):
                reg_w[offsets[i]:offsets[i + 1]] = np.float32(case['reg_weight'] / (offsets[i + 1] - offsets[i]))
            gf = np.clip(g.astype(np.float32), -65504, 65504) if g.dtype == np.float16 else g
            expected[b] = numpy_adam(p0, gf, m0, v0, np.float32(1.0 / case['grad_scales'][b]), reg_w, case['beta1'], case['beta2'], case['eps'], 1e-2, step)
            assert np.array_equal(params[b], expected[b][0]) and np.array_equal(ms[b], expected[b][1]) and np.array_equal(vs[b], expected[b][2])
            assert not grads[b].any()  # zeroed for the next accumulation
            assert np.isfinite(params[b]).all()
        levels = [(p[o[i]:o[i + 1]].astype(np.float64) ** 2).mean() for p, o in zip(params, case['level_offsets']) for i in range(len(o) - 1)]
        np.testing.assert_allclose(mags, np.sqrt(case['max_value'] ** 2 + np.array(levels)), rtol=1e-6)
        np.testing.assert_allclose(reg, 0.5 * case['reg_weight'] * sum(levels), rtol=1e-5)

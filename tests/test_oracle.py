"""The C oracle against the golden vectors (outputs of the reference's own featurization code, see
tests/golden/make_golden.py): bit-exact forward outputs, corner rows, weights and sample positions; gradients equal
up to the summation order of the parameter reductions."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import zf_testdata as td
from oracle.zf_oracle import GridSpec, RefCpu

GOLDEN = Path(__file__).resolve().parent / 'golden'
CASES = {case.name: case for case in td.golden_cases()}


def load_golden(name: str):
    path = GOLDEN / f'{name}.npz'
    assert path.exists(), f'missing golden vector {path.name} (tests/golden/make_golden.py)'
    return np.load(path)


def grid_of(case) -> GridSpec:
    return GridSpec(case['level'], case['sizes'], case['entries'], case['n_features'], case['mlp_width'])


def dense_grad(rows, values, n_rows, n_features, dtype):
    out = np.zeros((n_rows, n_features), dtype)
    out[rows] = values
    return out.reshape(-1)


def run_oracle(oracle, case):
    grid = grid_of(case)
    rays = (case['origins'], case['directions'], case['radii'], case['tdist'])
    table, mags = td.table(case), td.scale_magnitudes(case)
    if case['mlp_width'] > 0:
        fwd = oracle.forward(grid, *rays, case['seed'], table, mags, mlp=case['mlp'], raw_density=True, features_float=True)
        bwd = oracle.backward_mlp(grid, *rays, case['seed'], fwd['features_float'], case['grad_raw_density'], *case['mlp'][:3])
        return grid, fwd, bwd
    width = (grid.n_output_features + 7) // 8 * 8
    fwd = oracle.forward(grid, *rays, case['seed'], table, mags, features_float=True, features_bf16_width=width,
                         encoded_directions=case['encoded'], nerf_inputs_width=96)
    g32, g16 = oracle.backward(grid, *rays, case['seed'], np.ascontiguousarray(case['grad_features']))
    return grid, fwd, {'grad_table': g32, 'grad_table_half': g16}


@pytest.mark.parametrize('name', sorted(CASES))
def test_oracle_matches_golden(oracle, name):
    case = CASES[name]
    gold = load_golden(name)
    from golden.make_golden import input_digest
    assert str(gold['digest']) == input_digest(case), 'regenerated inputs differ from the ones the golden vectors were made from'
    grid, fwd, bwd = run_oracle(oracle, case)
    for key, value in fwd.items():
        np.testing.assert_array_equal(value, gold[key], err_msg=key)
    F = grid.n_features
    if case['mlp_width'] > 0:
        np.testing.assert_array_equal(bwd['grad_table'], dense_grad(gold['grad_rows'], gold['grad_values'], grid.n_rows, F, np.float32))
        # parameter gradients: the reference's host build reduces per thread, the oracle in sample order
        for key in ['grad_w0', 'grad_b0', 'grad_w1', 'grad_b1']:
            np.testing.assert_allclose(bwd[key], gold[key], rtol=1e-5, atol=1e-6 * max(1.0, float(np.abs(gold[key]).max())), err_msg=key)
    else:
        np.testing.assert_array_equal(bwd['grad_table'], dense_grad(gold['grad_rows'], gold['grad_values'], grid.n_fp32_grad_rows, F, np.float32))
        np.testing.assert_array_equal(bwd['grad_table_half'],
                                      dense_grad(gold['grad_half_rows'], gold['grad_half_values'], grid.n_rows - grid.n_fp32_grad_rows, F, np.uint16))
    rays = (case['origins'], case['directions'], case['radii'], case['tdist'])
    for i, sample in enumerate(gold['debug_samples']):
        d = oracle.debug_interval(grid, *rays, case['seed'], int(sample))
        np.testing.assert_array_equal(d['x'], gold['debug_x'][i])
        np.testing.assert_array_equal(d['scale'], gold['debug_scale'][i])
        np.testing.assert_array_equal(d['n_groups'], gold['debug_n_groups'][i])
        np.testing.assert_array_equal(d['rows'], gold['debug_rows'][i])
        np.testing.assert_array_equal(d['weights'], gold['debug_weights'][i])


@pytest.mark.skipif(not RefCpu.available(), reason='oracle/_ref is built only where the reference sources exist')
@pytest.mark.parametrize('name', ['grids_F3_R33_I5_S37', 'config2nerf_R24', 'proposals_L8_R65_I3_S37'])
def test_oracle_matches_reference_host_build(oracle, name):
    """Live comparison with the reference's featurization header compiled for the host (when built here)."""
    case = CASES[name]
    ref = RefCpu()
    grid, fwd, bwd = run_oracle(oracle, case)
    _, fwd_ref, bwd_ref = run_oracle(ref, case)
    for key in fwd:
        np.testing.assert_array_equal(fwd[key], fwd_ref[key])
    np.testing.assert_array_equal(bwd['grad_table'], bwd_ref['grad_table'])


def test_float_conversions(oracle):
    rng = np.random.default_rng(0)
    values = np.concatenate([rng.standard_normal(10000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 5, 10000).astype(np.float32),
                             np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e-8, 5.96e-8, 2.98e-8, 6.1e-5, -3e-7], np.float32)]).astype(np.float32)
    import ctypes
    oracle.lib.zfo_float_to_half.restype = ctypes.c_uint16
    oracle.lib.zfo_float_to_half.argtypes = [ctypes.c_float]
    oracle.lib.zfo_float_to_bf16.restype = ctypes.c_uint16
    oracle.lib.zfo_float_to_bf16.argtypes = [ctypes.c_float]
    half = np.array([oracle.lib.zfo_float_to_half(float(v)) for v in values], np.uint16)
    with np.errstate(over='ignore'):  # values beyond the half range round to infinity, as the oracle's conversion does
        np.testing.assert_array_equal(half, values.astype(np.float16).view(np.uint16))
    bf16 = np.array([oracle.lib.zfo_float_to_bf16(float(v)) for v in values], np.uint16)
    np.testing.assert_array_equal(bf16, td.bf16_bits(values))


def test_layout_of_reference_configs():
    """Layout of featurizer.cu:145-155 for the benchmark grids: offsets, hashed levels and the fp32 gradient split."""
    sizes, entries = td.grid_layout(10, 21, 16, 8192)
    grid = GridSpec(2, sizes, entries, 4, 0)
    assert sizes == [16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192]
    assert grid.n_rows == 14979072 and grid.n_fp32_grad_levels == 3 and grid.n_fp32_grad_rows == 4096 + 32768 + 262144
    sizes, entries = td.grid_layout(10, 21, 16, 512)
    assert GridSpec(0, sizes, entries, 1, 64).n_rows == 10334929
    sizes, entries = td.grid_layout(12, 22, 16, 16384)
    assert GridSpec(2, sizes, entries, 4, 0).n_fp32_grad_levels == 3

"""Generates the golden vectors of tests/golden/*.npz from the reference itself.

The reference has no CPU featurization and no stored fixtures (its only test, tests/compare_backends.py, compares two
CUDA builds). These vectors are outputs of the reference's own featurization header
(ZipNeRFCudaBackend/ZipNeRFCudaBackend/featurization/rtc/featurize_common.cuh) compiled for the host by
oracle/ref_cpu (oracle/_ref/libzf_ref_cpu.so), on the deterministic inputs of tests/zf_testdata.py. They pin the C
oracle bit for bit and the CUDA kernels within their fast-math tolerances.

Run where the reference sources exist (they are needed to build oracle/_ref):
    make -C oracle all ref && python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE.parent.parent))

import zf_testdata as td  # noqa: E402
from oracle.zf_oracle import GridSpec, RefCpu  # noqa: E402

DEBUG_SAMPLES = 6


def input_digest(case: td.Case) -> str:
    """sha256 of the regenerated inputs (detects any drift of the input generator)"""
    h = hashlib.sha256()
    for key in ['origins', 'directions', 'radii', 'tdist', 'encoded', 'grad_features', 'grad_raw_density']:
        if key in case:
            h.update(np.ascontiguousarray(case[key]).tobytes())
    for array in case.get('mlp', ()):
        h.update(np.ascontiguousarray(array).tobytes())
    t = td.table(case)
    h.update(t[:4096].tobytes())
    h.update(t[-4096:].tobytes())
    h.update(td.scale_magnitudes(case).tobytes())
    return h.hexdigest()


def sparse_rows(grad: np.ndarray, n_features: int):
    rows = grad.reshape(-1, n_features)
    index = np.nonzero(np.any(rows != 0, axis=1))[0].astype(np.int64)
    return index, rows[index]


def run_case(ref: RefCpu, case: td.Case) -> dict:
    grid = GridSpec(case['level'], case['sizes'], case['entries'], case['n_features'], case['mlp_width'])
    rays = (case['origins'], case['directions'], case['radii'], case['tdist'])
    table = td.table(case)
    mags = td.scale_magnitudes(case)
    out = {'digest': np.array(input_digest(case))}
    n_samples = case['tdist'].shape[0] * (case['tdist'].shape[1] - 1)
    if case['mlp_width'] > 0:
        fwd = ref.forward(grid, *rays, case['seed'], table, mags, mlp=case['mlp'], raw_density=True, features_float=True)
        out['raw_density'] = fwd['raw_density']
        out['features_float'] = fwd['features_float']
        bwd = ref.backward_mlp(grid, *rays, case['seed'], fwd['features_float'], case['grad_raw_density'], *case['mlp'][:3])
        out['grad_rows'], out['grad_values'] = sparse_rows(bwd['grad_table'], grid.n_features)
        for key in ['grad_w0', 'grad_b0', 'grad_w1', 'grad_b1']:
            out[key] = bwd[key]
    else:
        width = (grid.n_output_features + 7) // 8 * 8
        fwd = ref.forward(grid, *rays, case['seed'], table, mags, features_float=True, features_bf16_width=width,
                          encoded_directions=case['encoded'], nerf_inputs_width=96)
        out.update(fwd)
        g32, g16 = ref.backward(grid, *rays, case['seed'], np.ascontiguousarray(case['grad_features']))
        out['grad_rows'], out['grad_values'] = sparse_rows(g32, grid.n_features)
        out['grad_half_rows'], out['grad_half_values'] = sparse_rows(g16, grid.n_features)
    samples = np.unique(np.linspace(0, n_samples - 1, DEBUG_SAMPLES).round().astype(np.int64))
    debug = [ref.debug_interval(grid, *rays, case['seed'], int(s)) for s in samples]
    out['debug_samples'] = samples
    for key in ['x', 'scale', 'n_groups', 'rows', 'weights']:
        out[f'debug_{key}'] = np.stack([d[key] for d in debug])
    return out


def main() -> None:
    ref = RefCpu()
    for case in td.golden_cases():
        np.savez_compressed(HERE / f'{case.name}.npz', **run_case(ref, case))
        print('wrote', case.name)


if __name__ == '__main__':
    main()

"""Generates tests/golden/sampling.npz: golden vectors of the sampling steps from the reference itself.

The reference has no stored fixtures for its sampling kernels. These vectors are outputs of the reference's own per-ray
sampling and final-level functions (ZipNeRFCudaBackend/ZipNeRFCudaBackend/sampling/include/ray_ops.cuh,
common/include/random.cuh) compiled for the host by oracle/ref_cpu/ref_sampling.cpp
(oracle/_ref/libzf_ref_sampling_cpu.so), on the seeded inputs of tests/sampling_cases.py. They pin the C restatement
(oracle/zf_step_oracle.c) bit for bit.

Run where the reference sources exist (they are needed to build oracle/_ref):
    make -C oracle all ref && python tests/golden/make_golden_sampling.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE.parent.parent))

import sampling_cases as sc  # noqa: E402
from oracle.zf_step_oracle import RefSamplingCpu  # noqa: E402

# (rays, intervals, new intervals, input seed, anneal, jitter seed (-1: centered), next level)
RESAMPLE_CASES = [(33, 64, 64, 7, 1.0, 11, 1), (5, 2, 2, 8, 0.0, -1, 2), (17, 64, 32, 3, 10.0, 3, 2), (1, 32, 64, 4, 0.5, 5, 1)]


def cases(ref: RefSamplingCpu) -> dict:
    out = {}
    for i, (n_rays, n, m, seed, anneal, jitter_seed, level) in enumerate(RESAMPLE_CASES):
        c = sc.resample_case(n_rays, n, m, seed)
        w, s, t = ref.composite_and_resample(c['raw_density'], c['sdist'], c['tdist'], c['directions'], anneal, m, jitter_seed, level, sc.WARP)
        out.update({f'resample{i}_weights': w, f'resample{i}_sdist': s, f'resample{i}_tdist': t})
    rng = np.random.default_rng(5)
    d = sc.directions(rng, 9)
    for name, seed in [('initialize_jitter', 5), ('initialize_centered', -1)]:
        encoded, s, t = ref.initialize_rays(seed, d, sc.DEGREE, 64, sc.WARP)
        out.update({f'{name}_encoded': encoded, f'{name}_sdist': s, f'{name}_tdist': t})
    pool = sc.ray_pool(21)
    n_local = int(pool['camera_offsets'][1])
    pixels = np.random.default_rng(6).integers(0, n_local, size=11).astype(np.int64)
    for key, value in zip(['origins', 'directions', 'radii', 'encoded', 'sdist', 'tdist'],
                          ref.view_rays(pixels, pool['local_directions'][:n_local], pool['c2w'][0], 0.01, sc.DEGREE, 64, sc.WARP)):
        out[f'view_{key}'] = value
    gen = ref.generate_rays(123, 40, pool['view_offsets'], pool['view_cameras'], pool['camera_offsets'], pool['local_directions'], pool['c2w'],
                            pool['camera_radii'], pool['pool_rgb'], sc.DEGREE, 64, sc.WARP)
    for key, value in zip(['origins', 'directions', 'radii', 'rgb', 'encoded', 'sdist', 'tdist'], gen):
        out[f'generate_{key}'] = value
    out['uniforms'] = ref.sample_uniforms(9, 2, 100)
    # the final level on inputs from the resampling chain (computed here by the reference's own functions)
    fin = sc.final_case(ref, 33, 4)
    grad, proposal_grads, sums = ref.train_final(fin['nerf_outputs'], fin['sdist'], fin['tdist'], fin['proposals'], fin['directions'], fin['seed'],
                                                 fin['rgb_target'], *sc.LOSS_ARGS)
    out.update({'final_outputs_grad': grad, 'final_proposal0_grad': proposal_grads[0], 'final_proposal1_grad': proposal_grads[1], 'final_loss_sums': sums})
    pixels = np.random.default_rng(7).permutation(33)
    for median in (False, True):
        rgb, alpha, depth = ref.composite_final(fin['nerf_outputs'], fin['tdist'], fin['directions'], np.array([0.2, 0.5, 0.9], np.float32), pixels, 33,
                                                median)
        out.update({f'composite_median{int(median)}_rgb': rgb, f'composite_median{int(median)}_alpha': alpha, f'composite_median{int(median)}_depth': depth})
    return out


def main() -> None:
    out = cases(RefSamplingCpu())
    path = HERE / 'sampling.npz'
    np.savez_compressed(path, **out)
    print(f'wrote {path.name}: {len(out)} arrays, {path.stat().st_size} bytes')


if __name__ == '__main__':
    main()

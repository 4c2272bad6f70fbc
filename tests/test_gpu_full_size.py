"""The benchmark's own step at full size against the reference's kernels: config 2 (65,536 rays x (64 + 64 + 32)
intervals, seed 1), run exactly as bench.py times it (bench.Step: the PyTorch binding ZipNeRFCudaBackend._C, the
cooperative task lists at full occupancy, the NeRF level's level passes), and through the reference's own four kernels
on the same inputs (bench.ReferenceStep, oracle/ref_cuda).

Forward outputs (raw densities, fp32 features, packed bf16 features, NeRF-input tail) are equal bit for bit; sample
positions, contraction masks, corner rows and weights of a strided subset of every level's samples are equal bit for
bit; the NeRF level's fp32 / fp16 grid gradients and the proposal levels' grid and MLP parameter gradients agree within
the reference's own repeat noise (the rule of the reference's tests/compare_backends.py:64-74)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from test_ref_cuda import as_bits, assert_intermediates_equal, noise_limited_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def steps(cuda_device):
    import bench
    from zipnerf_b200 import workloads
    why = bench.ReferenceStep.unavailable()
    if why is not None:
        pytest.skip(why)
    ours = bench.Step(workloads.config2(n_rays=65536, seed=1), cuda_device, rank=0)
    ref = bench.ReferenceStep(ours)
    ours.run()
    ref.run()
    # a second reference run into zeroed gradients: the repeat noise of its atomics
    first = {'nerf': {k: v.clone() for k, v in ref.nerf_grads.items()}, 'props': [{k: v.clone() for k, v in g.items()} for g in ref.prop_grads]}
    ref.zero_grads()
    ref.run()
    torch.cuda.synchronize()
    yield ours, ref, first
    del ours, ref, first
    torch.cuda.empty_cache()


def test_full_size_forward_bit_exact(steps):
    ours, ref, _ = steps
    for i, (a, b) in enumerate(zip(ours.prop_out, ref.prop_out)):
        for key in ('raw', 'features'):
            np.testing.assert_array_equal(as_bits(a[key]), as_bits(b[key]), err_msg=f'proposal level {i} {key}')
    for key in ('features', 'inputs'):
        np.testing.assert_array_equal(as_bits(ours.nerf_out[key]), as_bits(ref.nerf_out[key]), err_msg=f'NeRF level {key}')


def test_full_size_gradients_within_reference_noise(steps):
    ours, ref, first = steps
    noise_limited_close(ours.nerf_grads['g32'], first['nerf']['g32'], ref.nerf_grads['g32'], False, 'NeRF fp32 grid gradient')
    noise_limited_close(ours.nerf_grads['g16'].float(), first['nerf']['g16'].float(), ref.nerf_grads['g16'].float(), True,
                        'NeRF fp16 grid gradient')
    for i, (a, b, r) in enumerate(zip(ours.prop_grads, first['props'], ref.prop_grads)):
        for key in ('table', 'w0', 'b0', 'w1', 'b1'):
            noise_limited_close(a[key], b[key], r[key], False, f'proposal level {i} grad {key}')


@pytest.mark.parametrize('level', [0, 1, 2])
def test_full_size_intermediates_bit_exact(steps, level):
    """Every 61st sample of the level (~69,000 of the proposal levels' 4.2 M, ~34,000 of the NeRF level's 2.1 M),
    including contracted and uncontracted multisamples."""
    from zipnerf_b200 import capi
    ours, ref, _ = steps
    wl, lvl = ours.wl, ours.wl.levels[level]
    n = wl.n_rays * lvl.n_intervals
    samples = torch.arange(0, n, 61, dtype=torch.int32, device=ours.device)
    c = capi.CFeaturizer(lvl.level, lvl.sizes, lvl.entries, lvl.n_features, lvl.mlp_width)
    rays = (wl.origins, wl.directions, wl.radii, lvl.tdist)
    a = c.debug(*rays, wl.pattern_seed, samples)
    b = ref.featurizers[level].debug(*rays, wl.pattern_seed, samples)
    assert_intermediates_equal(a, b)
    flags = a['contracted'].cpu().numpy()
    assert flags.any() and not flags.all(), 'the subset holds contracted and uncontracted multisamples'

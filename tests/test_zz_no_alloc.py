"""The allocation-free proposal-level backward (zf_featurize_backward_mlp_no_alloc, called through the C ABI) gives the
same gradients as zf_featurize_backward_mlp, on two calls in a row, and rejects batches beyond its static workspace.

It exists for callers that must not allocate device memory while they run (a host with a fixed device-memory budget,
or a plugin inside a framework that owns all device allocations) and cannot hand the library a workspace: its
scratch is a static 32 MiB device array of the library. This file is collected last, so a run that stops at the first
failure has run every other test before it.
"""
from __future__ import annotations

import pytest
import torch

import zf_testdata as td
from zipnerf_b200 import workloads

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def capi():
    from zipnerf_b200 import capi as module
    module.load()
    return module


def within_noise(actual, reference, repeat, what: str) -> None:
    """The gradient tolerance of the GPU tests (tests/compare_backends.py:64-74 of the reference): 1e-5 relative to
    max|reference| (+2e-7), or 10x the reference path's own repeat-to-repeat noise (fp32 atomics), whichever is larger."""
    a, b, r = (x.double() for x in (actual, reference, repeat))
    scale = b.abs().max().item()
    noise = (r - b).abs().max().item()
    limit = max(2e-7 + 1e-5 * scale, 10 * noise)
    err = (a - b).abs().max().item()
    assert torch.isfinite(a).all()
    assert err <= limit, f'{what}: max error {err:.3e} > {limit:.3e}'


def proposal_level(n_rays: int, device):
    wl = workloads.config2(n_rays=n_rays, seed=3, samples=(64, 32)).to(device)
    return wl, wl.levels[0]


@pytest.mark.parametrize('n_rays', [24, 2048])
def test_no_alloc_backward_matches_allocating_backward(capi, cuda_device, n_rays):
    wl, lvl = proposal_level(n_rays, cuda_device)
    f = capi.CFeaturizer(lvl.level, lvl.sizes, lvl.entries, lvl.n_features, lvl.mlp_width)
    R, n = wl.n_rays, lvl.n_intervals
    rays = (wl.origins, wl.directions, wl.radii, lvl.tdist)
    feats = torch.empty(R * n, lvl.n_output_features, device=cuda_device)
    f.forward(*rays, wl.pattern_seed, False, lvl.table, lvl.scale_magnitudes, *lvl.mlp, raw_density=torch.empty(R, n, device=cuda_device),
              features_float=feats)
    g = torch.Generator().manual_seed(n_rays)
    grad_raw = (torch.randn(R, n, generator=g) * 1e-2).to(cuda_device)
    grad_raw[:, ::7] = 0.0  # samples without a gradient are not scattered

    def run(call):
        out = [torch.zeros(lvl.table.numel(), device=cuda_device), torch.zeros(lvl.mlp_width, lvl.n_output_features, device=cuda_device),
               torch.zeros(lvl.mlp_width, device=cuda_device), torch.zeros(lvl.mlp_width, device=cuda_device), torch.zeros(1, device=cuda_device)]
        call(*rays, wl.pattern_seed, feats, grad_raw, *lvl.mlp[:3], *out)
        torch.cuda.synchronize()
        return out

    reference, repeat = run(f.backward_mlp), run(f.backward_mlp)
    for _ in range(2):  # two calls in a row share (and overwrite) the static workspace
        result = run(f.backward_mlp_no_alloc)
        for name, a, b, r in zip(['grid', 'w0', 'b0', 'w1', 'b1'], result, reference, repeat):
            within_noise(a, b, r, f'grad {name}')


def test_no_alloc_backward_rejects_batches_beyond_its_workspace(capi, cuda_device):
    sizes, entries = td.grid_layout(10, 21, 16, 512)
    f = capi.CFeaturizer(0, sizes, entries, 1, 64)
    limit = (32 << 20) // (4 * f.n_output_features)
    n_intervals = 64
    n_rays = limit // n_intervals + 1
    tdist = torch.zeros(n_rays, n_intervals + 1, device=cuda_device)
    small = torch.zeros(8, device=cuda_device)
    with pytest.raises(capi.ZfError, match=f'at most {limit} samples'):
        f.backward_mlp_no_alloc(small, small, small, tdist, 0, small, small, small, small, small, small, small, small, small, small)


@pytest.mark.parametrize('n_intervals', [1, 64, 4096])
def test_no_alloc_backward_rejects_overflowing_ray_counts(capi, cuda_device, n_intervals):
    """Ray counts whose sample count would overflow 64 bits are rejected by the size check on the host, before any
    product is formed and before anything is launched (no tensors are needed: the arguments point nowhere)."""
    import ctypes
    sizes, entries = td.grid_layout(10, 21, 16, 512)
    f = capi.CFeaturizer(0, sizes, entries, 1, 64)
    for n_rays in ((2 ** 63 - 1) // n_intervals, (2 ** 63 - 1) // n_intervals - 1, 2 ** 62 // n_intervals + 3):
        rays = capi.zf_rays(None, None, None, None, n_rays, n_intervals, 0, 0)
        a = capi.zf_backward_mlp_args(rays, None, 0, None, 0, None, None, None, 64 * f.n_output_features, None, f.n_rows, None,
                                      64 * f.n_output_features, None, None, None, None, 0)
        with pytest.raises(capi.ZfError, match='samples of this featurizer'):
            capi.check(capi.load().zf_featurize_backward_mlp_no_alloc(f.handle, ctypes.byref(a), None))
        with pytest.raises(capi.ZfError, match='32-bit indexing'):
            capi.check(capi.load().zf_featurize_backward_mlp(f.handle, ctypes.byref(a), None))

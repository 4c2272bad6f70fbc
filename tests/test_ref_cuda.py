"""Bit-exact parity with the reference's own CUDA kernels (compiled ahead of time from the reference sources by
oracle/ref_cuda/build.py, with the reference's fast-math options), on identical inputs: forward outputs (fp32 and bf16
features, raw density, NeRF-input tail), sample positions, multisample radii, corner rows and weights are equal bit for
bit; gradients agree within the noise of atomic summation order (the rule of the reference's
tests/compare_backends.py:64-74)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.zf_ref_cuda import RefCuda, available_variants
from test_gpu_parity import case_tensors, cuda
from test_oracle import CASES

pytestmark = pytest.mark.gpu

VARIANT_OF = {}
for _name in CASES:
    if _name.startswith('grids_F'):
        VARIANT_OF[_name] = f'grids_F{_name[7]}'
    elif _name.startswith('proposals_L'):
        VARIANT_OF[_name] = f'proposals_L{_name.split("_")[1][1:]}'
    elif _name.startswith('config1'):
        VARIANT_OF[_name] = 'config1'
    elif _name.startswith('config2nerf'):
        VARIANT_OF[_name] = 'config2_nerf'
    elif _name.startswith('config2prop'):
        VARIANT_OF[_name] = f'config2_prop{_name[-1]}'

BUILT = available_variants()
needs_reference = pytest.mark.skipif(not BUILT, reason='reference kernels not built (oracle/ref_cuda/build.py, where the reference sources exist)')


@pytest.fixture(scope='module')
def capi():
    from zipnerf_b200 import capi as module
    module.load()
    return module


def forward_outputs(featurizer, case, device, interleave):
    rays, table, mags = case_tensors(case, device)
    R, n = case['tdist'].shape[0], case['tdist'].shape[1] - 1
    n_out = len(case['sizes']) * (case['n_features'] + 1)
    if case['mlp_width'] > 0:
        mlp = [cuda(m, device) for m in case['mlp']]
        out = {'raw_density': torch.full((R, n), float('nan'), device=device), 'features_float': torch.full((R * n, n_out), float('nan'), device=device)}
        featurizer.forward(*rays, case['seed'], interleave, table, mags, *mlp, raw_density=out['raw_density'], features_float=out['features_float'])
        return out
    width = (n_out + 7) // 8 * 8
    enc = cuda(case['encoded'], device, torch.bfloat16)
    # packed bf16 path (no fp32 output) as the NeRF level renders, then the generic path with fp32 features
    packed = {'features_bf16': torch.full((R * n, width), -1.0, device=device, dtype=torch.bfloat16),
              'nerf_inputs': torch.zeros(R * n, 96, device=device, dtype=torch.bfloat16)}
    featurizer.forward(*rays, case['seed'], interleave, table, mags, features_bf16=packed['features_bf16'], encoded_directions=enc,
                       nerf_inputs=packed['nerf_inputs'])
    generic = {'features_float': torch.full((R * n, n_out), float('nan'), device=device),
               'features_bf16_generic': torch.full((R * n, width), -1.0, device=device, dtype=torch.bfloat16)}
    featurizer.forward(*rays, case['seed'], interleave, table, mags, features_float=generic['features_float'],
                       features_bf16=generic['features_bf16_generic'])
    return packed | generic


def as_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16 if t.element_size() == 2 else torch.int32).cpu().numpy()


@needs_reference
@pytest.mark.parametrize('name', sorted(VARIANT_OF))
@pytest.mark.parametrize('interleave', [False, True])
def test_forward_bit_exact_with_reference_kernels(capi, cuda_device, name, interleave):
    case = CASES[name]
    ref = RefCuda(VARIANT_OF[name])
    ours = capi.CFeaturizer(case['level'], case['sizes'], case['entries'], case['n_features'], case['mlp_width'])
    a = forward_outputs(ours, case, cuda_device, interleave)
    b = forward_outputs(ref, case, cuda_device, interleave)
    torch.cuda.synchronize()
    for key in a:
        np.testing.assert_array_equal(as_bits(a[key]), as_bits(b[key]), err_msg=f'{key} differs from the reference kernel')


@needs_reference
@pytest.mark.parametrize('name', sorted(VARIANT_OF))
def test_intermediates_bit_exact_with_reference_device_code(capi, cuda_device, name):
    """Sample placement, multisample radii, contraction masks, merged corner rows (hash indices) and weights on every
    sample."""
    case = CASES[name]
    ref = RefCuda(VARIANT_OF[name])
    ours = capi.CFeaturizer(case['level'], case['sizes'], case['entries'], case['n_features'], case['mlp_width'])
    rays, _, _ = case_tensors(case, cuda_device)
    n_samples = case['tdist'].shape[0] * (case['tdist'].shape[1] - 1)
    samples = torch.arange(n_samples, dtype=torch.int32, device=cuda_device)
    assert_intermediates_equal(ours.debug(*rays, case['seed'], samples), ref.debug(*rays, case['seed'], samples))


def assert_intermediates_equal(a: dict, b: dict) -> None:
    # the reference harness's contraction flag comes from a restated position p; the contracted position formed again
    # from that p must be the reference's own x bit for bit, or the flag would not be the reference's
    np.testing.assert_array_equal(as_bits(b['x_check']), as_bits(b['x']), err_msg='restated reference position')
    for key in ['x', 'scale', 'contracted', 'n_groups', 'rows', 'weights']:
        np.testing.assert_array_equal(as_bits(a[key]) if a[key].dtype != torch.int64 else a[key].cpu().numpy(),
                                      as_bits(b[key]) if b[key].dtype != torch.int64 else b[key].cpu().numpy(), err_msg=key)


def noise_limited_close(actual, reference, repeat, half: bool, what: str):
    """compare_backends.py:64-74: four fp16 epsilons (fp16) or 1e-5 (fp32) relative to max|reference|, or 10x the
    reference's own repeat-to-repeat noise, whichever is larger."""
    a, b, r = (x.double() for x in (actual, reference, repeat))
    tolerance = 4 * torch.finfo(torch.float16).eps if half else 1e-5
    scale = b.abs().max().item() if b.numel() else 0.0
    noise = (r - b).abs().max().item() if b.numel() else 0.0
    limit = max(2e-7 + tolerance * scale, 10 * noise)
    err = (a - b).abs().max().item() if b.numel() else 0.0
    assert torch.isfinite(a).all()
    assert err <= limit, f'{what}: max error {err:.3e} > {limit:.3e} (max |ref| {scale:.3e}, repeat noise {noise:.3e})'


@needs_reference
@pytest.mark.parametrize('name', sorted(n for n in VARIANT_OF if CASES[n]['mlp_width'] == 0))
def test_backward_matches_reference_kernels(capi, cuda_device, name):
    case = CASES[name]
    ref = RefCuda(VARIANT_OF[name])
    ours = capi.CFeaturizer(case['level'], case['sizes'], case['entries'], case['n_features'], 0)
    rays, _, _ = case_tensors(case, cuda_device)
    F, split, rows = case['n_features'], ours.n_fp32_grad_rows, ours.n_rows
    grad = cuda(case['grad_features'], cuda_device, torch.bfloat16)[:, :ours.n_output_features]
    results = []
    for f in (ours, ref, ref):
        g32 = torch.zeros(split * F, device=cuda_device)
        g16 = torch.zeros((rows - split) * F, device=cuda_device, dtype=torch.float16)
        f.backward(*rays, case['seed'], grad, g32, g16)
        results.append((g32, g16))
    torch.cuda.synchronize()
    (a32, a16), (b32, b16), (r32, r16) = results
    noise_limited_close(a32, b32, r32, False, 'fp32 grid gradient')
    noise_limited_close(a16.float(), b16.float(), r16.float(), True, 'fp16 grid gradient')


@needs_reference
@pytest.mark.parametrize('name', sorted(n for n in VARIANT_OF if CASES[n]['mlp_width'] > 0))
def test_backward_mlp_matches_reference_kernels(capi, cuda_device, name):
    case = CASES[name]
    ref = RefCuda(VARIANT_OF[name])
    ours = capi.CFeaturizer(case['level'], case['sizes'], case['entries'], 1, case['mlp_width'])
    rays, table, mags = case_tensors(case, cuda_device)
    mlp = [cuda(m, cuda_device) for m in case['mlp']]
    R, n = case['tdist'].shape[0], case['tdist'].shape[1] - 1
    feats = torch.empty(R * n, ours.n_output_features, device=cuda_device)
    ours.forward(*rays, case['seed'], False, table, mags, *mlp, raw_density=torch.empty(R, n, device=cuda_device), features_float=feats)
    grad_raw = cuda(case['grad_raw_density'], cuda_device)
    W, n_out = case['mlp_width'], ours.n_output_features
    results = []
    for f in (ours, ref, ref):
        g = [torch.zeros(ours.n_rows, device=cuda_device), torch.zeros(W, n_out, device=cuda_device), torch.zeros(W, device=cuda_device),
             torch.zeros(W, device=cuda_device), torch.zeros(1, device=cuda_device)]
        f.backward_mlp(*rays, case['seed'], feats, grad_raw, *mlp[:3], *g)
        results.append(g)
    torch.cuda.synchronize()
    for i, key in enumerate(['grid', 'w0', 'b0', 'w1', 'b1']):
        noise_limited_close(results[0][i], results[1][i], results[2][i], False, f'grad {key}')


def workload_tensors(wl, lvl):
    return (wl.origins, wl.directions, wl.radii, lvl.tdist)


@needs_reference
def test_inference_render_bit_exact_with_reference_kernels(capi, cuda_device):
    """Config 3 (inference render): Morton-ordered pinhole rays of a 1296 x 840 frame (its first 16384 pixels),
    deterministic patterns, the interleaved thread mapping, forward only: raw densities of both proposal levels and the
    NeRF level's packed bf16 features and inputs equal the reference kernels' bit for bit."""
    from zipnerf_b200 import workloads
    wl = workloads.config3(n_rays=16384).to(cuda_device)
    R = wl.n_rays
    for lvl, variant in zip(wl.levels, ['config2_prop0', 'config2_prop1', 'config2_nerf']):
        ref = RefCuda(variant)
        ours = capi.CFeaturizer(lvl.level, lvl.sizes, lvl.entries, lvl.n_features, lvl.mlp_width)
        outs = []
        for f in (ours, ref):
            if lvl.mlp_width:
                raw = torch.full((R, lvl.n_intervals), float('nan'), device=cuda_device)
                f.forward(*workload_tensors(wl, lvl), -1, True, lvl.table, lvl.scale_magnitudes, *lvl.mlp, raw_density=raw)
                outs.append([raw])
            else:
                n = R * lvl.n_intervals
                bf16 = torch.full((n, 56), -1.0, device=cuda_device, dtype=torch.bfloat16)
                inputs = torch.zeros(n, 96, device=cuda_device, dtype=torch.bfloat16)
                f.forward(*workload_tensors(wl, lvl), -1, True, lvl.table, lvl.scale_magnitudes, features_bf16=bf16,
                          encoded_directions=wl.encoded_directions, nerf_inputs=inputs)
                outs.append([bf16, inputs])
        torch.cuda.synchronize()
        for a, b in zip(*outs):
            np.testing.assert_array_equal(as_bits(a), as_bits(b), err_msg=f'level {lvl.level}')


@needs_reference
def test_contention_stress_matches_reference_kernels(capi, cuda_device):
    """Config 5 (atomic contention): rays from a 0.05-radius ball within a 5 degree cone, 160 intervals, 12 x 4
    features, table 2^22; forward bit-exact, fp32 (levels 0-2) and fp16 (levels 3-11) gradients within the
    reference's own repeat noise, although coarse rows receive thousands of contributions."""
    from zipnerf_b200 import workloads
    wl = workloads.config5(n_rays=1024).to(cuda_device)
    lvl = wl.levels[0]
    ref = RefCuda('config5')
    ours = capi.CFeaturizer(lvl.level, lvl.sizes, lvl.entries, lvl.n_features, lvl.mlp_width)
    n = wl.n_rays * lvl.n_intervals
    feats = []
    for f in (ours, ref):
        out = torch.full((n, lvl.n_output_features), float('nan'), device=cuda_device)
        f.forward(*workload_tensors(wl, lvl), wl.pattern_seed, False, lvl.table, lvl.scale_magnitudes, features_float=out)
        feats.append(out)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(as_bits(feats[0]), as_bits(feats[1]))
    g = torch.Generator().manual_seed(55)
    grad = (torch.randn(n, 64, generator=g) * 1e-6).bfloat16().to(cuda_device)[:, :lvl.n_output_features]
    split, rows = ours.n_fp32_grad_rows, ours.n_rows
    results = []
    for f in (ours, ref, ref):
        g32 = torch.zeros(split * 4, device=cuda_device)
        g16 = torch.zeros((rows - split) * 4, device=cuda_device, dtype=torch.float16)
        f.backward(*workload_tensors(wl, lvl), wl.pattern_seed, grad, g32, g16)
        results.append((g32, g16))
    torch.cuda.synchronize()
    (a32, a16), (b32, b16), (r32, r16) = results
    assert b32.abs().max().item() > 0 and b16.float().abs().max().item() > 0
    noise_limited_close(a32, b32, r32, False, 'fp32 grid gradient')
    noise_limited_close(a16.float(), b16.float(), r16.float(), True, 'fp16 grid gradient')

"""Parity of the CUDA kernels (called through the C ABI, and through the ZipNeRFCudaBackend._C binding) with the
golden vectors / CPU oracle, on the reference's differential-test cases and on ray subsets of the benchmark
configurations. Tolerances: tests/parity.py."""
from __future__ import annotations


import numpy as np
import pytest
import torch

import parity
import zf_testdata as td
from test_oracle import CASES, load_golden

pytestmark = pytest.mark.gpu

GRAD_SCALE = 1048576.0


def cuda(array, device, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(array))
    if dtype is not None:
        t = t.view(dtype)
    return t.to(device)


def case_tensors(case, device):
    rays = [cuda(case[k], device) for k in ('origins', 'directions', 'radii', 'tdist')]
    table = cuda(td.table(case), device)
    mags = cuda(td.scale_magnitudes(case), device)
    return rays, table, mags


@pytest.fixture(scope='module')
def capi():
    from zipnerf_b200 import capi as module
    module.load()
    return module


@pytest.fixture(scope='module')
def backend():
    import ZipNeRFCudaBackend
    return ZipNeRFCudaBackend


def run_forward(featurizer, case, device, interleave=False, bf16_offset=0):
    """Forward with every output of the case's kind; returns numpy outputs."""
    rays, table, mags = case_tensors(case, device)
    n_samples = case['tdist'].shape[0] * (case['tdist'].shape[1] - 1)
    n_out = len(case['sizes']) * (case['n_features'] + 1)
    out = {}
    if case['mlp_width'] > 0:
        mlp = [cuda(m, device) for m in case['mlp']]
        raw = torch.empty(case['tdist'].shape[0], case['tdist'].shape[1] - 1, device=device)
        feats = torch.empty(n_samples, n_out, device=device)
        featurizer.forward(*rays, case['seed'], interleave, table, mags, *mlp, raw_density=raw, features_float=feats)
        out['raw_density'], out['features_float'] = raw, feats
    else:
        width = (n_out + 7) // 8 * 8
        storage = torch.full((n_samples * width + bf16_offset,), -1.0, device=device, dtype=torch.bfloat16)
        bf16 = storage[bf16_offset:].view(n_samples, width)
        feats = torch.empty(n_samples, n_out, device=device)
        inputs = torch.zeros(n_samples, 96, device=device, dtype=torch.bfloat16)
        enc = cuda(case['encoded'], device, torch.bfloat16)
        featurizer.forward(*rays, case['seed'], interleave, table, mags, features_float=feats, features_bf16=bf16, encoded_directions=enc,
                           nerf_inputs=inputs)
        out['features_float'], out['features_bf16'], out['nerf_inputs'] = feats, bf16, inputs
    torch.cuda.synchronize()
    return {k: (v.view(torch.int16).cpu().numpy().view(np.uint16) if v.dtype == torch.bfloat16 else v.cpu().numpy()) for k, v in out.items()}


def mlp_reference(features: np.ndarray, mlp) -> np.ndarray:
    w0, b0, w1, b1 = [m.astype(np.float64) for m in mlp]
    pre = features.astype(np.float64) @ w0.T + b0
    return (np.maximum(pre, 0.0) @ w1.reshape(-1) + b1[0]).astype(np.float64)


@pytest.mark.parametrize('name', sorted(CASES))
def test_forward_matches_oracle(capi, cuda_device, name):
    case = CASES[name]
    gold = load_golden(name)
    f = capi.CFeaturizer(case['level'], case['sizes'], case['entries'], case['n_features'], case['mlp_width'])
    out = run_forward(f, case, cuda_device)
    table_max = float(np.abs(td.table(case)).max())
    parity.assert_features_close(out['features_float'], gold['features_float'], case['sizes'], case['n_features'], table_max)
    if case['mlp_width'] > 0:
        # the MLP against a float64 evaluation on the kernel's own features (accumulation order only)
        raw_ref = mlp_reference(out['features_float'], case['mlp'])
        scale = max(float(np.abs(raw_ref).max()), 1e-6)
        np.testing.assert_allclose(out['raw_density'].reshape(-1), raw_ref, rtol=0, atol=1e-5 * scale)
    else:
        n_out = out['features_float'].shape[1]
        # bf16 features are the round-to-nearest-even of the fp32 features, zero-padded
        np.testing.assert_array_equal(out['features_bf16'][:, :n_out], td.bf16_bits(out['features_float']))
        assert not out['features_bf16'][:, n_out:].any()
        # the encoded direction tail and the bias lane are copies
        np.testing.assert_array_equal(out['nerf_inputs'][:, 64:], gold['nerf_inputs'][:, 64:])
        assert (out['nerf_inputs'][:, -1] == 0x3F80).all()
        assert not out['nerf_inputs'][:, :64].any()


@pytest.mark.parametrize('name', sorted(CASES))
def test_sample_placement_and_hashing(capi, cuda_device, name):
    """Positions within the fast-math tolerance; corner rows exact away from cell boundaries."""
    case = CASES[name]
    gold = load_golden(name)
    f = capi.CFeaturizer(case['level'], case['sizes'], case['entries'], case['n_features'], case['mlp_width'])
    rays, _, _ = case_tensors(case, cuda_device)
    samples = torch.from_numpy(gold['debug_samples'].astype(np.int32)).to(cuda_device)
    d = {k: v.cpu().numpy() for k, v in f.debug(*rays, case['seed'], samples).items()}
    np.testing.assert_allclose(d['x'], gold['debug_x'], rtol=0, atol=parity.X_ATOL)
    np.testing.assert_allclose(d['scale'], gold['debug_scale'], rtol=parity.SCALE_RTOL, atol=1e-12)
    checked = skipped = 0
    for i in range(len(gold['debug_samples'])):
        for level, size in enumerate(case['sizes']):
            p = gold['debug_x'][i].astype(np.float64) * size - 0.5
            distance = np.abs(p - np.round(p))
            if (distance < 4 * parity.X_ATOL * size + 1e-6).any():
                skipped += 1
                continue
            checked += 1
            n = gold['debug_n_groups'][i][level]
            assert d['n_groups'][i][level] == n
            np.testing.assert_array_equal(d['rows'][i][level][:n].astype(np.uint32), gold['debug_rows'][i][level][:n])
            np.testing.assert_allclose(d['weights'][i][level][:n], gold['debug_weights'][i][level][:n], rtol=1e-4,
                                       atol=3 * size * parity.X_ATOL + 1e-6)
    assert checked >= 3 * skipped, f'too many boundary cases skipped ({skipped} of {checked + skipped})'


@pytest.mark.parametrize('name', sorted(n for n in CASES if CASES[n]['mlp_width'] == 0))
def test_backward_matches_oracle(capi, cuda_device, name):
    case = CASES[name]
    gold = load_golden(name)
    f = capi.CFeaturizer(case['level'], case['sizes'], case['entries'], case['n_features'], 0)
    rays, table, _ = case_tensors(case, cuda_device)
    F = case['n_features']
    split, rows = f.n_fp32_grad_rows, f.n_rows
    g32 = torch.zeros(split * F, device=cuda_device)
    g16 = torch.zeros((rows - split) * F, device=cuda_device, dtype=torch.float16)
    n_out = f.n_output_features
    grad = cuda(case['grad_features'], cuda_device, torch.bfloat16)[:, :n_out]  # row-strided column slice
    f.backward(*rays, case['seed'], grad, g32, g16)
    torch.cuda.synchronize()
    offsets = np.cumsum([0] + case['entries'])
    g_max = float(np.abs(parity.bf16_to_float(case['grad_features'])).max()) * parity.FEATURE_SCALE * GRAD_SCALE
    exp32 = np.zeros((split, F), np.float32)
    exp32[gold['grad_rows']] = gold['grad_values']
    parity.assert_grad_close(g32.cpu().numpy(), exp32, offsets, case['sizes'], F, g_max, half=False, what='fp32 grad')
    exp16 = np.zeros((rows - split, F), np.uint16)
    exp16[gold['grad_half_rows']] = gold['grad_half_values']
    parity.assert_grad_close(g16.cpu().numpy().astype(np.float32), parity.half_to_float(exp16), offsets, case['sizes'], F, g_max, half=True,
                             row_base=split, what='fp16 grad')


@pytest.mark.parametrize('name', sorted(n for n in CASES if CASES[n]['mlp_width'] > 0))
def test_backward_mlp_matches_oracle(capi, cuda_device, oracle, name):
    case = CASES[name]
    gold = load_golden(name)
    f = capi.CFeaturizer(case['level'], case['sizes'], case['entries'], 1, case['mlp_width'])
    rays, table, _ = case_tensors(case, cuda_device)
    mlp = [cuda(m, cuda_device) for m in case['mlp']]
    feats = cuda(gold['features_float'], cuda_device)
    grad_raw = cuda(case['grad_raw_density'], cuda_device)
    W, n_out = case['mlp_width'], f.n_output_features
    grads = {'grad_table': torch.zeros(f.n_rows, device=cuda_device), 'grad_w0': torch.zeros(W, n_out, device=cuda_device),
             'grad_b0': torch.zeros(W, device=cuda_device), 'grad_w1': torch.zeros(W, device=cuda_device), 'grad_b1': torch.zeros(1, device=cuda_device)}
    f.backward_mlp(*rays, case['seed'], feats, grad_raw, *mlp[:3], grads['grad_table'], grads['grad_w0'], grads['grad_b0'], grads['grad_w1'],
                   grads['grad_b1'])
    torch.cuda.synchronize()
    offsets = np.cumsum([0] + case['entries'])
    exp = np.zeros((f.n_rows, 1), np.float32)
    exp[gold['grad_rows']] = gold['grad_values']
    w0, w1 = case['mlp'][0], case['mlp'][2]
    g_max = float(np.abs(case['grad_raw_density']).max() * np.abs(w1).sum() * np.abs(w0).max()) * parity.FEATURE_SCALE
    parity.assert_grad_close(grads['grad_table'].cpu().numpy(), exp, offsets, case['sizes'], 1, g_max, half=False, what='grid grad')
    for key in ['grad_w0', 'grad_b0', 'grad_w1', 'grad_b1']:
        a, b = grads[key].cpu().numpy().reshape(-1), gold[key].reshape(-1)
        np.testing.assert_allclose(a, b, rtol=0, atol=1e-4 * max(float(np.abs(b).max()), 1e-12), err_msg=key)


def test_level_passes_of_the_benchmark_grids(capi, cuda_device):
    """Grids larger than the L2 run their forward and backward as level passes (config 2's NeRF grid: 7 forward passes
    of one 32 MB hashed table, 2 backward passes); the proposal grids fit and take one launch, their backward two (the
    MLP kernel and the scatter)."""
    from zipnerf_b200 import workloads
    wl = workloads.config2(n_rays=32)
    prop, nerf = wl.levels[0], wl.levels[2]
    fp = capi.CFeaturizer(prop.level, prop.sizes, prop.entries, prop.n_features, prop.mlp_width)
    fn = capi.CFeaturizer(nerf.level, nerf.sizes, nerf.entries, nerf.n_features, nerf.mlp_width)
    assert [fp.launches(c) for c in ('forward', 'forward_mlp', 'backward', 'backward_mlp')] == [1, 1, 1, 2]
    assert [fn.launches(c) for c in ('forward', 'forward_mlp', 'backward', 'backward_mlp')] == [7, 0, 2, 0]


@pytest.mark.parametrize('n_levels', [7, 8])
def test_mlp_weight_loads_are_bit_identical(capi, cuda_device, oracle, n_levels):
    """The fused MLP reads its weight rows as 16-byte words when w0 is 16-byte aligned and the MLP input width a multiple
    of 4, element by element otherwise (7 levels: 14 inputs; or a w0 4 bytes off alignment). Raw density and features
    are bit-identical either way, and match the oracle and a float64 MLP."""
    from oracle.zf_oracle import GridSpec
    case = td.proposals_case(n_levels, 33, 5, 37)
    rays, table, mags = case_tensors(case, cuda_device)
    mlp = [cuda(m, cuda_device) for m in case['mlp']]
    storage = torch.empty(mlp[0].numel() + 1, device=cuda_device)
    w0_offset = storage[1:].view_as(mlp[0])
    w0_offset.copy_(mlp[0])
    f = capi.CFeaturizer(case['level'], case['sizes'], case['entries'], 1, 64)
    n_rays, n = case['tdist'].shape[0], case['tdist'].shape[1] - 1
    outs = []
    for w0 in (mlp[0], w0_offset):
        raw = torch.full((n_rays, n), float('nan'), device=cuda_device)
        feats = torch.full((n_rays * n, f.n_output_features), float('nan'), device=cuda_device)
        f.forward(*rays, case['seed'], False, table, mags, w0, *mlp[1:], raw_density=raw, features_float=feats)
        torch.cuda.synchronize()
        outs.append((raw.cpu().numpy(), feats.cpu().numpy()))
    np.testing.assert_array_equal(outs[0][0], outs[1][0])
    np.testing.assert_array_equal(outs[0][1], outs[1][1])
    grid = GridSpec(case['level'], case['sizes'], case['entries'], 1, 64)
    gold = oracle.forward(grid, *(case[k] for k in ('origins', 'directions', 'radii', 'tdist')), case['seed'], td.table(case),
                          td.scale_magnitudes(case), features_float=True)
    parity.assert_features_close(outs[0][1], gold['features_float'], case['sizes'], 1, float(np.abs(td.table(case)).max()))
    raw_ref = mlp_reference(outs[0][1], case['mlp'])
    np.testing.assert_allclose(outs[0][0].reshape(-1), raw_ref, rtol=0, atol=1e-5 * max(float(np.abs(raw_ref).max()), 1e-6))


@pytest.mark.parametrize('name', ['grids_F1_R65_I3_S-1', 'grids_F3_R33_I5_S37', 'proposals_L8_R129_I32_S37', 'config2nerf_R24'])
def test_interleave_and_layouts_are_bit_identical(capi, cuda_device, name):
    """The thread mapping (interleave) and the output layout (aligned or not) never change a result bit."""
    case = CASES[name]
    f = capi.CFeaturizer(case['level'], case['sizes'], case['entries'], case['n_features'], case['mlp_width'])
    base = run_forward(f, case, cuda_device, interleave=False)
    for variant in [dict(interleave=True), dict(bf16_offset=1), dict(interleave=True, bf16_offset=1)]:
        if 'bf16_offset' in variant and case['mlp_width'] > 0:
            continue
        other = run_forward(f, case, cuda_device, **variant)
        for key in base:
            np.testing.assert_array_equal(other[key], base[key], err_msg=f'{key} {variant}')


@pytest.mark.parametrize('name', ['grids_F4_R33_I5_S37', 'proposals_L6_R65_I3_S37', 'config2nerf_R24'])
def test_torch_binding_matches_c_abi(capi, backend, cuda_device, name):
    """ZipNeRFCudaBackend._C.Featurizer (the reference's API) and the C ABI give identical forward outputs."""
    case = CASES[name]
    f = capi.CFeaturizer(case['level'], case['sizes'], case['entries'], case['n_features'], case['mlp_width'])
    g = backend.Featurizer(case['level'], case['sizes'], case['entries'], case['n_features'], case['mlp_width'])
    assert g.n_fp32_grad_rows == f.n_fp32_grad_rows
    base = run_forward(f, case, cuda_device)
    rays, table, mags = case_tensors(case, cuda_device)
    empty = torch.empty(0, device=cuda_device)
    n_samples = case['tdist'].shape[0] * (case['tdist'].shape[1] - 1)
    if case['mlp_width'] > 0:
        mlp = [cuda(m, cuda_device) for m in case['mlp']]
        raw = torch.empty(case['tdist'].shape[0], case['tdist'].shape[1] - 1, device=cuda_device)
        feats = torch.empty(n_samples, f.n_output_features, device=cuda_device)
        g.forward(*rays, case['seed'], False, table, mags, *mlp, raw, feats, empty, empty, empty)
        np.testing.assert_array_equal(raw.cpu().numpy(), base['raw_density'])
        np.testing.assert_array_equal(feats.cpu().numpy(), base['features_float'])
    else:
        width = (f.n_output_features + 7) // 8 * 8
        bf16 = torch.empty(n_samples, width, device=cuda_device, dtype=torch.bfloat16)
        inputs = torch.zeros(n_samples, 96, device=cuda_device, dtype=torch.bfloat16)
        enc = cuda(case['encoded'], cuda_device, torch.bfloat16)
        g.forward(*rays, case['seed'], False, table, mags, empty, empty, empty, empty, empty, empty, bf16, enc, inputs)
        np.testing.assert_array_equal(bf16.view(torch.int16).cpu().numpy().view(np.uint16), base['features_bf16'])
        np.testing.assert_array_equal(inputs.view(torch.int16).cpu().numpy().view(np.uint16), base['nerf_inputs'])


def test_torch_binding_backward_and_errors(backend, cuda_device):
    case = CASES['grids_F4_R65_I3_S-1']
    g = backend.Featurizer(case['level'], case['sizes'], case['entries'], 4, 0)
    rays, table, _ = case_tensors(case, cuda_device)
    split = g.n_fp32_grad_rows
    g32 = torch.zeros(split, 4, device=cuda_device)
    g16 = torch.zeros(sum(case['entries']) - split, 4, device=cuda_device, dtype=torch.float16)
    grad = cuda(case['grad_features'], cuda_device, torch.bfloat16)[:, :g.n_output_features]
    g.backward(*rays, case['seed'], grad, g32, g16)
    torch.cuda.synchronize()
    assert g32.abs().sum().item() > 0 and g16.float().abs().sum().item() > 0
    with pytest.raises(RuntimeError, match='ZipNeRF: invalid grid gradient split'):
        g.backward(*rays, case['seed'], grad, g32[:-1], g16)
    with pytest.raises(RuntimeError, match='ZipNeRF: grad_features has an invalid layout'):
        g.backward(*rays, case['seed'], grad[:-1], g32, g16)
    with pytest.raises(RuntimeError, match='ZipNeRF: origins must be a contiguous cuda tensor'):
        g.backward(rays[0].cpu(), *rays[1:], case['seed'], grad, g32, g16)


def test_empty_batches_are_no_ops(capi, backend, cuda_device):
    case = CASES['grids_F2_R33_I5_S37']
    f = capi.CFeaturizer(case['level'], case['sizes'], case['entries'], 2, 0)
    _, table, mags = case_tensors(case, cuda_device)
    empty_rays = [torch.empty(0, 3, device=cuda_device), torch.empty(0, 3, device=cuda_device), torch.empty(0, device=cuda_device),
                  torch.empty(0, 6, device=cuda_device)]
    f.forward(*empty_rays, 0, False, table, mags, features_float=torch.empty(0, f.n_output_features, device=cuda_device))
    g = backend.Featurizer(case['level'], case['sizes'], case['entries'], 2, 0)
    empty = torch.empty(0, device=cuda_device)
    g.forward(*empty_rays, 0, False, table, mags, empty, empty, empty, empty, empty, empty, empty, empty, empty)
    torch.cuda.synchronize()


def test_unsupported_layouts_fail_loudly(capi, backend, cuda_device):
    with pytest.raises(capi.ZfError, match='features per level'):
        capi.CFeaturizer(0, [16], [4096], 5, 0)
    with pytest.raises(capi.ZfError, match='grid levels'):
        capi.CFeaturizer(0, [16] * 17, [4096] * 17, 1, 0)
    with pytest.raises(RuntimeError, match='ZipNeRF: grid table too large'):
        backend.Featurizer(0, [2048, 2048], [2 ** 31, 2 ** 31], 4, 0)


def test_erf_saturation_is_exact(capi, cuda_device):
    """The kernels skip the erf downweighting for arguments >= the build's threshold and use exactly 1.0f: this holds
    only if the fast-math erf of the reference's formula (featurize_common.cuh:45-47) is exactly 1.0f for every float
    argument from the threshold to +inf, which is checked exhaustively on the device."""
    threshold = capi.load().zf_erf_saturation_threshold()
    n_not_one, largest = capi.check_erf_saturation(threshold)
    assert n_not_one == 0, f'{n_not_one} arguments >= {threshold} give an erf below 1 (largest {largest})'
    # and below the threshold the erf is not constant 1 (the early-out changes nothing there)
    n_below, _ = capi.check_erf_saturation(0.0, 1.0)
    assert n_below > 0


@pytest.mark.parametrize('name', ['config2prop_R24_P0', 'grids_F4_R33_I5_S37'])
def test_ray_shards_reproduce_the_whole_batch(capi, cuda_device, name):
    """Two ray shards with their sample offsets draw the random multisample patterns of the whole batch: the forward
    outputs of the shards are bit-identical to the whole batch's rows."""
    from zipnerf_b200 import sharding
    case = CASES[name]
    assert case['seed'] >= 0
    whole = run_forward(capi.CFeaturizer(case['level'], case['sizes'], case['entries'], case['n_features'], case['mlp_width']), case, cuda_device)
    R, n = case['tdist'].shape[0], case['tdist'].shape[1] - 1
    for rank in range(2):
        start, count = sharding.shard_range(R, 2, rank)
        shard = dict(case)
        for key in ('origins', 'directions', 'radii', 'tdist', 'encoded'):
            if key in case:
                shard[key] = np.ascontiguousarray(case[key][start:start + count])
        f = capi.CFeaturizer(case['level'], case['sizes'], case['entries'], case['n_features'], case['mlp_width'])
        f.sample_offset = sharding.sample_offset(start, n)
        out = run_forward(f, shard, cuda_device)
        for key in out:
            expected = whole[key].reshape(R, n, -1)[start:start + count].reshape(out[key].shape)
            np.testing.assert_array_equal(out[key], expected, err_msg=f'{key} of shard {rank}')

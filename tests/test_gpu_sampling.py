"""GPU parity of the sampling, final-level and Adam kernels: against the reference's own kernels compiled for sm_100a
(oracle/_ref/cuda/libzfref_sampling.so, bit for bit: same per-ray arithmetic, same fast-math build), against the CPU
restatement (oracle/zf_step_oracle.c, within the differences of the GPU's fast-math intrinsics from libm), through the
C ABI and the PyTorch binding, with the edge cases the reference handles (empty batches, single rays, ragged warps, the
smallest and largest interval counts, centered and jittered patterns, clipped and non-finite densities, empty bins,
non-finite and fp16 gradients) and its argument errors."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import sampling_cases as sc
from oracle.zf_ref_sampling_cuda import RefAdamCuda, RefSamplingCuda, available
from oracle.zf_step_oracle import StepOracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def ref(cuda_device):
    if not available():
        pytest.fail('the reference sampling kernels are not built (python oracle/ref_cuda/build.py)')
    return RefSamplingCuda()


@pytest.fixture(scope='module')
def capi(cuda_device):
    from zipnerf_b200 import capi as module
    module.load()
    return module


@pytest.fixture(scope='module')
def step_oracle():
    return StepOracle()


def cuda(array, device):
    return torch.from_numpy(np.ascontiguousarray(array)).to(device)


def bits(t: torch.Tensor) -> torch.Tensor:
    """bit patterns, so that NaNs compare equal to themselves"""
    t = t.contiguous()
    return t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)


def assert_same_bits(a: torch.Tensor, b: torch.Tensor, what: str) -> None:
    assert a.shape == b.shape and a.dtype == b.dtype, what
    diff = (bits(a) != bits(b))
    assert not diff.any(), f'{what}: {int(diff.sum())} of {diff.numel()} values differ'


RESAMPLE = [  # rays, intervals, new intervals, input seed, anneal, jitter seed (-1: centered), next level
    (1, 64, 64, 1, 1.0, 3, 1), (33, 64, 64, 2, 1.0, 11, 1), (65, 2, 2, 3, 0.0, -1, 2), (129, 64, 32, 4, 10.0, 5, 2), (300, 32, 64, 5, 0.5, -1, 1),
    (1000, 48, 17, 6, 3.0, 7, 2), (4096, 64, 64, 7, 1.0, 8, 1),
]


@pytest.mark.parametrize('n_rays,n,m,seed,anneal,jitter_seed,level', RESAMPLE)
def test_composite_and_resample_matches_reference_kernel(ref, capi, cuda_device, n_rays, n, m, seed, anneal, jitter_seed, level):
    c = sc.resample_case(n_rays, n, m, seed)
    args = [cuda(c[k], cuda_device) for k in ('raw_density', 'sdist', 'tdist', 'directions')] + [anneal, m, jitter_seed, level, sc.WARP]
    ours = capi.composite_and_resample(*args)
    theirs = ref.composite_and_resample(*args)
    torch.cuda.synchronize()
    for a, b, name in zip(ours, theirs, ['weights', 'sdist', 'tdist']):
        assert_same_bits(a, b, name)
    # the PyTorch binding is the same launch
    import ZipNeRFCudaBackend
    for a, b in zip(ZipNeRFCudaBackend.composite_and_resample(*args), ours):
        assert_same_bits(a, b, 'binding')
    # without the weights output (inference), the intervals are unchanged
    _, s, t = capi.composite_and_resample(*args, with_weights=False)
    assert_same_bits(s, ours[1], 'sdist without weights')
    assert_same_bits(t, ours[2], 'tdist without weights')


def test_composite_and_resample_at_benchmark_size(ref, capi, cuda_device):
    """config 2's proposal level: 65,536 rays x 64 intervals -> 64 (bit for bit) and -> 32 (the NeRF level)"""
    c = sc.resample_case(65536, 64, 64, 99)
    tensors = [cuda(c[k], cuda_device) for k in ('raw_density', 'sdist', 'tdist', 'directions')]
    for m, level in [(64, 1), (32, 2)]:
        ours = capi.composite_and_resample(*tensors, 0.7, m, 12345, level, sc.WARP)
        theirs = ref.composite_and_resample(*tensors, 0.7, m, 12345, level, sc.WARP)
        for a, b, name in zip(ours, theirs, ['weights', 'sdist', 'tdist']):
            assert_same_bits(a, b, name)


@pytest.mark.parametrize('n_rays,n,m,seed,anneal,jitter_seed,level', RESAMPLE[:6])
def test_composite_and_resample_against_cpu_oracle(capi, step_oracle, cuda_device, n_rays, n, m, seed, anneal, jitter_seed, level):
    """Fast-math exp / log / expm1 / pow against libm: weights within 2e-5 relative; resampled edges within 1e-5 except
    where a position falls into a bin whose cdf step is a few float ulps wide (the inverse cdf is ill-conditioned
    there: at most 0.1 % of the edges, and never by more than that bin's width)."""
    c = sc.resample_case(n_rays, n, m, seed)
    args = [cuda(c[k], cuda_device) for k in ('raw_density', 'sdist', 'tdist', 'directions')] + [anneal, m, jitter_seed, level, sc.WARP]
    w, s, t = [x.cpu().numpy() for x in capi.composite_and_resample(*args)]
    w_ref, s_ref, t_ref = step_oracle.composite_and_resample(c['raw_density'], c['sdist'], c['tdist'], c['directions'], anneal, m, jitter_seed, level,
                                                             sc.WARP)
    np.testing.assert_allclose(w, w_ref, rtol=2e-5, atol=1e-7)
    ds = np.abs(s - s_ref)
    assert np.mean(ds > 1e-5) <= 1e-3 and ds.max() <= np.diff(c['sdist'], axis=1).max() + 1e-5
    assert (np.diff(s, axis=1) >= 0).all() and (np.diff(t, axis=1) >= 0).all()
    assert t.min() >= sc.WARP[0] and t.max() <= sc.WARP[1]
    # the metric edges are the warp of the normalized ones (checked above): compare them through the same edges
    assert_metric_close(t, sc.to_metric(s))


@pytest.mark.parametrize('n_rays,degree,n_samples,seed', [(1, 4, 64, 5), (33, 4, 64, -1), (129, 0, 2, 7), (300, 2, 17, -1), (5000, 4, 64, 11)])
def test_initialize_rays_matches_reference_kernel(ref, capi, step_oracle, cuda_device, n_rays, degree, n_samples, seed):
    d = sc.directions(np.random.default_rng(n_rays), n_rays)
    dt = cuda(d, cuda_device)
    ours = capi.initialize_rays(seed, dt, degree, n_samples, sc.WARP)
    theirs = ref.initialize_rays(seed, dt, degree, n_samples, sc.WARP)
    for a, b, name in zip(ours, theirs, ['encoded', 'sdist', 'tdist']):
        assert_same_bits(a, b, name)
    import ZipNeRFCudaBackend
    for a, b in zip(ZipNeRFCudaBackend.initialize_rays(seed, dt, degree, n_samples, sc.WARP), ours):
        assert_same_bits(a, b, 'binding')
    # the CPU restatement: bf16 encodings within one bf16 step of the libm values, edges within float rounding
    enc_ref, s_ref, t_ref = step_oracle.initialize_rays(seed, d, degree, n_samples, sc.WARP)
    enc = ours[0].view(torch.int16).cpu().numpy().astype(np.uint16)
    as_float = lambda e: (e.astype(np.uint32) << 16).view(np.float32)  # noqa: E731
    np.testing.assert_allclose(as_float(enc), as_float(enc_ref), rtol=2 ** -7, atol=2e-5)
    np.testing.assert_allclose(ours[1].cpu().numpy(), s_ref, rtol=0, atol=2e-6)
    assert_metric_close(ours[2].cpu().numpy(), sc.to_metric(ours[1].cpu().numpy()))


def test_view_and_generate_rays_match_reference_kernels(ref, capi, step_oracle, cuda_device):
    pool = sc.ray_pool(21)
    pt = {k: cuda(v, cuda_device) for k, v in pool.items()}
    n_local = int(pool['camera_offsets'][1])
    pixels = np.random.default_rng(6).integers(0, n_local, size=77).astype(np.int64)
    view_args = (cuda(pixels, cuda_device), pt['local_directions'][:n_local].contiguous(), pt['c2w'][0].contiguous(), 0.01, sc.DEGREE, 64, sc.WARP)
    ours = capi.view_rays(*view_args)
    for a, b, name in zip(ours, ref.view_rays(*view_args), ['origins', 'directions', 'radii', 'encoded', 'sdist', 'tdist']):
        assert_same_bits(a, b, f'view_rays {name}')
    import ZipNeRFCudaBackend
    for a, b in zip(ZipNeRFCudaBackend.view_rays(*view_args), ours):
        assert_same_bits(a, b, 'view_rays binding')
    for n_rays, seed in [(1, 3), (40, 123), (1000, 77)]:
        gen_args = (seed, n_rays, pt['view_offsets'], pt['view_cameras'], pt['camera_offsets'], pt['local_directions'], pt['c2w'], pt['camera_radii'],
                    pt['pool_rgb'], sc.DEGREE, 64, sc.WARP)
        ours = capi.generate_rays(*gen_args)
        names = ['origins', 'directions', 'radii', 'rgb', 'encoded', 'sdist', 'tdist']
        for a, b, name in zip(ours, ref.generate_rays(*gen_args), names):
            assert_same_bits(a, b, f'generate_rays {name}')
        for a, b in zip(ZipNeRFCudaBackend.generate_rays(*gen_args), ours):
            assert_same_bits(a, b, 'generate_rays binding')
        # the pixel draw is integer arithmetic: origins and radii equal the CPU restatement's exactly, the colors (a
        # fast-math division by 255) within one float ulp, the directions within rounding
        cpu = step_oracle.generate_rays(seed, n_rays, pool['view_offsets'], pool['view_cameras'], pool['camera_offsets'], pool['local_directions'],
                                        pool['c2w'], pool['camera_radii'], pool['pool_rgb'], sc.DEGREE, 64, sc.WARP)
        for i in (0, 2):
            np.testing.assert_array_equal(ours[i].cpu().numpy(), cpu[i], err_msg=names[i])
        np.testing.assert_allclose(ours[3].cpu().numpy(), cpu[3], rtol=1.2e-7, atol=0)
        np.testing.assert_allclose(ours[1].cpu().numpy(), cpu[1], rtol=1e-6, atol=1e-7)
        assert_metric_close(ours[6].cpu().numpy(), sc.to_metric(ours[5].cpu().numpy()))


def test_sample_uniforms_match_reference(ref, capi, step_oracle, cuda_device):
    for seed, stream, n in [(9, 2, 100), (123456789, 16, 1 << 20), (0, 0, 1)]:
        ours = capi.sample_uniforms(seed, stream, n)
        assert_same_bits(ours, ref.sample_uniforms(seed, stream, n), 'uniforms')
        np.testing.assert_array_equal(ours.cpu().numpy(), step_oracle.sample_uniforms(seed, stream, n))
    import ZipNeRFCudaBackend
    assert_same_bits(ZipNeRFCudaBackend.sample_uniforms(5, 3, 1000), capi.sample_uniforms(5, 3, 1000), 'binding')


def test_sampling_edge_cases_and_errors(capi, cuda_device):
    import ZipNeRFCudaBackend
    d = torch.zeros(0, 3, device=cuda_device)
    enc, s, t = capi.initialize_rays(1, d, 4, 64, sc.WARP)
    assert enc.shape == (0, 32) and s.shape == (0, 65)
    w, s, t = capi.composite_and_resample(torch.zeros(0, 64, device=cuda_device), torch.zeros(0, 65, device=cuda_device),
                                          torch.zeros(0, 65, device=cuda_device), d, 1.0, 64, 1, 1, sc.WARP)
    assert w.shape == (0, 64) and s.shape == (0, 65)
    assert capi.sample_uniforms(1, 2, 0).numel() == 0
    c = sc.resample_case(4, 64, 64, 1)
    args = [cuda(c[k], cuda_device) for k in ('raw_density', 'sdist', 'tdist', 'directions')]
    for m in (1, 65):
        with pytest.raises(capi.ZfError, match='unsupported number of samples per level'):
            capi.composite_and_resample(*args, 1.0, m, 1, 1, sc.WARP)
        with pytest.raises(RuntimeError, match='ZipNeRF: unsupported number of samples per level'):
            ZipNeRFCudaBackend.composite_and_resample(*args, 1.0, m, 1, 1, list(sc.WARP))
    with pytest.raises(RuntimeError, match='ZipNeRF: invalid ray warp'):
        ZipNeRFCudaBackend.initialize_rays(1, args[3], 4, 64, list(sc.WARP)[:6])
    with pytest.raises(RuntimeError, match='ZipNeRF: raw_density must be a contiguous cuda tensor'):
        ZipNeRFCudaBackend.composite_and_resample(args[0].double(), *args[1:], 1.0, 64, 1, 1, list(sc.WARP))
    with pytest.raises(RuntimeError, match='ZipNeRF: c2w must be a 3x4 matrix'):
        ZipNeRFCudaBackend.view_rays(torch.zeros(3, dtype=torch.int64, device=cuda_device), torch.zeros(4, 3, device=cuda_device),
                                     torch.zeros(3, 3, device=cuda_device), 0.01, 4, 64, list(sc.WARP))


def final_case(capi, device, n_rays: int, seed: int, n_final: int = 32) -> dict:
    """The inputs of a training step's final level: rays initialized and resampled through both proposal levels by
    the product's own (bit-exact) sampling kernels, raw proposal densities N(0, 3), NeRF outputs N(0, 2) in bf16 with
    a few non-finite entries (empty samples), random targets."""
    rng = np.random.default_rng(seed)
    d = cuda(sc.directions(rng, n_rays), device)
    _, s, t = capi.initialize_rays(seed, d, sc.DEGREE, 64, sc.WARP)
    proposals = []
    for level, n_next in ((1, 64), (2, n_final)):
        raw = cuda((rng.normal(size=(n_rays, s.shape[1] - 1)) * 3.0).astype(np.float32), device)
        w, s_next, t_next = capi.composite_and_resample(raw, s, t, d, 0.7, n_next, seed, level, sc.WARP)
        proposals.append({'raw_density': raw, 'sdist': s, 'tdist': t, 'weights': w, 'interlevel_weight': 0.01,
                          'interlevel_blur': (0.03, 0.003)[level - 1]})
        s, t = s_next, t_next
    outputs = (rng.normal(size=(n_rays, n_final, 8)) * 2.0).astype(np.float32)
    outputs[..., 4:] = 0.0
    outputs[rng.uniform(size=outputs.shape) < 0.002] = np.nan
    outputs[rng.uniform(size=outputs.shape) < 0.002] = np.inf
    return {'nerf_outputs': cuda(outputs, device).to(torch.bfloat16).contiguous(), 'sdist': s, 'tdist': t, 'proposals': proposals, 'directions': d,
            'seed': seed + 1000, 'rgb_target': cuda(rng.uniform(size=(n_rays, 3)).astype(np.float32), device)}


LOSS_ARGS = (0.001, 0.01, -0.25, 10000.0)  # charbonnier padding, distortion weight, power, premult (Trainer.py:24-33)


@pytest.mark.parametrize('n_rays', [1, 33, 300, 4096, 65536])
def test_train_final_matches_reference_kernel(ref, capi, cuda_device, n_rays):
    c = final_case(capi, cuda_device, n_rays, 17 + n_rays)
    args = (c['nerf_outputs'], c['sdist'], c['tdist'], c['proposals'], c['directions'], c['seed'], c['rgb_target'], *LOSS_ARGS)
    ours = capi.train_final(*args)
    theirs = ref.train_final(*args)
    assert_same_bits(ours[0], theirs[0], 'nerf_outputs_grad')
    for level, (a, b) in enumerate(zip(ours[1], theirs[1])):
        assert_same_bits(a, b, f'proposal {level} raw density gradient')
    torch.testing.assert_close(ours[2], theirs[2], rtol=1e-5, atol=1e-12)  # warp sums added atomically, in varying order
    assert torch.isfinite(ours[0].float()).all() and all(torch.isfinite(g).all() for g in ours[1])
    import ZipNeRFCudaBackend
    p = c['proposals']
    grad, grads, sums = ZipNeRFCudaBackend.train_final(
        c['nerf_outputs'], c['sdist'], c['tdist'], [x['raw_density'] for x in p], [x['sdist'] for x in p], [x['tdist'] for x in p],
        [x['weights'] for x in p], c['directions'], c['seed'], c['rgb_target'], LOSS_ARGS[0], [x['interlevel_weight'] for x in p],
        [x['interlevel_blur'] for x in p], *LOSS_ARGS[1:], True)
    assert_same_bits(grad, ours[0], 'binding')
    for a, b in zip(grads, ours[1]):
        assert_same_bits(a, b, 'binding proposal gradient')
    torch.testing.assert_close(sums, ours[2], rtol=1e-5, atol=1e-12)


@pytest.mark.parametrize('use_median_depth', [False, True])
def test_composite_final_matches_reference_kernel(ref, capi, cuda_device, use_median_depth):
    c = final_case(capi, cuda_device, 1000, 5)
    pixels = torch.randperm(1000, generator=torch.Generator().manual_seed(3)).to(cuda_device)
    background = torch.tensor([0.2, 0.5, 0.9], device=cuda_device)
    images = {}
    for impl in ('ours', 'reference'):
        rgb, alpha, depth = torch.full((1000, 3), -1.0, device=cuda_device), torch.full((1000,), -1.0, device=cuda_device), torch.full((1000,), -1.0, device=cuda_device)
        fn = capi.composite_final if impl == 'ours' else ref.composite_final
        fn(c['nerf_outputs'], c['tdist'], c['directions'], background, pixels, rgb, alpha, depth, use_median_depth=use_median_depth)
        images[impl] = (rgb, alpha, depth)
    for a, b, name in zip(images['ours'], images['reference'], ['rgb', 'alpha', 'depth']):
        assert_same_bits(a, b, name)
    assert (images['ours'][1] >= 0).all() and (images['ours'][2] > 0).all()
    # without the optional outputs, and through the binding
    import ZipNeRFCudaBackend
    rgb = torch.zeros(1000, 3, device=cuda_device)
    empty = torch.empty(0, device=cuda_device)
    ZipNeRFCudaBackend.composite_final(c['nerf_outputs'], c['tdist'], c['directions'], background, pixels, rgb, empty, empty, use_median_depth)
    assert_same_bits(rgb, images['ours'][0], 'binding rgb')


@pytest.mark.parametrize('n_rays,seed', [(33, 4), (300, 8)])
def test_final_level_against_cpu_oracle(capi, step_oracle, cuda_device, n_rays, seed):
    """Fast-math against libm: the bf16 output gradients within a bf16 step; the proposal gradients within 1e-3 relative
    plus 1e-4 of their maximum (the interlevel term has a kink at r = 0, where a rounding moves a value between 0 and a
    tiny gradient); loss sums within 1e-4; images within 1e-5, median depths equal except where a cumulative weight
    lands within rounding of half the opacity (at most 0.5 % of the pixels)."""
    c = sc.final_case(step_oracle, n_rays, seed)
    g_ref, p_ref, l_ref = step_oracle.train_final(c['nerf_outputs'], c['sdist'], c['tdist'], c['proposals'], c['directions'], c['seed'], c['rgb_target'],
                                                  *sc.LOSS_ARGS)
    to = lambda x: cuda(x, cuda_device)  # noqa: E731
    proposals = [{k: (to(v) if isinstance(v, np.ndarray) else v) for k, v in p.items()} for p in c['proposals']]
    outputs = to(c['nerf_outputs'].view(np.int16)).view(torch.bfloat16)
    grad, p_grads, sums = capi.train_final(outputs, to(c['sdist']), to(c['tdist']), proposals, to(c['directions']), c['seed'], to(c['rgb_target']),
                                           *sc.LOSS_ARGS)
    as_float = lambda e: (e.astype(np.uint32) << 16).view(np.float32)  # noqa: E731
    got = as_float(grad.view(torch.int16).cpu().numpy().astype(np.uint16))
    want = as_float(g_ref)
    np.testing.assert_allclose(got, want, rtol=2 ** -7, atol=1e-6 * np.abs(want).max())
    for a, b in zip(p_grads, p_ref):
        np.testing.assert_allclose(a.cpu().numpy(), b, rtol=1e-3, atol=1e-4 * np.abs(b).max())
    np.testing.assert_allclose(sums.cpu().numpy(), l_ref, rtol=1e-4)
    pixels = np.random.default_rng(seed).permutation(n_rays)
    background = np.array([0.2, 0.5, 0.9], np.float32)
    for median in (False, True):
        rgb_ref, alpha_ref, depth_ref = step_oracle.composite_final(c['nerf_outputs'], c['tdist'], c['directions'], background, pixels, n_rays, median)
        rgb, alpha, depth = (torch.full(shape, -1.0, device=cuda_device) for shape in ((n_rays, 3), (n_rays,), (n_rays,)))
        capi.composite_final(outputs, to(c['tdist']), to(c['directions']), to(background), to(pixels), rgb, alpha, depth, use_median_depth=median)
        np.testing.assert_allclose(rgb.cpu().numpy(), rgb_ref, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(alpha.cpu().numpy(), alpha_ref, rtol=1e-5, atol=1e-6)
        if median:
            assert np.mean(depth.cpu().numpy() != depth_ref) <= 0.005
        else:
            np.testing.assert_allclose(depth.cpu().numpy(), depth_ref, rtol=1e-4)


def test_final_level_edge_cases_and_errors(capi, cuda_device):
    import ZipNeRFCudaBackend
    c = final_case(capi, cuda_device, 40, 9)
    grad, grads, sums = capi.train_final(c['nerf_outputs'], c['sdist'], c['tdist'], c['proposals'], c['directions'], c['seed'], c['rgb_target'],
                                         *LOSS_ARGS, compute_loss_sums=False)
    assert sums is None and grad.shape == c['nerf_outputs'].shape
    # no proposal levels: the data and distortion terms only
    grad0, grads0, _ = capi.train_final(c['nerf_outputs'], c['sdist'], c['tdist'], [], c['directions'], c['seed'], c['rgb_target'], *LOSS_ARGS)
    assert grads0 == [] and torch.equal(grad0.view(torch.int16), grad.view(torch.int16))
    empty = capi.train_final(c['nerf_outputs'][:0], c['sdist'][:0], c['tdist'][:0], [], c['directions'][:0], 1, c['rgb_target'][:0], *LOSS_ARGS)
    assert empty[0].numel() == 0
    p = c['proposals']
    lists = ([x['raw_density'] for x in p], [x['sdist'] for x in p], [x['tdist'] for x in p], [x['weights'] for x in p])
    with pytest.raises(RuntimeError, match='ZipNeRF: inconsistent proposal levels'):
        ZipNeRFCudaBackend.train_final(c['nerf_outputs'], c['sdist'], c['tdist'], *lists[:3], lists[3][:1], c['directions'], 1, c['rgb_target'], 0.001,
                                       [0.01, 0.01], [0.03, 0.003], 0.01, -0.25, 1e4, True)
    with pytest.raises(RuntimeError, match='ZipNeRF: invalid nerf_outputs'):
        ZipNeRFCudaBackend.train_final(c['nerf_outputs'][:, :16].contiguous(), c['sdist'], c['tdist'], *lists, c['directions'], 1, c['rgb_target'], 0.001,
                                       [0.01, 0.01], [0.03, 0.003], 0.01, -0.25, 1e4, True)
    with pytest.raises(RuntimeError, match='ZipNeRF: nerf_outputs must be a contiguous cuda tensor'):
        ZipNeRFCudaBackend.train_final(c['nerf_outputs'].float(), c['sdist'], c['tdist'], *lists, c['directions'], 1, c['rgb_target'], 0.001,
                                       [0.01, 0.01], [0.03, 0.003], 0.01, -0.25, 1e4, True)


def metric_rtol(t: np.ndarray) -> np.ndarray:
    """Relative tolerance of metric distances from the fast-math inverse power ladder against libm. With power -1.5 and
    premult 2 the ladder's base is b = (0.8 t + 1)^-1.5; a rounding difference of the normalized coordinate (~2.4e-7
    after scaling) moves b by that absolute amount, i.e. t by about 1.6e-7 (0.8 t + 1)^1.5 relative: ~2e-5 near the
    camera, ~4e-3 at the far plane (1000). Twice that, plus 2e-5."""
    return 2e-5 + 4e-7 * (0.8 * np.abs(t) + 1.0) ** 1.5


def assert_metric_close(t: np.ndarray, t_ref: np.ndarray) -> None:
    bad = np.abs(t - t_ref) > metric_rtol(t_ref) * np.abs(t_ref)
    assert not bad.any(), f'{int(bad.sum())} metric distances differ beyond the conditioning bound, e.g. {t[bad][:4]} vs {t_ref[bad][:4]}'


def adam_tensors(case, device):
    return ([cuda(p, device) for p in case['params']], [cuda(g, device) for g in case['grads']])


@pytest.mark.parametrize('seed', [3, 4])
def test_adam_matches_reference_kernel(ref, capi, step_oracle, cuda_device, seed):
    """Three steps: parameters, moments and zeroed gradients bit for bit with the reference kernel (through the C ABI
    and the PyTorch binding); magnitudes and regularizer to float summation order; all within rounding of the CPU
    restatement."""
    import ZipNeRFCudaBackend
    case = sc.adam_case(seed)
    hyper = (case['reg_weight'], case['max_value'], case['beta1'], case['beta2'], case['eps'])
    n_levels = sum(max(len(o) - 1, 0) for o in case['level_offsets'])
    runs = {}
    for name in ('ours', 'binding', 'reference'):
        params, grads = adam_tensors(case, cuda_device)
        mags = torch.zeros(n_levels, device=cuda_device)
        if name == 'ours':
            opt = capi.CAdam(params, grads, case['grad_scales'], case['level_offsets'], *hyper, mags)
        elif name == 'binding':
            opt = ZipNeRFCudaBackend.Adam(params, grads, case['grad_scales'], case['level_offsets'], *hyper, mags)
        else:
            opt = RefAdamCuda(ref, params, grads, case['grad_scales'], case['level_offsets'], *hyper, mags)
        regs = []
        for step, lr in enumerate([1e-2, 5e-3, 1e-3]):
            if step > 0:  # a new accumulation into the zeroed gradients
                for g, g0 in zip(grads, case['grads']):
                    g.copy_(torch.from_numpy(g0).to(cuda_device) * (step + 1))
            opt.step(lr)
            for g in grads:
                assert not g.any(), 'gradients are zeroed by the step'
            regs.append((opt.regularization() if name == 'binding' else opt.regularization).clone())
        torch.cuda.synchronize()
        if name == 'ours':
            moments = [opt.state(b)[:2] for b in range(len(params))]
        elif name == 'binding':
            moments = [opt.state(b) for b in range(len(params))]
        else:
            moments = list(zip(opt.exp_avgs, opt.exp_avg_sqs))
        runs[name] = (params, moments, mags.clone(), torch.stack(regs))
    for name in ('binding', 'reference'):
        for b, (pa, pb) in enumerate(zip(runs['ours'][0], runs[name][0])):
            assert_same_bits(pa, pb, f'{name} params {b}')
            assert_same_bits(runs['ours'][1][b][0], runs[name][1][b][0], f'{name} exp_avg {b}')
            assert_same_bits(runs['ours'][1][b][1], runs[name][1][b][1], f'{name} exp_avg_sq {b}')
        torch.testing.assert_close(runs['ours'][2], runs[name][2], rtol=1e-5, atol=0)
        torch.testing.assert_close(runs['ours'][3], runs[name][3], rtol=1e-5, atol=0)
    # the CPU restatement (IEEE division and square root against the fast-math build)
    params = [p.copy() for p in case['params']]
    ms = [np.zeros_like(p) for p in params]
    vs = [np.zeros_like(p) for p in params]
    for step, lr in enumerate([1e-2, 5e-3, 1e-3]):
        grads = [g.copy() if step == 0 else (g.astype(np.float32) * (step + 1)).astype(g.dtype) for g in case['grads']]
        mags, reg = step_oracle.adam_step(params, grads, ms, vs, case['grad_scales'], case['level_offsets'], *hyper, step + 1, lr)
    for b, p in enumerate(params):
        # fast-math division and square root against IEEE: each update (~lr) to about 1e-6 of itself
        np.testing.assert_allclose(runs['ours'][0][b].cpu().numpy(), p, rtol=1e-5, atol=1e-2 * 1e-6 * 3)
    np.testing.assert_allclose(runs['ours'][2].cpu().numpy(), mags, rtol=1e-5)
    np.testing.assert_allclose(float(runs['ours'][3][-1]), float(reg), rtol=1e-4)


def test_adam_argument_errors(capi, cuda_device):
    import ZipNeRFCudaBackend
    p = torch.zeros(16, device=cuda_device)
    g = torch.zeros(16, device=cuda_device)
    mags = torch.zeros(2, device=cuda_device)
    with pytest.raises(RuntimeError, match='ZipNeRF: invalid level offsets'):
        ZipNeRFCudaBackend.Adam([p], [g], [1.0], [[0, 6, 16]], 0.1, 1e-5, 0.9, 0.99, 1e-15, mags)
    with pytest.raises(RuntimeError, match='ZipNeRF: level offsets must cover the buffer'):
        ZipNeRFCudaBackend.Adam([p], [g], [1.0], [[0, 8, 12]], 0.1, 1e-5, 0.9, 0.99, 1e-15, mags)
    with pytest.raises(RuntimeError, match='ZipNeRF: optimizer gradient size mismatch'):
        ZipNeRFCudaBackend.Adam([p], [torch.zeros(8, device=cuda_device)], [1.0], [[]], 0.1, 1e-5, 0.9, 0.99, 1e-15, mags[:0])
    with pytest.raises(RuntimeError, match='ZipNeRF: param must be a contiguous float'):
        ZipNeRFCudaBackend.Adam([torch.zeros(6, device=cuda_device)], [torch.zeros(6, device=cuda_device)], [1.0], [[]], 0.1, 1e-5, 0.9, 0.99, 1e-15, mags[:0])
    with pytest.raises(RuntimeError, match='ZipNeRF: magnitudes must be'):
        ZipNeRFCudaBackend.Adam([p], [g], [1.0], [[0, 8, 16]], 0.1, 1e-5, 0.9, 0.99, 1e-15, mags[:1])
    with pytest.raises(RuntimeError, match='ZipNeRF: invalid optimizer buffers'):
        ZipNeRFCudaBackend.Adam([p], [g, g], [1.0], [[]], 0.1, 1e-5, 0.9, 0.99, 1e-15, mags[:0])
    # an optimizer without grid levels: no magnitudes, no regularizer
    opt = ZipNeRFCudaBackend.Adam([p], [g], [1.0], [[]], 0.1, 1e-5, 0.9, 0.99, 1e-15, mags[:0])
    g.fill_(1.0)
    opt.step(0.1)
    torch.cuda.synchronize()
    assert float(opt.regularization()) == 0.0 and not g.any() and (p < 0).all()

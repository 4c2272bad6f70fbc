"""Host-side checks that need no GPU: the C-ABI library loads and exports every function include/*.h declares, its
constants and argument validation behave like the reference's, the PyTorch binding imports with the reference's
module surface, and the workload generators produce the benchmark shapes."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
HEADERS = sorted((REPO / 'include').glob('*.h'))


def declared_functions() -> list[str]:
    text = '\n'.join(h.read_text() for h in HEADERS)
    return sorted(set(re.findall(r'ZF_API\s+[\w\s\*]+?\b(zf_\w+)\s*\(', text)))


def test_header_declares_the_reference_entry_points():
    names = declared_functions()
    for name in ['zf_featurizer_create', 'zf_featurizer_destroy', 'zf_featurizer_n_fp32_grad_rows', 'zf_featurize_forward',
                 'zf_featurize_backward', 'zf_featurize_backward_mlp', 'zf_last_error']:
        assert name in names
    # sampling_api.h:10-58 and optimizer_api.h:14-40
    for name in ['zf_generate_rays', 'zf_view_rays', 'zf_initialize_rays', 'zf_sample_uniforms', 'zf_composite_and_resample',
                 'zf_train_final', 'zf_composite_final', 'zf_adam_create', 'zf_adam_step', 'zf_adam_destroy']:
        assert name in names


def test_library_exports_every_declared_function():
    from zipnerf_b200 import capi
    lib = capi.load()
    for name in declared_functions():
        assert hasattr(lib, name), f'{name} is declared in include/ but not exported'
    assert sorted(capi.EXPORTED) == declared_functions()


def test_module_constants():
    from zipnerf_b200 import capi
    lib = capi.load()
    assert lib.zf_grid_max_value() == pytest.approx(1e-5, rel=0, abs=1e-20)  # bindings.cu:14
    assert lib.zf_nerf_grid_grad_scale() == 1048576.0  # zipnerf_config.h:12


def test_create_validates_layout_before_touching_a_device():
    from zipnerf_b200 import capi
    lib = capi.load()
    handle = ctypes.c_void_p()
    sizes = (ctypes.c_int64 * 3)(2, 4, 128)
    entries = (ctypes.c_int64 * 3)(8, 64, 1 << 20)
    assert lib.zf_featurizer_create(0, sizes, entries, 3, 5, 0, ctypes.byref(handle)) == capi.ZF_ERROR_UNSUPPORTED
    assert b'features per level' in lib.zf_last_error()
    assert lib.zf_featurizer_create(0, sizes, entries, 0, 4, 0, ctypes.byref(handle)) == capi.ZF_ERROR_UNSUPPORTED
    assert lib.zf_featurizer_create(0, sizes, entries, 3, 4, -1, ctypes.byref(handle)) == capi.ZF_ERROR_INVALID_ARGUMENT
    big = (ctypes.c_int64 * 2)(1 << 31, 1 << 31)
    assert lib.zf_featurizer_create(0, (ctypes.c_int64 * 2)(2048, 2048), big, 2, 4, 0, ctypes.byref(handle)) == capi.ZF_ERROR_INVALID_ARGUMENT
    assert b'32-bit indexing' in lib.zf_last_error()
    # cell coordinates are packed into 16 bits
    wide = (ctypes.c_int64 * 1)(70000)
    for n_features in (2, 4):
        assert lib.zf_featurizer_create(0, wide, (ctypes.c_int64 * 1)(1 << 20), 1, n_features, 0, ctypes.byref(handle)) == capi.ZF_ERROR_UNSUPPORTED
        assert b'65534' in lib.zf_last_error()
    assert lib.zf_featurize_forward(None, None, None) == capi.ZF_ERROR_INVALID_ARGUMENT
    assert lib.zf_featurizer_n_output_features(None) == 0


def test_sampling_and_adam_validate_before_touching_a_device():
    """The checks of sampling_api.cu:443-445 and optimizer_api.cu:123-155 come before any launch or allocation."""
    from zipnerf_b200 import capi
    lib = capi.load()
    assert lib.zf_direction_block_width(4) == 32 and lib.zf_direction_block_width(0) == 8
    warp = capi.make_ray_warp([0.2, 1000.0, 0.0, 1.0, -1.5, 2.0, 1.6])
    for n_intervals, n_samples in [(64, 1), (64, 65), (1, 64), (65, 64)]:
        a = capi.zf_resample_args(None, None, None, None, 4, n_intervals, 1.0, n_samples, 0, 1, warp, None, None, None)
        assert lib.zf_composite_and_resample(ctypes.byref(a), None) == capi.ZF_ERROR_UNSUPPORTED
        assert b'unsupported number of samples per level' in lib.zf_last_error()
    empty = capi.zf_resample_args(None, None, None, None, 0, 64, 1.0, 64, 0, 1, warp, None, None, None)
    assert lib.zf_composite_and_resample(ctypes.byref(empty), None) == capi.ZF_OK  # nothing to launch
    init = capi.zf_initialize_rays_args(0, None, 0, 4, 64, warp, None, None, None)
    assert lib.zf_initialize_rays(ctypes.byref(init), None) == capi.ZF_OK
    init.n_rays = 3
    assert lib.zf_initialize_rays(ctypes.byref(init), None) == capi.ZF_ERROR_INVALID_ARGUMENT
    assert lib.zf_sample_uniforms(1, 2, 0, None, None) == capi.ZF_OK
    assert lib.zf_sample_uniforms(1, 2, 5, None, None) == capi.ZF_ERROR_INVALID_ARGUMENT
    handle = ctypes.c_void_p()
    fake = 1 << 20  # never dereferenced: creation fails in validation
    offsets = (ctypes.c_int64 * 3)(0, 6, 16)
    buf = capi.zf_adam_buffer(fake, fake, 0, 16, 1.0, offsets, 3)
    assert lib.zf_adam_create(ctypes.byref(buf), 1, 0.1, 1e-5, 0.9, 0.99, 1e-15, fake, 2, fake, ctypes.byref(handle)) == capi.ZF_ERROR_INVALID_ARGUMENT
    assert b'invalid level offsets' in lib.zf_last_error()
    buf.level_offsets, buf.n_level_offsets = (ctypes.c_int64 * 3)(0, 8, 12), 3
    assert lib.zf_adam_create(ctypes.byref(buf), 1, 0.1, 1e-5, 0.9, 0.99, 1e-15, fake, 2, fake, ctypes.byref(handle)) == capi.ZF_ERROR_INVALID_ARGUMENT
    assert b'level offsets must cover the buffer' in lib.zf_last_error()
    buf.level_offsets, buf.n_level_offsets = (ctypes.c_int64 * 3)(0, 8, 16), 3
    assert lib.zf_adam_create(ctypes.byref(buf), 1, 0.1, 1e-5, 0.9, 0.99, 1e-15, fake, 1, fake, ctypes.byref(handle)) == capi.ZF_ERROR_INVALID_ARGUMENT
    assert b'one entry per level' in lib.zf_last_error()
    assert lib.zf_adam_create(ctypes.byref(buf), 9, 0.1, 1e-5, 0.9, 0.99, 1e-15, fake, 2, fake, ctypes.byref(handle)) == capi.ZF_ERROR_INVALID_ARGUMENT
    assert b'invalid optimizer buffers' in lib.zf_last_error()
    assert lib.zf_adam_step(None, 0.1, None) == capi.ZF_ERROR_INVALID_ARGUMENT


def test_relu_backward_validates_its_layout():
    from zipnerf_b200 import capi
    lib = capi.load()
    fake = 1 << 20  # never dereferenced
    for cols, grad_stride, act_stride in [(12, 16, 16), (520, 520, 520), (64, 60, 64), (64, 64, 100), (0, 8, 8)]:
        assert lib.zf_relu_backward_bf16(fake, grad_stride, fake, act_stride, 10, cols, None, None) == capi.ZF_ERROR_INVALID_ARGUMENT
    assert lib.zf_relu_backward_bf16(fake + 2, 64, fake, 64, 10, 64, None, None) == capi.ZF_ERROR_INVALID_ARGUMENT
    assert b'16-byte aligned' in lib.zf_last_error()
    assert lib.zf_relu_backward_bf16(None, 64, None, 64, 0, 64, None, None) == capi.ZF_OK  # nothing to do


@pytest.mark.skipif(torch.cuda.is_available(), reason='checks the error path of a machine without a GPU')
def test_create_without_device_reports_cuda_error():
    from zipnerf_b200 import capi
    lib = capi.load()
    handle = ctypes.c_void_p()
    rc = lib.zf_featurizer_create(0, (ctypes.c_int64 * 1)(16), (ctypes.c_int64 * 1)(4096), 1, 1, 0, ctypes.byref(handle))
    assert rc == capi.ZF_ERROR_CUDA and not handle


def test_torch_binding_has_the_reference_surface():
    import ZipNeRFCudaBackend
    from ZipNeRFCudaBackend import _C
    from ZipNeRFCudaBackend.torch_bindings import pipeline
    assert _C.grid_max_value == pytest.approx(1e-5) and _C.nerf_grid_grad_scale == 1048576.0
    _C.set_rtc_dirs('/nonexistent/cache', '/nonexistent/kernels')  # accepted and unused (kernels are compiled ahead of time)
    for method in ['forward', 'backward', 'backward_mlp']:
        assert hasattr(_C.Featurizer, method)
    for name in ['generate_rays', 'view_rays', 'initialize_rays', 'sample_uniforms', 'composite_and_resample', 'train_final', 'composite_final',
                 'Adam']:
        assert getattr(ZipNeRFCudaBackend, name) is getattr(_C, name) is getattr(pipeline, name)
    assert hasattr(_C.Adam, 'step') and hasattr(_C.Adam, 'regularization')
    assert isinstance(_C.Featurizer.n_fp32_grad_rows, property)
    assert pipeline.Featurizer is _C.Featurizer
    from zipnerf_b200 import nerf_mlp
    assert ZipNeRFCudaBackend.NerfMlp is pipeline.NerfMlp is nerf_mlp.NerfMlp
    assert ZipNeRFCudaBackend.nerf_mlp_parameters is pipeline.nerf_mlp_parameters is nerf_mlp.nerf_mlp_parameters
    with pytest.raises(AttributeError):
        ZipNeRFCudaBackend.not_an_entry_point
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError, match='ZipNeRF: '):
            _C.Featurizer(0, [16, 32], [4096, 32768], 1, 64)


def test_workload_shapes():
    from zipnerf_b200 import workloads
    wl = workloads.config2(n_rays=64)
    assert [l.n_intervals for l in wl.levels] == [64, 64, 32]
    assert [l.n_features for l in wl.levels] == [1, 1, 4] and [l.mlp_width for l in wl.levels] == [64, 64, 0]
    assert wl.levels[2].sizes == [16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192]
    assert sum(wl.levels[0].entries) == 10334929 and sum(wl.levels[2].entries) == 14979072
    for level in wl.levels:
        t = level.tdist
        assert (t[:, 1:] >= t[:, :-1]).all() and t.min() >= 0.2 and t.max() <= 1000.0
    wl1 = workloads.config1(n_rays=16)
    assert wl1.levels[0].sizes == [16, 27, 47, 81, 138, 237, 406, 697, 1195, 2048]
    assert wl.n_intervals_total == 64 * 160


def test_every_declared_function_names_what_it_replaces():
    """The comment above each declaration in include/*.h cites the reference interface it replaces (file:line) or
    says that it has no counterpart there."""
    missing = []
    for header in HEADERS:
        text = header.read_text()
        for m in re.finditer(r'ZF_API\s+[\w\s\*]+?\b(zf_\w+)\s*\(', text):
            before = text[:m.start()].rstrip()
            comment = before[before.rindex('/*'):] if before.endswith('*/') else ''
            if not (re.search(r'\.(cu|cuh|h|py):\d+', comment) or 'counterpart' in comment or 'lifetime' in comment):
                missing.append(f'{header.name}:{m.group(1)}')
    assert not missing, missing


@pytest.mark.parametrize('width,height', [(16, 16), (37, 23), (1, 9), (1296, 840)])
def test_morton_order_interleaves_the_pixel_bits(width, height):
    """workloads.morton_order against a per-bit restatement of the Z-order key (x bits even, y bits odd) of
    Renderer.pixel_order (Renderer.py:120-130): a permutation of the pixels sorted by key."""
    import numpy as np
    from zipnerf_b200 import workloads
    order = workloads.morton_order(width, height).numpy()
    y, x = np.divmod(np.arange(width * height), width)
    key = np.zeros(width * height, dtype=np.int64)
    for bit in range(16):
        key |= ((x >> bit) & 1) << (2 * bit) | ((y >> bit) & 1) << (2 * bit + 1)
    assert np.array_equal(np.sort(order), np.arange(width * height))
    np.testing.assert_array_equal(order, np.argsort(key, kind='stable'))


def test_nerf_mlp_forward_validates_before_touching_a_device():
    from zipnerf_b200 import capi
    lib = capi.load()
    fake = 1 << 20  # 16-byte aligned, never dereferenced
    w = capi.zf_nerf_mlp_weights(*([fake] * 9))
    assert lib.zf_nerf_mlp_forward_tc(fake, 56, fake, 96, ctypes.byref(w), fake, None, 0, fake, None) == capi.ZF_OK  # nothing to do
    assert lib.zf_nerf_mlp_forward_tc(fake, 56, fake, 96, None, fake, None, 4, fake, None) == capi.ZF_ERROR_INVALID_ARGUMENT
    w.view_1 = fake + 8
    assert lib.zf_nerf_mlp_forward_tc(fake, 56, fake, 96, ctypes.byref(w), fake, None, 4, fake, None) == capi.ZF_ERROR_INVALID_ARGUMENT
    assert b'16-byte aligned' in lib.zf_last_error()
    w.view_1 = fake
    # the training forward's activations buffer must be 16-byte aligned too
    assert lib.zf_nerf_mlp_forward_tc(fake, 56, fake, 96, ctypes.byref(w), fake, fake + 2, 4, fake, None) == capi.ZF_ERROR_INVALID_ARGUMENT
    assert b'activations' in lib.zf_last_error()
    for features_stride, inputs_stride in [(50, 96), (56, 90), (48, 96), (56, 88)]:
        assert lib.zf_nerf_mlp_forward_tc(fake, features_stride, fake, inputs_stride, ctypes.byref(w), fake, None, 4, fake, None) == capi.ZF_ERROR_INVALID_ARGUMENT
        assert b'row strides' in lib.zf_last_error()


def test_nerf_mlp_training_record_and_backward_limits():
    """The training record's size (v0-v2 in bf16, then the ReLU masks as bits) is the same on both sides of the ABI,
    and the tensor-core backward rejects sample counts its 32-bit tensor-copy coordinates cannot address before it
    touches a device."""
    from zipnerf_b200 import capi
    lib = capi.load()
    for n in (0, 1, 127, 2_097_152):
        assert lib.zf_nerf_mlp_activations_size(n) == capi.nerf_mlp_record_size(n) == n * (3 * 512 + 3 * 32 + 8)
    fake = 1 << 20
    w = capi.zf_nerf_mlp_weights_t(*([fake] * 6))
    g = capi.zf_nerf_mlp_grads(*([fake] * 9))
    n = 2 ** 31
    assert lib.zf_nerf_mlp_backward_tc(fake, fake, 56, fake, 96, fake, ctypes.byref(w), fake, 56, ctypes.byref(g), fake, 1 << 62, n, fake,
                                       None) == capi.ZF_ERROR_INVALID_ARGUMENT
    assert b'too many samples' in lib.zf_last_error()


def test_nerf_mlp_pack_and_unfold_validate_before_touching_a_device():
    """The pack and unfold entry points reject missing pointers and a misaligned fp32 bias target before any launch,
    and the parameter count they assume is the table's of the reference model's widths."""
    from zipnerf_b200 import capi, nerf_mlp as nm
    lib = capi.load()
    assert lib.zf_nerf_mlp_parameter_count() == nm.NerfMlpLayout().size == 227_556
    fake = 1 << 20
    targets = capi.zf_nerf_mlp_packed(*([fake] * len(capi.NERF_MLP_PACK_TARGETS)))
    assert lib.zf_nerf_mlp_pack(None, ctypes.byref(targets), None) == capi.ZF_ERROR_INVALID_ARGUMENT
    assert lib.zf_nerf_mlp_pack(fake, None, None) == capi.ZF_ERROR_INVALID_ARGUMENT
    targets.tc_view_1_bias = fake + 2  # fp32 biases need 4-byte alignment
    assert lib.zf_nerf_mlp_pack(fake, ctypes.byref(targets), None) == capi.ZF_ERROR_INVALID_ARGUMENT
    assert b'misaligned' in lib.zf_last_error()
    grads = capi.zf_nerf_mlp_grads(*([fake] * 9))
    assert lib.zf_nerf_mlp_unfold_grads(fake, ctypes.byref(grads), None, None) == capi.ZF_ERROR_INVALID_ARGUMENT
    grads.rgb = None
    assert lib.zf_nerf_mlp_unfold_grads(fake, ctypes.byref(grads), fake, None) == capi.ZF_ERROR_INVALID_ARGUMENT
    assert b'gradients must be given' in lib.zf_last_error()

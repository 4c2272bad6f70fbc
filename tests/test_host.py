"""Host-side checks that need no GPU: the C-ABI library loads and exports every function include/zf_featurize.h
declares, its constants and argument validation behave like the reference's, the PyTorch binding imports with the
reference's module surface, and the workload generators produce the benchmark shapes."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / 'include' / 'zf_featurize.h'


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r'ZF_API\s+[\w\s\*]+?\b(zf_\w+)\s*\(', text)))


def test_header_declares_the_reference_entry_points():
    names = declared_functions()
    for name in ['zf_featurizer_create', 'zf_featurizer_destroy', 'zf_featurizer_n_fp32_grad_rows', 'zf_featurize_forward',
                 'zf_featurize_backward', 'zf_featurize_backward_mlp', 'zf_last_error']:
        assert name in names


def test_library_exports_every_declared_function():
    from zipnerf_b200 import capi
    lib = capi.load()
    for name in declared_functions():
        assert hasattr(lib, name), f'{name} is declared in zf_featurize.h but not exported'
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
    assert isinstance(_C.Featurizer.n_fp32_grad_rows, property)
    assert pipeline.Featurizer is _C.Featurizer
    with pytest.raises(AttributeError, match='not part of the B200 featurization backend'):
        ZipNeRFCudaBackend.NerfMlp
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

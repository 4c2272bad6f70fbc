"""B200 (sm_100a) featurization backend, importable as the reference's extension package ``ZipNeRFCudaBackend``.

The compiled module ``ZipNeRFCudaBackend._C`` (PyTorch binding) and ``libzf_featurize.so`` (kernels and C ABI) sit in
this directory; build them with ``python fused-zipnerf_b200/build.py``. The featurization entry points mirror the
reference binding (ZipNeRFCudaBackend/ZipNeRFCudaBackend/torch_bindings/bindings.cu:14-22): ``grid_max_value``,
``nerf_grid_grad_scale``, ``set_rtc_dirs`` and ``Featurizer``; the sampling functions ``generate_rays``, ``view_rays``,
``initialize_rays``, ``sample_uniforms``, ``composite_and_resample``, ``train_final`` and ``composite_final``
(sampling_api.h:10-90); ``Adam`` (optimizer_api.h:14-40); and the NeRF MLP's ``NerfMlp`` and ``nerf_mlp_parameters``
(nerf_mlp.h:31-73) with the reference's parameter layout, from ``zipnerf_b200.nerf_mlp`` in the directory above.
"""
from __future__ import annotations

from pathlib import Path

_HERE = Path(__file__).resolve().parent

try:
    from . import _C  # noqa: F401  (loads libzf_featurize.so through its rpath)
except ImportError as error:  # the product has no fallback: without the compiled extension nothing works
    raise ImportError(
        f'ZipNeRFCudaBackend._C is not built in {_HERE} (run: python fused-zipnerf_b200/build.py): {error}') from error

grid_max_value = _C.grid_max_value
nerf_grid_grad_scale = _C.nerf_grid_grad_scale
Featurizer = _C.Featurizer
set_rtc_dirs = _C.set_rtc_dirs
Adam = _C.Adam
generate_rays = _C.generate_rays
view_rays = _C.view_rays
initialize_rays = _C.initialize_rays
sample_uniforms = _C.sample_uniforms
composite_and_resample = _C.composite_and_resample
train_final = _C.train_final
composite_final = _C.composite_final
relu_backward_ = _C.relu_backward_  # addition: the ReLU backward + bias gradient of a bf16 layer (zf_mlp.h)

import sys as _sys  # noqa: E402

if str(_HERE.parent) not in _sys.path:  # zipnerf_b200 sits beside this package
    _sys.path.append(str(_HERE.parent))
from zipnerf_b200.nerf_mlp import NerfMlp, nerf_mlp_parameters  # noqa: E402

__all__ = ['grid_max_value', 'nerf_grid_grad_scale', 'Featurizer', 'set_rtc_dirs', 'Adam', 'generate_rays', 'view_rays', 'initialize_rays',
           'sample_uniforms', 'composite_and_resample', 'train_final', 'composite_final', 'nerf_mlp_parameters', 'NerfMlp']

"""B200 (sm_100a) featurization backend, importable as the reference's extension package ``ZipNeRFCudaBackend``.

The compiled module ``ZipNeRFCudaBackend._C`` (PyTorch binding) and ``libzf_featurize.so`` (kernels and C ABI) sit in
this directory; build them with ``python fused-zipnerf_b200/build.py``. The featurization entry points mirror the
reference binding (ZipNeRFCudaBackend/ZipNeRFCudaBackend/torch_bindings/bindings.cu:14-22): ``grid_max_value``,
``nerf_grid_grad_scale``, ``set_rtc_dirs`` and ``Featurizer``; the sampling functions ``generate_rays``, ``view_rays``,
``initialize_rays``, ``sample_uniforms``, ``composite_and_resample``, ``train_final`` and ``composite_final``
(sampling_api.h:10-90); and ``Adam`` (optimizer_api.h:14-40). The reference's NeRF MLP (``NerfMlp``,
``nerf_mlp_parameters``) is not provided here; accessing it raises an ``AttributeError`` that says so.
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

_OTHER_SUBSYSTEMS = {'nerf_mlp_parameters', 'NerfMlp'}

__all__ = ['grid_max_value', 'nerf_grid_grad_scale', 'Featurizer', 'set_rtc_dirs', 'Adam', 'generate_rays', 'view_rays', 'initialize_rays',
           'sample_uniforms', 'composite_and_resample', 'train_final', 'composite_final']


def __getattr__(name: str):
    if name in _OTHER_SUBSYSTEMS:
        raise AttributeError(f'ZipNeRFCudaBackend.{name} is not part of the B200 featurization backend; it belongs to the reference '
                             f"backend's NeRF MLP subsystem")
    raise AttributeError(f'module ZipNeRFCudaBackend has no attribute {name}')

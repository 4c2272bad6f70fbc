"""Re-exports of the featurization entry points under the reference's module path
(ZipNeRFCudaBackend/ZipNeRFCudaBackend/torch_bindings/pipeline.py:1-5)."""
from ZipNeRFCudaBackend import _C

grid_max_value = _C.grid_max_value
nerf_grid_grad_scale = _C.nerf_grid_grad_scale
Featurizer = _C.Featurizer
set_rtc_dirs = _C.set_rtc_dirs

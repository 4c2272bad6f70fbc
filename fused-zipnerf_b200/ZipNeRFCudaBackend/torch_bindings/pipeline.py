"""Re-exports of the backend's entry points under the reference's module path
(ZipNeRFCudaBackend/ZipNeRFCudaBackend/torch_bindings/pipeline.py:1-15): featurization, sampling, Adam and the NeRF
MLP."""
import ZipNeRFCudaBackend as _backend
from ZipNeRFCudaBackend import _C

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
nerf_mlp_parameters = _backend.nerf_mlp_parameters
NerfMlp = _backend.NerfMlp

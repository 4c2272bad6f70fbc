"""ctypes binding of the C ABI in include/zf_featurize.h, zf_sampling.h, zf_optim.h and zf_mlp.h (libzf_featurize.so).

This is the binding a Python host without the PyTorch extension would write against the library. ``CFeaturizer``
adds a thin convenience layer that takes PyTorch CUDA tensors and passes their device pointers; the computation
happens in the library. No CPU fallback exists: calls fail with ``ZfError`` when the
library reports an error, and loading fails when the library is not built.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent.parent / 'ZipNeRFCudaBackend' / 'libzf_featurize.so'

ZF_OK, ZF_ERROR_INVALID_ARGUMENT, ZF_ERROR_UNSUPPORTED, ZF_ERROR_CUDA = 0, 1, 2, 3

EXPORTED = ['zf_featurizer_create', 'zf_featurizer_destroy', 'zf_featurizer_n_output_features', 'zf_featurizer_n_fp32_grad_rows',
            'zf_featurizer_n_rows', 'zf_featurizer_launches', 'zf_featurize_forward', 'zf_featurize_backward', 'zf_featurize_backward_mlp',
            'zf_featurize_backward_mlp_workspace_size', 'zf_featurize_backward_mlp_no_alloc', 'zf_featurize_debug',
            'zf_check_erf_saturation', 'zf_erf_saturation_threshold', 'zf_last_error', 'zf_grid_max_value', 'zf_nerf_grid_grad_scale',
            'zf_direction_block_width', 'zf_initialize_rays', 'zf_view_rays', 'zf_generate_rays', 'zf_sample_uniforms',
            'zf_composite_and_resample', 'zf_train_final', 'zf_composite_final', 'zf_adam_create', 'zf_adam_destroy', 'zf_adam_step',
            'zf_adam_state', 'zf_relu_backward_bf16', 'zf_nerf_mlp_activations_size', 'zf_nerf_mlp_forward_tc', 'zf_nerf_mlp_backward_workspace_size',
            'zf_nerf_mlp_backward_tc', 'zf_nerf_mlp_parameter_count', 'zf_nerf_mlp_pack', 'zf_nerf_mlp_unfold_grads']

_p = ctypes.c_void_p
_i64 = ctypes.c_int64


class zf_rays(ctypes.Structure):
    _fields_ = [('origins', _p), ('directions', _p), ('radii', _p), ('tdist', _p), ('n_rays', _i64), ('n_intervals', _i64),
                ('pattern_seed', _i64), ('sample_offset', _i64)]


class zf_forward_args(ctypes.Structure):
    _fields_ = [('rays', zf_rays), ('interleave', ctypes.c_int), ('table', _p), ('table_rows', _i64), ('scale_magnitudes', _p),
                ('w0', _p), ('b0', _p), ('w1', _p), ('b1', _p), ('w0_numel', _i64), ('raw_density', _p), ('features_float', _p),
                ('features_bf16', _p), ('features_bf16_width', _i64), ('encoded_directions', _p), ('encoded_width', _i64),
                ('nerf_inputs', _p), ('nerf_inputs_width', _i64)]


class zf_backward_args(ctypes.Structure):
    _fields_ = [('rays', zf_rays), ('grad_features', _p), ('grad_features_cols', _i64), ('grad_features_stride', _i64),
                ('grad_table', _p), ('grad_table_numel', _i64), ('grad_table_half', _p), ('grad_table_half_numel', _i64)]


class zf_backward_mlp_args(ctypes.Structure):
    _fields_ = [('rays', zf_rays), ('features', _p), ('features_numel', _i64), ('grad_raw_density', _p),
                ('grad_raw_density_numel', _i64), ('w0', _p), ('b0', _p), ('w1', _p), ('w0_numel', _i64), ('grad_table', _p),
                ('grad_table_numel', _i64), ('grad_w0', _p), ('grad_w0_numel', _i64), ('grad_b0', _p), ('grad_w1', _p), ('grad_b1', _p),
                ('workspace', _p), ('workspace_bytes', _i64)]


class zf_ray_warp(ctypes.Structure):
    _fields_ = [(name, ctypes.c_float) for name in ('near', 'far', 'fn_near', 'fn_far', 'power', 'premult', 'y_max')]


class zf_initialize_rays_args(ctypes.Structure):
    _fields_ = [('seed', _i64), ('directions', _p), ('n_rays', _i64), ('direction_degree', ctypes.c_int), ('n_samples', ctypes.c_int),
                ('warp', zf_ray_warp), ('encoded_directions', _p), ('sdist', _p), ('tdist', _p)]


class zf_view_rays_args(ctypes.Structure):
    _fields_ = [('pixel_indices', _p), ('n_rays', _i64), ('local_directions', _p), ('c2w', _p), ('radius', ctypes.c_float),
                ('direction_degree', ctypes.c_int), ('n_samples', ctypes.c_int), ('warp', zf_ray_warp), ('origins', _p), ('directions', _p),
                ('radii', _p), ('encoded_directions', _p), ('sdist', _p), ('tdist', _p)]


class zf_generate_rays_args(ctypes.Structure):
    _fields_ = [('seed', _i64), ('n_rays', _i64), ('view_offsets', _p), ('n_views', ctypes.c_int), ('view_cameras', _p), ('camera_offsets', _p),
                ('local_directions', _p), ('c2w', _p), ('camera_radii', _p), ('pool_rgb', _p), ('n_pixels', _i64),
                ('direction_degree', ctypes.c_int), ('n_samples', ctypes.c_int), ('warp', zf_ray_warp), ('origins', _p), ('directions', _p),
                ('radii', _p), ('rgb', _p), ('encoded_directions', _p), ('sdist', _p), ('tdist', _p)]


class zf_resample_args(ctypes.Structure):
    _fields_ = [('raw_density', _p), ('sdist', _p), ('tdist', _p), ('directions', _p), ('n_rays', _i64), ('n_intervals', ctypes.c_int),
                ('anneal', ctypes.c_float), ('n_samples', ctypes.c_int), ('seed', _i64), ('next_level', ctypes.c_int), ('warp', zf_ray_warp),
                ('weights', _p), ('sdist_next', _p), ('tdist_next', _p)]


class zf_proposal_level(ctypes.Structure):
    _fields_ = [('n_intervals', ctypes.c_int), ('raw_density', _p), ('sdist', _p), ('tdist', _p), ('weights', _p), ('raw_density_grad', _p),
                ('interlevel_weight', ctypes.c_float), ('interlevel_blur', ctypes.c_float)]


class zf_train_final_args(ctypes.Structure):
    _fields_ = [('nerf_outputs', _p), ('sdist', _p), ('tdist', _p), ('n_rays', _i64), ('n_intervals', ctypes.c_int),
                ('proposals', ctypes.POINTER(zf_proposal_level)), ('n_proposal_levels', ctypes.c_int), ('directions', _p), ('seed', _i64),
                ('rgb_target', _p), ('charbonnier_padding', ctypes.c_float), ('distortion_weight', ctypes.c_float),
                ('distortion_power', ctypes.c_float), ('distortion_premult', ctypes.c_float), ('nerf_outputs_grad', _p), ('loss_sums', _p)]


class zf_composite_final_args(ctypes.Structure):
    _fields_ = [('nerf_outputs', _p), ('tdist', _p), ('n_rays', _i64), ('n_intervals', ctypes.c_int), ('directions', _p), ('background', _p),
                ('pixel_indices', _p), ('rgb', _p), ('alpha', _p), ('depth', _p), ('use_median_depth', ctypes.c_int)]


class zf_adam_buffer(ctypes.Structure):
    _fields_ = [('param', _p), ('grad', _p), ('grad_half', ctypes.c_int), ('numel', _i64), ('grad_scale', ctypes.c_double),
                ('level_offsets', ctypes.POINTER(_i64)), ('n_level_offsets', ctypes.c_int)]


class zf_nerf_mlp_weights(ctypes.Structure):
    _fields_ = [(name, _p) for name in ('density', 'density_bias', 'combined', 'skip', 'view_1', 'view_1_bias', 'view_2', 'view_2_bias', 'rgb')]


class zf_nerf_mlp_weights_t(ctypes.Structure):
    _fields_ = [(name, _p) for name in ('rgb_t', 'view_2_t', 'view_1_t', 'combined_t', 'skip_t', 'density_t')]


class zf_nerf_mlp_grads(ctypes.Structure):
    _fields_ = [(name, _p) for name in ('density', 'density_bias', 'combined', 'skip', 'view_1', 'view_1_bias', 'view_2', 'view_2_bias', 'rgb')]


# the targets of zf_nerf_mlp_pack: the row-major section, the tensor-core forward's, the transposed weights
NERF_MLP_PACK_TARGETS = ('density', 'density_bias', 'combined', 'skip', 'view_1', 'view_1_bias', 'view_2', 'view_2_bias', 'rgb',
                         'tc_density', 'tc_density_bias', 'tc_combined', 'tc_skip', 'tc_view_1', 'tc_view_1_bias', 'tc_view_2', 'tc_view_2_bias',
                         'tc_rgb', 'rgb_t', 'view_2_t', 'view_1_t', 'combined_t', 'skip_t', 'density_t')


class zf_nerf_mlp_packed(ctypes.Structure):
    _fields_ = [(name, _p) for name in NERF_MLP_PACK_TARGETS]


class ZfError(RuntimeError):
    def __init__(self, code: int, message: str) -> None:
        super().__init__(message)
        self.code = code


_lib = None


def load() -> ctypes.CDLL:
    """Loads libzf_featurize.so (once) and declares the signatures of include/zf_featurize.h."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIBRARY.exists():
        raise FileNotFoundError(f'{LIBRARY} is not built (python fused-zipnerf_b200/build.py)')
    lib = ctypes.CDLL(str(LIBRARY))
    lib.zf_featurizer_create.argtypes = [ctypes.c_int, ctypes.POINTER(_i64), ctypes.POINTER(_i64), ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, ctypes.POINTER(_p)]
    lib.zf_featurizer_create.restype = ctypes.c_int
    lib.zf_featurizer_destroy.argtypes = [_p]
    lib.zf_featurizer_destroy.restype = None
    lib.zf_featurizer_n_output_features.argtypes = [_p]
    lib.zf_featurizer_n_output_features.restype = ctypes.c_int
    lib.zf_featurizer_n_fp32_grad_rows.argtypes = [_p]
    lib.zf_featurizer_n_fp32_grad_rows.restype = _i64
    lib.zf_featurizer_n_rows.argtypes = [_p]
    lib.zf_featurizer_n_rows.restype = _i64
    lib.zf_featurizer_launches.argtypes = [_p, ctypes.c_int]
    lib.zf_featurizer_launches.restype = ctypes.c_int
    lib.zf_featurize_forward.argtypes = [_p, ctypes.POINTER(zf_forward_args), _p]
    lib.zf_featurize_backward.argtypes = [_p, ctypes.POINTER(zf_backward_args), _p]
    lib.zf_featurize_backward_mlp.argtypes = [_p, ctypes.POINTER(zf_backward_mlp_args), _p]
    lib.zf_featurize_backward_mlp_no_alloc.argtypes = [_p, ctypes.POINTER(zf_backward_mlp_args), _p]
    lib.zf_featurize_backward_mlp_no_alloc.restype = ctypes.c_int
    lib.zf_featurize_backward_mlp_workspace_size.argtypes = [_p, _i64]
    lib.zf_featurize_backward_mlp_workspace_size.restype = _i64
    lib.zf_featurize_debug.argtypes = [_p, ctypes.POINTER(zf_rays), _p, _i64, _p, _p, _p, _p, _p, _p, _p]
    for name in ['zf_featurize_forward', 'zf_featurize_backward', 'zf_featurize_backward_mlp', 'zf_featurize_debug']:
        getattr(lib, name).restype = ctypes.c_int
    lib.zf_check_erf_saturation.argtypes = [ctypes.c_uint32, ctypes.c_uint32, _p, _p, _p]
    lib.zf_check_erf_saturation.restype = ctypes.c_int
    lib.zf_erf_saturation_threshold.argtypes = []
    lib.zf_erf_saturation_threshold.restype = ctypes.c_float
    lib.zf_last_error.argtypes = []
    lib.zf_last_error.restype = ctypes.c_char_p
    lib.zf_grid_max_value.restype = ctypes.c_double
    lib.zf_nerf_grid_grad_scale.restype = ctypes.c_double
    # zf_sampling.h
    lib.zf_direction_block_width.argtypes = [ctypes.c_int]
    lib.zf_direction_block_width.restype = _i64
    lib.zf_initialize_rays.argtypes = [ctypes.POINTER(zf_initialize_rays_args), _p]
    lib.zf_view_rays.argtypes = [ctypes.POINTER(zf_view_rays_args), _p]
    lib.zf_generate_rays.argtypes = [ctypes.POINTER(zf_generate_rays_args), _p]
    lib.zf_sample_uniforms.argtypes = [_i64, _i64, _i64, _p, _p]
    lib.zf_composite_and_resample.argtypes = [ctypes.POINTER(zf_resample_args), _p]
    lib.zf_train_final.argtypes = [ctypes.POINTER(zf_train_final_args), _p]
    lib.zf_composite_final.argtypes = [ctypes.POINTER(zf_composite_final_args), _p]
    for name in ['zf_initialize_rays', 'zf_view_rays', 'zf_generate_rays', 'zf_sample_uniforms', 'zf_composite_and_resample', 'zf_train_final',
                 'zf_composite_final']:
        getattr(lib, name).restype = ctypes.c_int
    # zf_optim.h
    lib.zf_adam_create.argtypes = [ctypes.POINTER(zf_adam_buffer), ctypes.c_int, ctypes.c_double, ctypes.c_double, ctypes.c_double,
                                   ctypes.c_double, ctypes.c_double, _p, _i64, _p, ctypes.POINTER(_p)]
    lib.zf_adam_create.restype = ctypes.c_int
    lib.zf_adam_destroy.argtypes = [_p]
    lib.zf_adam_destroy.restype = None
    lib.zf_adam_step.argtypes = [_p, ctypes.c_double, _p]
    lib.zf_adam_step.restype = ctypes.c_int
    lib.zf_adam_state.argtypes = [_p, ctypes.c_int, ctypes.POINTER(_p), ctypes.POINTER(_p), ctypes.POINTER(_i64)]
    lib.zf_adam_state.restype = ctypes.c_int
    # zf_mlp.h
    lib.zf_relu_backward_bf16.argtypes = [_p, _i64, _p, _i64, _i64, ctypes.c_int, _p, _p]
    lib.zf_relu_backward_bf16.restype = ctypes.c_int
    lib.zf_nerf_mlp_forward_tc.argtypes = [_p, _i64, _p, _i64, _p, _p, _p, _i64, _p, _p]
    lib.zf_nerf_mlp_forward_tc.restype = ctypes.c_int
    lib.zf_nerf_mlp_activations_size.argtypes = [_i64]
    lib.zf_nerf_mlp_activations_size.restype = _i64
    lib.zf_nerf_mlp_backward_workspace_size.argtypes = [_i64]
    lib.zf_nerf_mlp_backward_workspace_size.restype = _i64
    lib.zf_nerf_mlp_backward_tc.argtypes = [_p, _p, _i64, _p, _i64, _p, _p, _p, _i64, _p, _p, _i64, _i64, _p, _p]
    lib.zf_nerf_mlp_backward_tc.restype = ctypes.c_int
    lib.zf_nerf_mlp_parameter_count.argtypes = []
    lib.zf_nerf_mlp_parameter_count.restype = _i64
    lib.zf_nerf_mlp_pack.argtypes = [_p, _p, _p]
    lib.zf_nerf_mlp_pack.restype = ctypes.c_int
    lib.zf_nerf_mlp_unfold_grads.argtypes = [_p, _p, _p, _p]
    lib.zf_nerf_mlp_unfold_grads.restype = ctypes.c_int
    _lib = lib
    return lib


def check(code: int) -> None:
    if code != ZF_OK:
        raise ZfError(code, load().zf_last_error().decode())


def _ptr(tensor) -> int | None:
    return None if tensor is None or tensor.numel() == 0 else tensor.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream if isinstance(stream, int) else stream.cuda_stream


def check_erf_saturation(first: float, last: float = float('inf')) -> tuple[int, float]:
    """Runs zf_check_erf_saturation over the floats in [first, last] (non-negative): returns the number of arguments
    whose erf downweighting is not exactly 1.0f and the largest of them (0.0 if none)."""
    import numpy as np
    import torch
    lib = load()
    lo = int(np.float32(first).view(np.uint32))
    hi = int(np.float32(last).view(np.uint32))
    count = torch.zeros(1, dtype=torch.int64, device='cuda')
    max_bits = torch.zeros(1, dtype=torch.int32, device='cuda')
    check(lib.zf_check_erf_saturation(lo, hi, count.data_ptr(), max_bits.data_ptr(), _stream(None)))
    bits = np.array([max_bits.item()], np.int32).view(np.float32)[0]
    return int(count.item()), float(bits)


class CFeaturizer:
    """A zf_featurizer handle with tensor-level calls (device pointers of contiguous CUDA tensors)."""

    def __init__(self, level: int, sizes, entries, n_features: int, mlp_width: int) -> None:
        lib = load()
        n = len(sizes)
        handle = _p()
        check(lib.zf_featurizer_create(level, (_i64 * n)(*sizes), (_i64 * n)(*entries), n, n_features, mlp_width, ctypes.byref(handle)))
        self.handle = handle
        self.n_features, self.mlp_width = n_features, mlp_width
        self.sample_offset = 0  # batch index of the first sample (pattern random numbers of a shard)
        self.n_output_features = lib.zf_featurizer_n_output_features(handle)
        self.n_fp32_grad_rows = lib.zf_featurizer_n_fp32_grad_rows(handle)
        self.n_rows = lib.zf_featurizer_n_rows(handle)

    def __del__(self) -> None:
        if getattr(self, 'handle', None) and _lib is not None:
            _lib.zf_featurizer_destroy(self.handle)
            self.handle = None

    def rays(self, origins, directions, radii, tdist, pattern_seed: int) -> zf_rays:
        return zf_rays(_ptr(origins), _ptr(directions), _ptr(radii), _ptr(tdist), tdist.shape[0], tdist.shape[1] - 1, pattern_seed,
                       self.sample_offset)

    def forward(self, origins, directions, radii, tdist, pattern_seed, interleave, table, scale_magnitudes, w0=None, b0=None, w1=None,
                b1=None, raw_density=None, features_float=None, features_bf16=None, encoded_directions=None, nerf_inputs=None,
                stream=None) -> None:
        a = zf_forward_args(self.rays(origins, directions, radii, tdist, pattern_seed), int(bool(interleave)), _ptr(table),
                            table.numel() // self.n_features, _ptr(scale_magnitudes), _ptr(w0), _ptr(b0), _ptr(w1), _ptr(b1),
                            w0.numel() if w0 is not None else 0, _ptr(raw_density), _ptr(features_float), _ptr(features_bf16),
                            features_bf16.shape[1] if features_bf16 is not None and features_bf16.numel() else 0,
                            _ptr(encoded_directions), encoded_directions.shape[1] if encoded_directions is not None else 0,
                            _ptr(nerf_inputs), nerf_inputs.shape[1] if nerf_inputs is not None and nerf_inputs.numel() else 0)
        check(load().zf_featurize_forward(self.handle, ctypes.byref(a), _stream(stream)))

    def backward(self, origins, directions, radii, tdist, pattern_seed, grad_features, grad_table, grad_table_half, stream=None) -> None:
        a = zf_backward_args(self.rays(origins, directions, radii, tdist, pattern_seed), _ptr(grad_features), grad_features.shape[1],
                             grad_features.stride(0), _ptr(grad_table), grad_table.numel(), _ptr(grad_table_half), grad_table_half.numel())
        check(load().zf_featurize_backward(self.handle, ctypes.byref(a), _stream(stream)))

    def backward_mlp(self, origins, directions, radii, tdist, pattern_seed, features, grad_raw_density, w0, b0, w1, grad_table,
                     grad_w0, grad_b0, grad_w1, grad_b1, workspace=None, stream=None) -> None:
        """workspace: optional uint8 CUDA tensor of workspace_size(n_samples) bytes (None: allocated per call)."""
        a = zf_backward_mlp_args(self.rays(origins, directions, radii, tdist, pattern_seed), _ptr(features), features.numel(),
                                 _ptr(grad_raw_density), grad_raw_density.numel(), _ptr(w0), _ptr(b0), _ptr(w1), w0.numel(),
                                 _ptr(grad_table), grad_table.numel(), _ptr(grad_w0), grad_w0.numel(), _ptr(grad_b0), _ptr(grad_w1),
                                 _ptr(grad_b1), _ptr(workspace), workspace.numel() if workspace is not None else 0)
        check(load().zf_featurize_backward_mlp(self.handle, ctypes.byref(a), _stream(stream)))

    def backward_mlp_no_alloc(self, origins, directions, radii, tdist, pattern_seed, features, grad_raw_density, w0, b0, w1, grad_table,
                              grad_w0, grad_b0, grad_w1, grad_b1, stream=None) -> None:
        """backward_mlp through zf_featurize_backward_mlp_no_alloc (the library's static workspace; no allocation)."""
        a = zf_backward_mlp_args(self.rays(origins, directions, radii, tdist, pattern_seed), _ptr(features), features.numel(),
                                 _ptr(grad_raw_density), grad_raw_density.numel(), _ptr(w0), _ptr(b0), _ptr(w1), w0.numel(),
                                 _ptr(grad_table), grad_table.numel(), _ptr(grad_w0), grad_w0.numel(), _ptr(grad_b0), _ptr(grad_w1),
                                 _ptr(grad_b1), None, 0)
        check(load().zf_featurize_backward_mlp_no_alloc(self.handle, ctypes.byref(a), _stream(stream)))

    def launches(self, call: str) -> int:
        """Kernel launches of one call: 'forward', 'forward_mlp', 'backward' or 'backward_mlp'."""
        return load().zf_featurizer_launches(self.handle, ['forward', 'forward_mlp', 'backward', 'backward_mlp'].index(call))

    def workspace_size(self, n_samples: int) -> int:
        return load().zf_featurize_backward_mlp_workspace_size(self.handle, n_samples)

    def debug(self, origins, directions, radii, tdist, pattern_seed, samples, stream=None) -> dict:
        """Intermediate values of the given samples (int32 CUDA tensor): x, scale, contracted, n_groups, rows, weights."""
        import torch
        n = samples.numel()
        L = self.n_output_features // (self.n_features + 1)
        dev = samples.device
        out = {'x': torch.zeros(n, 6, 3, device=dev), 'scale': torch.zeros(n, 6, device=dev),
               'contracted': torch.zeros(n, 6, dtype=torch.int32, device=dev), 'n_groups': torch.zeros(n, L, dtype=torch.int32, device=dev),
               'rows': torch.zeros(n, L, 6, 8, dtype=torch.int32, device=dev), 'weights': torch.zeros(n, L, 6, 8, device=dev)}
        rays = self.rays(origins, directions, radii, tdist, pattern_seed)
        check(load().zf_featurize_debug(self.handle, ctypes.byref(rays), _ptr(samples), n, _ptr(out['x']), _ptr(out['scale']),
                                        _ptr(out['contracted']), _ptr(out['n_groups']), _ptr(out['rows']), _ptr(out['weights']),
                                        _stream(stream)))
        out['rows'] = out['rows'].to(torch.int64) & 0xFFFFFFFF
        return out


# ---------------------------------------------------------------------------------------------------------------------
# sampling and Adam through the C ABI, on PyTorch CUDA tensors (outputs allocated here, as the reference's wrappers do)

def make_ray_warp(values) -> zf_ray_warp:
    """The seven ray-warp constants of utils.ray_warp (near, far, fn(near), fn(far), power, premult, y_max)."""
    if len(values) != 7:
        raise ValueError('a ray warp has seven constants')
    return zf_ray_warp(*[float(v) for v in values])


def direction_block_width(degree: int) -> int:
    return load().zf_direction_block_width(degree)


def initialize_rays(seed: int, directions, degree: int, n_samples: int, warp, stream=None):
    """zf_initialize_rays: (encoded_directions bf16 [R, W], sdist [R, n + 1], tdist [R, n + 1])."""
    import torch
    n_rays = directions.shape[0]
    dev = directions.device
    encoded = torch.empty(n_rays, direction_block_width(degree), dtype=torch.bfloat16, device=dev)
    sdist = torch.empty(n_rays, n_samples + 1, device=dev)
    tdist = torch.empty(n_rays, n_samples + 1, device=dev)
    a = zf_initialize_rays_args(seed, _ptr(directions), n_rays, degree, n_samples, make_ray_warp(warp), _ptr(encoded), _ptr(sdist), _ptr(tdist))
    check(load().zf_initialize_rays(ctypes.byref(a), _stream(stream)))
    return encoded, sdist, tdist


def view_rays(pixel_indices, local_directions, c2w, radius: float, degree: int, n_samples: int, warp, stream=None):
    """zf_view_rays: (origins, directions, radii, encoded_directions, sdist, tdist)."""
    import torch
    n_rays = pixel_indices.numel()
    dev = local_directions.device
    origins, directions = torch.empty(n_rays, 3, device=dev), torch.empty(n_rays, 3, device=dev)
    radii = torch.empty(n_rays, device=dev)
    encoded = torch.empty(n_rays, direction_block_width(degree), dtype=torch.bfloat16, device=dev)
    sdist, tdist = torch.empty(n_rays, n_samples + 1, device=dev), torch.empty(n_rays, n_samples + 1, device=dev)
    a = zf_view_rays_args(_ptr(pixel_indices), n_rays, _ptr(local_directions), _ptr(c2w), radius, degree, n_samples, make_ray_warp(warp),
                          _ptr(origins), _ptr(directions), _ptr(radii), _ptr(encoded), _ptr(sdist), _ptr(tdist))
    check(load().zf_view_rays(ctypes.byref(a), _stream(stream)))
    return origins, directions, radii, encoded, sdist, tdist


def generate_rays(seed: int, n_rays: int, view_offsets, view_cameras, camera_offsets, local_directions, c2w, camera_radii, pool_rgb,
                  degree: int, n_samples: int, warp, stream=None):
    """zf_generate_rays: (origins, directions, radii, rgb, encoded_directions, sdist, tdist)."""
    import torch
    dev = local_directions.device
    origins, directions, rgb = (torch.empty(n_rays, 3, device=dev) for _ in range(3))
    radii = torch.empty(n_rays, device=dev)
    encoded = torch.empty(n_rays, direction_block_width(degree), dtype=torch.bfloat16, device=dev)
    sdist, tdist = torch.empty(n_rays, n_samples + 1, device=dev), torch.empty(n_rays, n_samples + 1, device=dev)
    a = zf_generate_rays_args(seed, n_rays, _ptr(view_offsets), view_cameras.numel(), _ptr(view_cameras), _ptr(camera_offsets),
                              _ptr(local_directions), _ptr(c2w), _ptr(camera_radii), _ptr(pool_rgb), pool_rgb.shape[0], degree, n_samples,
                              make_ray_warp(warp), _ptr(origins), _ptr(directions), _ptr(radii), _ptr(rgb), _ptr(encoded), _ptr(sdist), _ptr(tdist))
    check(load().zf_generate_rays(ctypes.byref(a), _stream(stream)))
    return origins, directions, radii, rgb, encoded, sdist, tdist


def sample_uniforms(seed: int, stream_index: int, n: int, device='cuda', stream=None):
    import torch
    values = torch.empty(n, device=device)
    check(load().zf_sample_uniforms(seed, stream_index, n, _ptr(values), _stream(stream)))
    return values


def composite_and_resample(raw_density, sdist, tdist, directions, anneal: float, n_samples: int, seed: int, next_level: int, warp,
                           with_weights: bool = True, stream=None):
    """zf_composite_and_resample: (weights [R, n] or None, sdist_next [R, m + 1], tdist_next [R, m + 1])."""
    import torch
    n_rays, n_intervals = raw_density.shape
    dev = raw_density.device
    weights = torch.empty_like(raw_density) if with_weights else None
    sdist_next, tdist_next = torch.empty(n_rays, n_samples + 1, device=dev), torch.empty(n_rays, n_samples + 1, device=dev)
    a = zf_resample_args(_ptr(raw_density), _ptr(sdist), _ptr(tdist), _ptr(directions), n_rays, n_intervals, anneal, n_samples, seed,
                         next_level, make_ray_warp(warp), _ptr(weights), _ptr(sdist_next), _ptr(tdist_next))
    check(load().zf_composite_and_resample(ctypes.byref(a), _stream(stream)))
    return weights, sdist_next, tdist_next


def train_final(nerf_outputs, sdist, tdist, proposals, directions, seed: int, rgb_target, charbonnier_padding: float, distortion_weight: float,
                distortion_power: float, distortion_premult: float, compute_loss_sums: bool = True, stream=None):
    """zf_train_final. proposals: a list of dicts (raw_density, sdist, tdist, weights, interlevel_weight, interlevel_blur).
    Returns (nerf_outputs_grad, [proposal raw density gradients], loss_sums or None)."""
    import torch
    n_rays, n1 = tdist.shape
    grads = [torch.empty_like(p['raw_density']) for p in proposals]
    levels = (zf_proposal_level * max(len(proposals), 1))(*[
        zf_proposal_level(p['raw_density'].shape[1], _ptr(p['raw_density']), _ptr(p['sdist']), _ptr(p['tdist']), _ptr(p['weights']), _ptr(g),
                          p['interlevel_weight'], p['interlevel_blur']) for p, g in zip(proposals, grads)])
    out_grad = torch.empty_like(nerf_outputs)
    loss_sums = torch.zeros(4, device=tdist.device) if compute_loss_sums else None
    a = zf_train_final_args(_ptr(nerf_outputs), _ptr(sdist), _ptr(tdist), n_rays, n1 - 1, levels, len(proposals), _ptr(directions), seed,
                            _ptr(rgb_target), charbonnier_padding, distortion_weight, distortion_power, distortion_premult, _ptr(out_grad),
                            _ptr(loss_sums))
    check(load().zf_train_final(ctypes.byref(a), _stream(stream)))
    return out_grad, grads, loss_sums


def composite_final(nerf_outputs, tdist, directions, background, pixel_indices, rgb, alpha=None, depth=None, use_median_depth: bool = False,
                    stream=None) -> None:
    """zf_composite_final into the given image buffers (alpha, depth optional)."""
    n_rays, n1 = tdist.shape
    a = zf_composite_final_args(_ptr(nerf_outputs), _ptr(tdist), n_rays, n1 - 1, _ptr(directions), _ptr(background), _ptr(pixel_indices), _ptr(rgb),
                                _ptr(alpha), _ptr(depth), 1 if use_median_depth else 0)
    check(load().zf_composite_final(ctypes.byref(a), _stream(stream)))


# shapes and dtypes of the packed NeRF MLP tensors the tensor-core kernel reads (zf_nerf_mlp_weights)
NERF_MLP_PACKED_SHAPES = {'density': ((64, 64), 'bfloat16'), 'density_bias': ((64,), 'float32'), 'combined': ((256, 96), 'bfloat16'),
                          'skip': ((16, 96), 'bfloat16'), 'view_1': ((256, 256), 'bfloat16'), 'view_1_bias': ((256,), 'float32'),
                          'view_2': ((256, 256), 'bfloat16'), 'view_2_bias': ((256,), 'float32'), 'rgb': ((16, 256), 'bfloat16')}


# bytes per sample of the training forward's record (zf_nerf_mlp_activations_size): v0, v1, v2 as [3, n, 256] bf16, their
# ReLU masks as [3, n, 8] uint32, h's as [n, 2] uint32
NERF_MLP_RECORD_BYTES_PER_SAMPLE = 3 * 256 * 2 + 3 * 8 * 4 + 2 * 4


def nerf_mlp_record_size(n: int) -> int:
    """Bytes of the training forward's record for n samples (zf_nerf_mlp_activations_size)."""
    return n * NERF_MLP_RECORD_BYTES_PER_SAMPLE


def _check_record(activations, n: int, on_device) -> None:
    import torch
    if not isinstance(activations, torch.Tensor) or not on_device(activations) or not activations.is_contiguous() \
            or activations.numel() * activations.element_size() < nerf_mlp_record_size(n):
        raise ValueError(f'activations must be a contiguous CUDA tensor of {nerf_mlp_record_size(n)} bytes (the training record of {n} samples)')


def check_nerf_mlp_forward_tc(features, inputs, packed: dict, outputs, status, require_cuda: bool = True, activations=None) -> None:
    """Raises ValueError unless the tensors have the shapes, dtypes and layouts the tensor-core kernel reads and writes
    (the C ABI sees only pointers and row strides, so a wrong shape here would make the kernel read or write out of
    bounds): features [n, >= 56] and inputs [n, >= 96] bf16 CUDA tensors with unit column stride, outputs a contiguous
    [n, 8] bf16 tensor, the packed weights as zipnerf_b200.nerf_mlp.pack gives them, status an int32 CUDA tensor.
    require_cuda=False checks the shapes of CPU tensors (host tests)."""
    import torch

    def on_device(t) -> bool:
        return t.is_cuda or not require_cuda
    tensors = {'features': features, 'inputs': inputs, 'outputs': outputs}
    for name, t in tensors.items():
        if not isinstance(t, torch.Tensor) or not on_device(t) or t.dtype != torch.bfloat16 or t.dim() != 2:
            raise ValueError(f'{name} must be a 2-d bf16 CUDA tensor')
        if t.stride(1) != 1:
            raise ValueError(f'{name} must have unit column stride')
    n = features.shape[0]
    if features.shape[1] < 56 or inputs.shape[1] < 96 or inputs.shape[0] != n:
        raise ValueError(f'features must be [n, >= 56] and inputs [n, >= 96] with the same n (got {tuple(features.shape)}, {tuple(inputs.shape)})')
    if tuple(outputs.shape) != (n, 8) or not outputs.is_contiguous():
        raise ValueError(f'outputs must be a contiguous [{n}, 8] tensor (got {tuple(outputs.shape)})')
    for name, (shape, dtype) in NERF_MLP_PACKED_SHAPES.items():
        t = packed.get(name)
        if not isinstance(t, torch.Tensor) or not on_device(t) or t.dtype != getattr(torch, dtype) or t.numel() != shape[0] * (shape[1] if len(shape) > 1 else 1) \
                or not t.is_contiguous():
            raise ValueError(f'packed[{name!r}] must be a contiguous {dtype} CUDA tensor of {shape} elements')
    if not isinstance(status, torch.Tensor) or not on_device(status) or status.dtype != torch.int32 or status.numel() < 1:
        raise ValueError('status must be an int32 CUDA tensor')
    if activations is not None:
        _check_record(activations, n, on_device)


def nerf_mlp_forward_tc(features, inputs, packed: dict, outputs, status, activations=None, stream=None) -> None:
    """zf_nerf_mlp_forward_tc: features [n, 56] and inputs [n, 96] bf16, packed as zipnerf_b200.nerf_mlp.pack gives it
    (the kernel's shapes), outputs [n, 8] bf16, status a device int32 the kernel sets on a timed-out wait; activations
    None (inference) or a contiguous tensor of nerf_mlp_record_size(n) bytes for the training record (v0, v1, v2 as
    [3, n, 256] bf16 at its start, then the ReLU masks). The tensors are checked first
    (check_nerf_mlp_forward_tc: ValueError on a mismatch)."""
    check_nerf_mlp_forward_tc(features, inputs, packed, outputs, status, activations=activations)
    w = zf_nerf_mlp_weights(*[packed[name].data_ptr() for name, _ in zf_nerf_mlp_weights._fields_])
    check(load().zf_nerf_mlp_forward_tc(_ptr(features), features.stride(0), _ptr(inputs), inputs.stride(0), ctypes.byref(w), _ptr(outputs),
                                        _ptr(activations), features.shape[0], _ptr(status), _stream(stream)))


# shapes of the transposed packed weights (zf_nerf_mlp_weights_t) and of the packed-weight gradients (zf_nerf_mlp_grads)
NERF_MLP_TRANSPOSED_SHAPES = {'rgb_t': (256, 16), 'view_2_t': (256, 256), 'view_1_t': (256, 256), 'combined_t': (96, 256), 'skip_t': (96, 16),
                              'density_t': (64, 64)}
NERF_MLP_GRAD_SHAPES = {'density': (64, 64), 'density_bias': (64,), 'combined': (256, 96), 'skip': (16, 96), 'view_1': (256, 256),
                        'view_1_bias': (256,), 'view_2': (256, 256), 'view_2_bias': (256,), 'rgb': (16, 256)}


def check_nerf_mlp_backward_tc(grad_outputs, features, inputs, activations, packed_t: dict, grad_features, grads: dict, workspace, status) -> None:
    """Raises ValueError unless the tensors have the shapes, dtypes and layouts the tensor-core backward reads and
    writes (its C ABI sees pointers and row strides only)."""
    import torch

    def cuda(t, dtype, what):
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != dtype:
            raise ValueError(f'{what} must be a {dtype} CUDA tensor')

    n = features.shape[0] if isinstance(features, torch.Tensor) and features.dim() == 2 else -1
    for t, width, what in ((grad_outputs, 8, 'grad_outputs'), (features, 56, 'features'), (inputs, 96, 'inputs'), (grad_features, 56, 'grad_features')):
        cuda(t, torch.bfloat16, what)
        if t.dim() != 2 or t.shape[0] != n or t.shape[1] < width or t.stride(1) != 1:
            raise ValueError(f'{what} must be [{n}, >= {width}] with unit column stride')
    if not grad_outputs.is_contiguous() or grad_outputs.shape[1] != 8:
        raise ValueError('grad_outputs must be a contiguous [n, 8] tensor')
    _check_record(activations, n, lambda t: t.is_cuda)
    for name, shape in NERF_MLP_TRANSPOSED_SHAPES.items():
        t = packed_t.get(name)
        cuda(t, torch.bfloat16, f'packed_t[{name!r}]')
        if tuple(t.shape) != shape or not t.is_contiguous():
            raise ValueError(f'packed_t[{name!r}] must be a contiguous {shape} tensor')
    for name, shape in NERF_MLP_GRAD_SHAPES.items():
        t = grads.get(name)
        cuda(t, torch.float32, f'grads[{name!r}]')
        if tuple(t.shape) != shape or not t.is_contiguous():
            raise ValueError(f'grads[{name!r}] must be a contiguous {shape} tensor')
    cuda(status, torch.int32, 'status')
    if not isinstance(workspace, torch.Tensor) or not workspace.is_cuda or workspace.numel() * workspace.element_size() < load().zf_nerf_mlp_backward_workspace_size(n):
        raise ValueError('workspace must be a CUDA tensor of zf_nerf_mlp_backward_workspace_size(n) bytes')


def nerf_mlp_backward_tc(grad_outputs, features, inputs, activations, packed_t: dict, grad_features, grads: dict, workspace, status, stream=None) -> None:
    """zf_nerf_mlp_backward_tc on PyTorch CUDA tensors (checked first: check_nerf_mlp_backward_tc)."""
    check_nerf_mlp_backward_tc(grad_outputs, features, inputs, activations, packed_t, grad_features, grads, workspace, status)
    w = zf_nerf_mlp_weights_t(*[packed_t[name].data_ptr() for name, _ in zf_nerf_mlp_weights_t._fields_])
    g = zf_nerf_mlp_grads(*[grads[name].data_ptr() for name, _ in zf_nerf_mlp_grads._fields_])
    check(load().zf_nerf_mlp_backward_tc(_ptr(grad_outputs), _ptr(features), features.stride(0), _ptr(inputs), inputs.stride(0), _ptr(activations),
                                         ctypes.byref(w), _ptr(grad_features), grad_features.stride(0), ctypes.byref(g), _ptr(workspace),
                                         workspace.numel() * workspace.element_size(), features.shape[0], _ptr(status), _stream(stream)))


def nerf_mlp_pack(params, targets: dict, stream=None) -> None:
    """zf_nerf_mlp_pack: the fp32 parameters (a CUDA tensor of at least zf_nerf_mlp_parameter_count() elements) into the
    given targets, device addresses by NERF_MLP_PACK_TARGETS name (missing names: not written); the caller sizes them
    (zipnerf_b200.nerf_mlp.NerfMlp lays them out in its packed buffer)."""
    import torch
    if not isinstance(params, torch.Tensor) or not params.is_cuda or params.dtype != torch.float32 or params.numel() < load().zf_nerf_mlp_parameter_count():
        raise ValueError('params must be a float32 CUDA tensor of the reference model widths\' parameter count')
    out = zf_nerf_mlp_packed(*[targets.get(name) for name in NERF_MLP_PACK_TARGETS])
    check(load().zf_nerf_mlp_pack(_ptr(params), ctypes.byref(out), _stream(stream)))


def nerf_mlp_unfold_grads(params, grads: dict, grad_params, stream=None) -> None:
    """zf_nerf_mlp_unfold_grads: grad_params (float32, the parameter layout) += the unfold of the packed-weight gradients
    (fp32 CUDA tensors of NERF_MLP_GRAD_SHAPES)."""
    import torch
    n = load().zf_nerf_mlp_parameter_count()
    for t, what in ((params, 'params'), (grad_params, 'grad_params')):
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != torch.float32 or t.numel() < n or not t.is_contiguous():
            raise ValueError(f'{what} must be a contiguous float32 CUDA tensor of at least {n} elements')
    for name, shape in NERF_MLP_GRAD_SHAPES.items():
        t = grads.get(name)
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != torch.float32 or tuple(t.shape) != shape or not t.is_contiguous():
            raise ValueError(f'grads[{name!r}] must be a contiguous float32 CUDA tensor of shape {shape}')
    g = zf_nerf_mlp_grads(*[grads[name].data_ptr() for name, _ in zf_nerf_mlp_grads._fields_])
    check(load().zf_nerf_mlp_unfold_grads(_ptr(params), ctypes.byref(g), _ptr(grad_params), _stream(stream)))


class CAdam:
    """A zf_adam over PyTorch CUDA tensors (params float32; grads float32 or float16), with the reference Adam's
    arguments (optimizer_api.h:14-24); keeps the tensors alive."""

    def __init__(self, params, grads, grad_scales, level_offsets, reg_weight, max_value, beta1, beta2, eps, magnitudes) -> None:
        import torch
        lib = load()
        self.tensors = (list(params), list(grads), magnitudes)
        self.regularization = torch.zeros((), device=params[0].device)
        self._offsets = [(_i64 * len(o))(*o) for o in level_offsets]
        buffers = (zf_adam_buffer * len(params))(*[
            zf_adam_buffer(p.data_ptr(), g.data_ptr(), 1 if g.dtype == torch.float16 else 0, p.numel(), s, self._offsets[i], len(level_offsets[i]))
            for i, (p, g, s) in enumerate(zip(params, grads, grad_scales))])
        handle = _p()
        check(lib.zf_adam_create(buffers, len(params), reg_weight, max_value, beta1, beta2, eps, _ptr(magnitudes), magnitudes.numel(),
                                 self.regularization.data_ptr(), ctypes.byref(handle)))
        self.handle = handle

    def __del__(self) -> None:
        if getattr(self, 'handle', None):
            load().zf_adam_destroy(self.handle)
            self.handle = None

    def step(self, lr: float, stream=None) -> None:
        check(load().zf_adam_step(self.handle, lr, _stream(stream)))

    def state(self, buffer: int):
        """(exp_avg, exp_avg_sq, steps): copies of one buffer's moments and the steps taken."""
        import torch
        m, v, steps = _p(), _p(), _i64()
        check(load().zf_adam_state(self.handle, buffer, ctypes.byref(m), ctypes.byref(v), ctypes.byref(steps)))
        n = self.tensors[0][buffer].numel()
        device = self.tensors[0][buffer].device
        return _device_floats(m.value, n, device).clone(), _device_floats(v.value, n, device).clone(), steps.value


def _device_floats(address: int, n: int, device):
    """A float32 tensor view of n floats of device memory at address (not owned)."""
    import torch

    class _View:
        __cuda_array_interface__ = {'shape': (n,), 'typestr': '<f4', 'data': (address, False), 'version': 3}

    return torch.as_tensor(_View(), device=device)

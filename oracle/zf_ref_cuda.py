"""ctypes binding of the reference's own featurization kernels compiled for sm_100a (TEST INFRASTRUCTURE ONLY).

oracle/ref_cuda/build.py compiles one library per grid layout (oracle/_ref/cuda/libzfref_<variant>.so) where the
reference sources exist; the libraries travel to the GPU box with oracle/_ref. The GPU tests use them as the bit-exact
checker of the product kernels, and bench.py's reference_cuda leg times them. Takes PyTorch CUDA tensors.
"""
from __future__ import annotations

import ctypes
import json
from pathlib import Path

REF_CUDA_DIR = Path(__file__).resolve().parent / '_ref' / 'cuda'

_p, _i64 = ctypes.c_void_p, ctypes.c_int64


def available_variants() -> dict:
    path = REF_CUDA_DIR / 'variants.json'
    if not path.exists():
        return {}
    return {name: layout for name, layout in json.loads(path.read_text()).items() if (REF_CUDA_DIR / f'libzfref_{name}.so').exists()}


def _ptr(t):
    return None if t is None or t.numel() == 0 else t.data_ptr()


def _stream(stream):
    import torch
    return (stream or torch.cuda.current_stream()).cuda_stream


class RefCuda:
    """The reference kernels of one layout variant (level, sizes, entries, n_features, mlp_width fixed at build)."""

    def __init__(self, variant: str) -> None:
        layouts = available_variants()
        if variant not in layouts:
            raise FileNotFoundError(f'reference kernel variant {variant} is not built (python oracle/ref_cuda/build.py)')
        self.layout = layouts[variant]
        self.lib = ctypes.CDLL(str(REF_CUDA_DIR / f'libzfref_{variant}.so'))
        self.lib.ref_forward.argtypes = [_p, _p, _p, _p, _i64, _i64, ctypes.c_longlong, ctypes.c_int, _p, _p, _p, _p, _p, _p, _p, _p, _p, ctypes.c_int,
                                         _p, ctypes.c_int, _p, ctypes.c_int, _p]
        self.lib.ref_backward.argtypes = [_p, _p, _p, _p, _i64, _i64, ctypes.c_longlong, _p, ctypes.c_int, _p, _p, _p]
        self.lib.ref_backward_mlp.argtypes = [_p, _p, _p, _p, _i64, _i64, ctypes.c_longlong, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p]
        self.lib.ref_debug.argtypes = [_p, _p, _p, _p, _i64, ctypes.c_longlong, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _p]
        n = (ctypes.c_int * 4)()
        self.lib.ref_layout(ctypes.byref(n, 0), ctypes.byref(n, 4), ctypes.byref(n, 8), ctypes.byref(n, 12))
        self.n_levels, self.n_features, self.mlp_width, self.n_fp32_grad_levels = list(n)
        self.n_output_features = self.n_levels * (self.n_features + 1)

    @staticmethod
    def _check(code: int, what: str) -> None:
        if code != 0:
            raise RuntimeError(f'reference {what} failed with CUDA error {code}')

    def forward(self, origins, directions, radii, tdist, pattern_seed, interleave, table, scale_magnitudes, w0=None, b0=None, w1=None, b1=None,
                raw_density=None, features_float=None, features_bf16=None, encoded_directions=None, nerf_inputs=None, stream=None) -> None:
        self._check(self.lib.ref_forward(_ptr(origins), _ptr(directions), _ptr(radii), _ptr(tdist), tdist.shape[0], tdist.shape[1] - 1, pattern_seed,
                                         int(bool(interleave)), _ptr(table), _ptr(scale_magnitudes), _ptr(w0), _ptr(b0), _ptr(w1), _ptr(b1),
                                         _ptr(raw_density), _ptr(features_float), _ptr(features_bf16),
                                         features_bf16.shape[1] if features_bf16 is not None and features_bf16.numel() else 0,
                                         _ptr(encoded_directions), encoded_directions.shape[1] if encoded_directions is not None else 0,
                                         _ptr(nerf_inputs), nerf_inputs.shape[1] if nerf_inputs is not None and nerf_inputs.numel() else 0,
                                         _stream(stream)), 'forward')

    def backward(self, origins, directions, radii, tdist, pattern_seed, grad_features, grad_table, grad_table_half, stream=None) -> None:
        self._check(self.lib.ref_backward(_ptr(origins), _ptr(directions), _ptr(radii), _ptr(tdist), tdist.shape[0], tdist.shape[1] - 1, pattern_seed,
                                          _ptr(grad_features), grad_features.stride(0), _ptr(grad_table), _ptr(grad_table_half), _stream(stream)),
                    'backward')

    def backward_mlp(self, origins, directions, radii, tdist, pattern_seed, features, grad_raw_density, w0, b0, w1, grad_table, grad_w0, grad_b0,
                     grad_w1, grad_b1, stream=None) -> None:
        self._check(self.lib.ref_backward_mlp(_ptr(origins), _ptr(directions), _ptr(radii), _ptr(tdist), tdist.shape[0], tdist.shape[1] - 1,
                                              pattern_seed, _ptr(features), _ptr(grad_raw_density), _ptr(w0), _ptr(b0), _ptr(w1), _ptr(grad_table),
                                              _ptr(grad_w0), _ptr(grad_b0), _ptr(grad_w1), _ptr(grad_b1), _stream(stream)), 'backward_mlp')

    def debug(self, origins, directions, radii, tdist, pattern_seed, samples, stream=None) -> dict:
        import torch
        n, L, dev = samples.numel(), self.n_levels, samples.device
        out = {'x': torch.zeros(n, 6, 3, device=dev), 'scale': torch.zeros(n, 6, device=dev),
               'contracted': torch.zeros(n, 6, dtype=torch.int32, device=dev), 'x_check': torch.zeros(n, 6, 3, device=dev),
               'n_groups': torch.zeros(n, L, dtype=torch.int32, device=dev), 'rows': torch.zeros(n, L, 6, 8, dtype=torch.int32, device=dev),
               'weights': torch.zeros(n, L, 6, 8, device=dev)}
        self._check(self.lib.ref_debug(_ptr(origins), _ptr(directions), _ptr(radii), _ptr(tdist), tdist.shape[1] - 1, pattern_seed, _ptr(samples), n,
                                       _ptr(out['x']), _ptr(out['scale']), _ptr(out['contracted']), _ptr(out['x_check']), _ptr(out['n_groups']),
                                       _ptr(out['rows']), _ptr(out['weights']), _stream(stream)), 'debug')
        out['rows'] = out['rows'].to(torch.int64) & 0xFFFFFFFF
        return out

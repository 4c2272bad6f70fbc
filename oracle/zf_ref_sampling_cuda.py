"""ctypes binding of the reference's own sampling, final-level and Adam kernels compiled for sm_100a (TEST
INFRASTRUCTURE ONLY).

oracle/ref_cuda/build.py compiles B/sampling/src/sampling_api.cu and B/optimizer/src/optimizer_api.cu (unmodified, with
the launchers of oracle/ref_cuda/ref_sampling.cu) into oracle/_ref/cuda/libzfref_sampling.so, which travels to the GPU
box with oracle/_ref. The GPU tests use it as the bit-exact checker of the product's sampling and Adam kernels, and
bench.py's rows leg times both. Takes PyTorch CUDA tensors; allocates outputs as the reference's
wrappers do (B/ = ZipNeRFCudaBackend/ZipNeRFCudaBackend/).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB = Path(__file__).resolve().parent / '_ref' / 'cuda' / 'libzfref_sampling.so'

_p, _i64, _i32, _f32, _f64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_double


def available() -> bool:
    return LIB.exists()


def _ptr(t):
    return None if t is None or t.numel() == 0 else t.data_ptr()


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def _warp(values):
    import torch
    return torch.tensor([float(v) for v in values], dtype=torch.float32)


def _check(code: int, what: str) -> None:
    if code != 0:
        raise RuntimeError(f'reference {what} failed with CUDA error {code}')


class RefSamplingCuda:
    def __init__(self) -> None:
        if not LIB.exists():
            raise FileNotFoundError(f'{LIB} is not built (python oracle/ref_cuda/build.py)')
        lib = ctypes.CDLL(str(LIB))
        lib.ref_generate_rays.argtypes = [_i64, _i32, _p, _i32, _p, _p, _p, _p, _p, _p, _i64, _i32, _i32, _p, _p, _p, _p, _p, _p, _p, _p, _p]
        lib.ref_view_rays.argtypes = [_p, _i32, _p, _p, _f32, _i32, _i32, _p, _p, _p, _p, _p, _p, _p, _p]
        lib.ref_initialize_rays.argtypes = [_i64, _p, _i32, _i32, _i32, _p, _p, _p, _p, _p]
        lib.ref_sample_uniforms.argtypes = [_i64, _i64, _i64, _p, _p]
        lib.ref_composite_and_resample.argtypes = [_p, _p, _p, _p, _i32, _i32, _f32, _i32, _i64, _i32, _p, _p, _p, _p, _p]
        lib.ref_train_final.argtypes = [_p, _p, _p, _i32, _i32, _i32, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p, _f32, _f32, _f32, _f32, _p, _p, _p]
        lib.ref_composite_final.argtypes = [_p, _p, _p, _p, _p, _i32, _i32, _p, _p, _p, _i32, _p]
        lib.ref_adam_step.argtypes = [_i32, _p, _p, _p, _p, _p, _p, _p, _p, _p, _f64, _f64, _f64, _f64, _f64, _i64, _f64, _p, _p, _p, _p, _p]
        self.lib = lib

    @staticmethod
    def width(degree: int) -> int:
        return (3 + 6 * degree + 1 + 7) // 8 * 8

    def initialize_rays(self, seed, directions, degree, n_samples, warp):
        import torch
        n, dev = directions.shape[0], directions.device
        encoded = torch.empty(n, self.width(degree), dtype=torch.bfloat16, device=dev)
        sdist, tdist = torch.empty(n, n_samples + 1, device=dev), torch.empty(n, n_samples + 1, device=dev)
        w = _warp(warp)
        _check(self.lib.ref_initialize_rays(seed, _ptr(directions), n, degree, n_samples, w.data_ptr(), _ptr(encoded), _ptr(sdist), _ptr(tdist),
                                            _stream()), 'initialize_rays')
        return encoded, sdist, tdist

    def view_rays(self, pixel_indices, local_directions, c2w, radius, degree, n_samples, warp):
        import torch
        n, dev = pixel_indices.numel(), local_directions.device
        origins, directions, radii = torch.empty(n, 3, device=dev), torch.empty(n, 3, device=dev), torch.empty(n, device=dev)
        encoded = torch.empty(n, self.width(degree), dtype=torch.bfloat16, device=dev)
        sdist, tdist = torch.empty(n, n_samples + 1, device=dev), torch.empty(n, n_samples + 1, device=dev)
        w = _warp(warp)
        _check(self.lib.ref_view_rays(_ptr(pixel_indices), n, _ptr(local_directions), _ptr(c2w), radius, degree, n_samples, w.data_ptr(),
                                      _ptr(origins), _ptr(directions), _ptr(radii), _ptr(encoded), _ptr(sdist), _ptr(tdist), _stream()), 'view_rays')
        return origins, directions, radii, encoded, sdist, tdist

    def generate_rays(self, seed, n_rays, view_offsets, view_cameras, camera_offsets, local_directions, c2w, camera_radii, pool_rgb, degree,
                      n_samples, warp):
        import torch
        dev = local_directions.device
        origins, directions, rgb = (torch.empty(n_rays, 3, device=dev) for _ in range(3))
        radii = torch.empty(n_rays, device=dev)
        encoded = torch.empty(n_rays, self.width(degree), dtype=torch.bfloat16, device=dev)
        sdist, tdist = torch.empty(n_rays, n_samples + 1, device=dev), torch.empty(n_rays, n_samples + 1, device=dev)
        w = _warp(warp)
        _check(self.lib.ref_generate_rays(seed, n_rays, _ptr(view_offsets), view_cameras.numel(), _ptr(view_cameras), _ptr(camera_offsets),
                                          _ptr(local_directions), _ptr(c2w), _ptr(camera_radii), _ptr(pool_rgb), pool_rgb.shape[0], degree, n_samples,
                                          w.data_ptr(), _ptr(origins), _ptr(directions), _ptr(radii), _ptr(rgb), _ptr(encoded), _ptr(sdist),
                                          _ptr(tdist), _stream()), 'generate_rays')
        return origins, directions, radii, rgb, encoded, sdist, tdist

    def sample_uniforms(self, seed, stream, n, device='cuda'):
        import torch
        values = torch.empty(n, device=device)
        _check(self.lib.ref_sample_uniforms(seed, stream, n, _ptr(values), _stream()), 'sample_uniforms')
        return values

    def composite_and_resample(self, raw_density, sdist, tdist, directions, anneal, n_samples, seed, next_level, warp):
        import torch
        n_rays, n = raw_density.shape
        dev = raw_density.device
        weights = torch.empty_like(raw_density)
        sdist_next, tdist_next = torch.empty(n_rays, n_samples + 1, device=dev), torch.empty(n_rays, n_samples + 1, device=dev)
        w = _warp(warp)
        _check(self.lib.ref_composite_and_resample(_ptr(raw_density), _ptr(sdist), _ptr(tdist), _ptr(directions), n_rays, n, anneal, n_samples, seed,
                                                   next_level, w.data_ptr(), _ptr(weights), _ptr(sdist_next), _ptr(tdist_next), _stream()),
               'composite_and_resample')
        return weights, sdist_next, tdist_next

    def train_final(self, nerf_outputs, sdist, tdist, proposals, directions, seed, rgb_target, charbonnier_padding, distortion_weight,
                    distortion_power, distortion_premult, compute_loss_sums=True):
        """train_final_wrapper (sampling_api.cu:580-645); proposals: dicts of raw_density, sdist, tdist, weights,
        interlevel_weight, interlevel_blur. Returns (nerf_outputs_grad, [proposal gradients], loss_sums or None)."""
        import torch
        n_rays, n1 = tdist.shape
        k = len(proposals)
        grads = [torch.empty_like(p['raw_density']) for p in proposals]
        arr = lambda ctype, values: (ctype * max(k, 1))(*values)  # noqa: E731
        out_grad = torch.empty_like(nerf_outputs)
        loss_sums = torch.zeros(4, device=tdist.device) if compute_loss_sums else None
        _check(self.lib.ref_train_final(
            _ptr(nerf_outputs), _ptr(sdist), _ptr(tdist), n_rays, n1 - 1, k, arr(_i32, [p['raw_density'].shape[1] for p in proposals]),
            arr(_p, [_ptr(p['raw_density']) for p in proposals]), arr(_p, [_ptr(p['sdist']) for p in proposals]),
            arr(_p, [_ptr(p['tdist']) for p in proposals]), arr(_p, [_ptr(p['weights']) for p in proposals]), arr(_p, [_ptr(g) for g in grads]),
            arr(_f32, [p['interlevel_weight'] for p in proposals]), arr(_f32, [p['interlevel_blur'] for p in proposals]), _ptr(directions), seed,
            _ptr(rgb_target), charbonnier_padding, distortion_weight, distortion_power, distortion_premult, _ptr(out_grad), _ptr(loss_sums),
            _stream()), 'train_final')
        return out_grad, grads, loss_sums

    def composite_final(self, nerf_outputs, tdist, directions, background, pixel_indices, rgb, alpha=None, depth=None, use_median_depth=False):
        n_rays, n1 = tdist.shape
        _check(self.lib.ref_composite_final(_ptr(nerf_outputs), _ptr(tdist), _ptr(directions), _ptr(background), _ptr(pixel_indices), n_rays, n1 - 1,
                                            _ptr(rgb), _ptr(alpha), _ptr(depth), 1 if use_median_depth else 0, _stream()), 'composite_final')


class RefAdamCuda:
    """The state of one reference Adam object (optimizer_api.cu:132-158) over PyTorch tensors, stepped by the
    reference kernel (optimizer_api.cu:160-220)."""

    def __init__(self, ref: RefSamplingCuda, params, grads, grad_scales, level_offsets, reg_weight, max_value, beta1, beta2, eps, magnitudes):
        import torch
        self.lib = ref.lib
        self.params, self.grads, self.magnitudes = list(params), list(grads), magnitudes
        self.exp_avgs = [torch.zeros_like(p) for p in params]
        self.exp_avg_sqs = [torch.zeros_like(p) for p in params]
        self.regularization = torch.zeros((), device=params[0].device)
        self.level_sums = torch.zeros(max(sum(max(len(o) - 1, 0) for o in level_offsets), 1), dtype=torch.float64, device=params[0].device)
        self.counter = torch.zeros(1, dtype=torch.int32, device=params[0].device)
        n = len(params)
        self._arrays = {
            'params': (_p * n)(*[p.data_ptr() for p in params]), 'grads': (_p * n)(*[g.data_ptr() for g in grads]),
            'half': (_i32 * n)(*[1 if g.dtype == torch.float16 else 0 for g in grads]),
            'm': (_p * n)(*[t.data_ptr() for t in self.exp_avgs]), 'v': (_p * n)(*[t.data_ptr() for t in self.exp_avg_sqs]),
            'numels': (_i64 * n)(*[p.numel() for p in params]), 'scales': (_f64 * n)(*grad_scales),
            'offsets': (_i64 * max(sum(len(o) for o in level_offsets), 1))(*[v for o in level_offsets for v in o]),
            'n_offsets': (_i32 * n)(*[len(o) for o in level_offsets]),
        }
        self.hyper = (reg_weight, max_value, beta1, beta2, eps)
        self.steps = 0

    def step(self, lr: float) -> None:
        self.steps += 1
        a = self._arrays
        reg_weight, max_value, beta1, beta2, eps = self.hyper
        _check(self.lib.ref_adam_step(len(self.params), a['params'], a['grads'], a['half'], a['m'], a['v'], a['numels'], a['scales'], a['offsets'],
                                      a['n_offsets'], reg_weight, max_value, beta1, beta2, eps, self.steps, lr, _ptr(self.magnitudes),
                                      self.regularization.data_ptr(), self.level_sums.data_ptr(), self.counter.data_ptr(), _stream()), 'adam_step')

"""ctypes bindings of the CPU checkers (TEST INFRASTRUCTURE ONLY).

* ``Oracle``  -- the C restatement of the reference featurization (``oracle/zf_oracle.c``, built into
  ``oracle/_build/libzf_oracle.so``).
* ``RefCpu``  -- the reference's own featurization header compiled for the host (``oracle/ref_cpu``, built into
  ``oracle/_ref/libzf_ref_cpu.so`` where the reference sources are present).

Both take and return numpy arrays and share one call signature, so tests can run the same case through either. Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs use this module; the product never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
ORACLE_LIB = ORACLE_DIR / '_build' / 'libzf_oracle.so'
REF_CPU_LIB = ORACLE_DIR / '_ref' / 'libzf_ref_cpu.so'
MAX_LEVELS = 32
N_MULTISAMPLES = 6
NERF_GRID_GRAD_SCALE = 1048576.0  # zipnerf_config.h:12


def build(reference: bool = False) -> None:
    """Builds the oracle library (and the host build of the reference when ``reference`` and its sources exist)."""
    targets = ['all'] + (['ref'] if reference else [])
    subprocess.run(['make', '-s', '-C', str(ORACLE_DIR), *targets], check=True)


def _ptr(array, ctype=ctypes.c_float):
    if array is None:
        return None
    assert array.flags['C_CONTIGUOUS'], 'oracle arrays must be contiguous'
    return array.ctypes.data_as(ctypes.POINTER(ctype))


class _Grid(ctypes.Structure):
    _fields_ = [
        ('level', ctypes.c_int), ('n_levels', ctypes.c_int), ('n_features', ctypes.c_int), ('mlp_width', ctypes.c_int),
        ('n_fp32_grad_levels', ctypes.c_int),
        ('sizes', ctypes.c_int64 * MAX_LEVELS), ('entries', ctypes.c_int64 * MAX_LEVELS),
        ('offsets', ctypes.c_int64 * (MAX_LEVELS + 1)), ('hashed', ctypes.c_int * MAX_LEVELS),
    ]


class GridSpec:
    """Layout of one featurizer (featurizer.cu:145-155)."""

    def __init__(self, level: int, sizes, entries, n_features: int, mlp_width: int) -> None:
        self.level, self.sizes, self.entries = int(level), [int(s) for s in sizes], [int(e) for e in entries]
        self.n_features, self.mlp_width = int(n_features), int(mlp_width)
        self.n_levels = len(self.sizes)
        self.offsets = np.cumsum([0] + self.entries).tolist()
        self.n_output_features = self.n_levels * (self.n_features + 1)
        n = 0
        while n < self.n_levels and self.entries[n] < (1 << 20):
            n += 1
        self.n_fp32_grad_levels = n
        self.n_fp32_grad_rows = self.offsets[n]
        self.n_rows = self.offsets[-1]


class _Checker:
    """Common call layer: subclasses bind the library's functions."""

    lib: ctypes.CDLL

    def forward(self, grid: GridSpec, origins, directions, radii, tdist, pattern_seed: int, table, scale_magnitudes,
                mlp=None, raw_density=False, features_float=False, features_bf16_width=0, encoded_directions=None,
                nerf_inputs_width=0, n_threads: int = 1) -> dict:
        n_rays, n_intervals = tdist.shape[0], tdist.shape[1] - 1
        n_samples, n_out = n_rays * n_intervals, grid.n_output_features
        out = {}
        if raw_density:
            out['raw_density'] = np.zeros((n_rays, n_intervals), np.float32)
        if features_float:
            out['features_float'] = np.zeros((n_samples, n_out), np.float32)
        if features_bf16_width:
            out['features_bf16'] = np.full((n_samples, features_bf16_width), 0xFFFF, np.uint16)
        if nerf_inputs_width:
            out['nerf_inputs'] = np.zeros((n_samples, nerf_inputs_width), np.uint16)
        w0, b0, w1, b1 = mlp if mlp is not None else (None,) * 4
        encoded_width = encoded_directions.shape[1] if encoded_directions is not None else 0
        self._forward(grid, n_rays, n_intervals, origins, directions, radii, tdist, pattern_seed, table, scale_magnitudes,
                      w0, b0, w1, b1, out.get('raw_density'), out.get('features_float'), out.get('features_bf16'),
                      features_bf16_width, encoded_directions, encoded_width, out.get('nerf_inputs'), nerf_inputs_width,
                      n_threads)
        return out

    def backward(self, grid: GridSpec, origins, directions, radii, tdist, pattern_seed: int, grad_features_bf16,
                 grad_table=None, grad_table_half=None, n_threads: int = 1):
        """grad_features_bf16: uint16 [n_samples, >= n_out] (bf16 bits). Returns (fp32 grads, fp16 grads as uint16)."""
        n_rays, n_intervals = tdist.shape[0], tdist.shape[1] - 1
        F = grid.n_features
        if grad_table is None:
            grad_table = np.zeros(grid.n_fp32_grad_rows * F, np.float32)
        if grad_table_half is None:
            grad_table_half = np.zeros((grid.n_rows - grid.n_fp32_grad_rows) * F, np.uint16)
        self._backward(grid, n_rays, n_intervals, origins, directions, radii, tdist, pattern_seed, grad_features_bf16,
                       grad_features_bf16.shape[1], NERF_GRID_GRAD_SCALE, grad_table, grad_table_half, n_threads)
        return grad_table, grad_table_half

    def backward_mlp(self, grid: GridSpec, origins, directions, radii, tdist, pattern_seed: int, features, grad_raw_density,
                     w0, b0, w1, n_threads: int = 1, out: dict | None = None) -> dict:
        """Accumulates into ``out`` (grad_table, grad_w0, grad_b0, grad_w1, grad_b1) when given, else into zeros."""
        n_rays, n_intervals = tdist.shape[0], tdist.shape[1] - 1
        W, n_out = grid.mlp_width, grid.n_output_features
        if out is None:
            out = {'grad_table': np.zeros(grid.n_rows * grid.n_features, np.float32), 'grad_w0': np.zeros((W, n_out), np.float32),
                   'grad_b0': np.zeros(W, np.float32), 'grad_w1': np.zeros(W, np.float32), 'grad_b1': np.zeros(1, np.float32)}
        self._backward_mlp(grid, n_rays, n_intervals, origins, directions, radii, tdist, pattern_seed, features,
                           grad_raw_density, w0, b0, w1, out['grad_table'], out['grad_w0'], out['grad_b0'], out['grad_w1'],
                           out['grad_b1'], n_threads)
        return out


class Oracle(_Checker):
    """The C restatement (zf_oracle.c)."""

    def __init__(self) -> None:
        if not ORACLE_LIB.exists():
            build()
        self.lib = ctypes.CDLL(str(ORACLE_LIB))
        self.lib.zfo_grid_init.restype = ctypes.c_int

    def _grid(self, grid: GridSpec) -> _Grid:
        g = _Grid()
        n = grid.n_levels
        rc = self.lib.zfo_grid_init(ctypes.byref(g), grid.level, (ctypes.c_int64 * n)(*grid.sizes),
                                    (ctypes.c_int64 * n)(*grid.entries), n, grid.n_features, grid.mlp_width)
        assert rc == 0, 'invalid grid layout'
        return g

    def _forward(self, grid, n_rays, n_intervals, origins, directions, radii, tdist, seed, table, mags, w0, b0, w1, b1,
                 raw, ff, fb, fb_width, enc, enc_width, inputs, inputs_width, n_threads):
        g = self._grid(grid)
        u16 = ctypes.c_uint16
        self.lib.zfo_forward(ctypes.byref(g), ctypes.c_int64(n_rays), ctypes.c_int64(n_intervals), _ptr(origins), _ptr(directions),
                             _ptr(radii), _ptr(tdist), ctypes.c_int64(seed), _ptr(table), _ptr(mags), _ptr(w0), _ptr(b0), _ptr(w1),
                             _ptr(b1), _ptr(raw), _ptr(ff), _ptr(fb, u16), ctypes.c_int64(fb_width), _ptr(enc, u16),
                             ctypes.c_int64(enc_width), _ptr(inputs, u16), ctypes.c_int64(inputs_width), ctypes.c_int(n_threads))

    def _backward(self, grid, n_rays, n_intervals, origins, directions, radii, tdist, seed, grad, stride, grad_scale, g32, g16,
                  n_threads):
        g = self._grid(grid)
        self.lib.zfo_backward(ctypes.byref(g), ctypes.c_int64(n_rays), ctypes.c_int64(n_intervals), _ptr(origins), _ptr(directions),
                              _ptr(radii), _ptr(tdist), ctypes.c_int64(seed), _ptr(grad, ctypes.c_uint16), ctypes.c_int64(stride),
                              ctypes.c_float(grad_scale), _ptr(g32), _ptr(g16, ctypes.c_uint16))

    def _backward_mlp(self, grid, n_rays, n_intervals, origins, directions, radii, tdist, seed, features, grad_raw, w0, b0, w1,
                      gt, gw0, gb0, gw1, gb1, n_threads):
        g = self._grid(grid)
        self.lib.zfo_backward_mlp(ctypes.byref(g), ctypes.c_int64(n_rays), ctypes.c_int64(n_intervals), _ptr(origins),
                                  _ptr(directions), _ptr(radii), _ptr(tdist), ctypes.c_int64(seed), _ptr(features), _ptr(grad_raw),
                                  _ptr(w0), _ptr(b0), _ptr(w1), _ptr(gt), _ptr(gw0), _ptr(gb0), _ptr(gw1), _ptr(gb1))

    def debug_interval(self, grid: GridSpec, origins, directions, radii, tdist, pattern_seed: int, sample_idx: int) -> dict:
        g = self._grid(grid)
        L = grid.n_levels
        out = {'x': np.zeros((N_MULTISAMPLES, 3), np.float32), 'scale': np.zeros(N_MULTISAMPLES, np.float32),
               'contracted': np.zeros(N_MULTISAMPLES, np.int32), 'n_groups': np.zeros(L, np.int32),
               'cells': np.zeros((L, N_MULTISAMPLES, 3), np.int32), 'rows': np.zeros((L, N_MULTISAMPLES, 8), np.uint32),
               'weights': np.zeros((L, N_MULTISAMPLES, 8), np.float32)}
        n_intervals = tdist.shape[1] - 1
        i32 = ctypes.c_int32
        self.lib.zfo_debug_interval(ctypes.byref(g), ctypes.c_int64(n_intervals), _ptr(origins), _ptr(directions), _ptr(radii),
                                    _ptr(tdist), ctypes.c_int64(pattern_seed), ctypes.c_int64(sample_idx), _ptr(out['x']),
                                    _ptr(out['scale']), _ptr(out['contracted'], i32), _ptr(out['n_groups'], i32),
                                    _ptr(out['cells'], i32), _ptr(out['rows'], ctypes.c_uint32), _ptr(out['weights']))
        return out


class RefCpu(_Checker):
    """The reference's featurization header compiled for the host (oracle/ref_cpu)."""

    def __init__(self) -> None:
        if not REF_CPU_LIB.exists():
            raise FileNotFoundError(f'{REF_CPU_LIB} is not built (make -C oracle ref, where the reference sources exist)')
        self.lib = ctypes.CDLL(str(REF_CPU_LIB))

    @staticmethod
    def available() -> bool:
        return REF_CPU_LIB.exists()

    @staticmethod
    def _layout(grid: GridSpec):
        n = grid.n_levels
        return (ctypes.c_int(grid.level), (ctypes.c_int64 * n)(*grid.sizes), (ctypes.c_int64 * n)(*grid.entries), ctypes.c_int(n),
                ctypes.c_int(grid.n_features))

    def _forward(self, grid, n_rays, n_intervals, origins, directions, radii, tdist, seed, table, mags, w0, b0, w1, b1,
                 raw, ff, fb, fb_width, enc, enc_width, inputs, inputs_width, n_threads):
        u16 = ctypes.c_uint16
        rc = self.lib.zfr_forward(*self._layout(grid), ctypes.c_int(grid.mlp_width), ctypes.c_int64(n_rays), ctypes.c_int64(n_intervals),
                                  _ptr(origins), _ptr(directions), _ptr(radii), _ptr(tdist), ctypes.c_int64(seed), _ptr(table),
                                  _ptr(mags), _ptr(w0), _ptr(b0), _ptr(w1), _ptr(b1), _ptr(raw), _ptr(ff), _ptr(fb, u16),
                                  ctypes.c_int64(fb_width), _ptr(enc, u16), ctypes.c_int64(enc_width), _ptr(inputs, u16),
                                  ctypes.c_int64(inputs_width), ctypes.c_int(n_threads))
        assert rc == 0

    def _backward(self, grid, n_rays, n_intervals, origins, directions, radii, tdist, seed, grad, stride, grad_scale, g32, g16,
                  n_threads):
        rc = self.lib.zfr_backward(*self._layout(grid), ctypes.c_int64(n_rays), ctypes.c_int64(n_intervals), _ptr(origins),
                                   _ptr(directions), _ptr(radii), _ptr(tdist), ctypes.c_int64(seed), _ptr(grad, ctypes.c_uint16),
                                   ctypes.c_int64(stride), ctypes.c_float(grad_scale), _ptr(g32), _ptr(g16, ctypes.c_uint16),
                                   ctypes.c_int(n_threads))
        assert rc == 0

    def _backward_mlp(self, grid, n_rays, n_intervals, origins, directions, radii, tdist, seed, features, grad_raw, w0, b0, w1,
                      gt, gw0, gb0, gw1, gb1, n_threads):
        rc = self.lib.zfr_backward_mlp(*self._layout(grid), ctypes.c_int(grid.mlp_width), ctypes.c_int64(n_rays),
                                       ctypes.c_int64(n_intervals), _ptr(origins), _ptr(directions), _ptr(radii), _ptr(tdist),
                                       ctypes.c_int64(seed), _ptr(features), _ptr(grad_raw), _ptr(w0), _ptr(b0), _ptr(w1), _ptr(gt),
                                       _ptr(gw0), _ptr(gb0), _ptr(gw1), _ptr(gb1), ctypes.c_int(n_threads))
        assert rc == 0

    def debug_interval(self, grid: GridSpec, origins, directions, radii, tdist, pattern_seed: int, sample_idx: int) -> dict:
        L = grid.n_levels
        out = {'x': np.zeros((N_MULTISAMPLES, 3), np.float32), 'scale': np.zeros(N_MULTISAMPLES, np.float32),
               'n_groups': np.zeros(L, np.int32), 'rows': np.zeros((L, N_MULTISAMPLES, 8), np.uint32),
               'weights': np.zeros((L, N_MULTISAMPLES, 8), np.float32)}
        rc = self.lib.zfr_debug_interval(*self._layout(grid), ctypes.c_int64(tdist.shape[1] - 1), _ptr(origins), _ptr(directions),
                                         _ptr(radii), _ptr(tdist), ctypes.c_int64(pattern_seed), ctypes.c_int64(sample_idx),
                                         _ptr(out['x']), _ptr(out['scale']), _ptr(out['n_groups'], ctypes.c_int32),
                                         _ptr(out['rows'], ctypes.c_uint32), _ptr(out['weights']))
        assert rc == 0
        return out


def n_threads_default() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, 'sched_getaffinity') else (os.cpu_count() or 1)

"""Compiles the reference's CUDA kernels ahead of time for the GPU checks (TEST INFRASTRUCTURE ONLY).

For each layout variant below this writes the preamble that the reference's host code generates before runtime
compilation (featurizer.cu:157-184: JIT_* constants and the per-level layout functions; written here by this script
from the layout, not copied) and compiles oracle/ref_cuda/ref_cuda.cu with the reference's kernel sources included
from where they lie, with the reference's compile options (--use_fast_math, rtc_kernel.cu:49), for sm_100a, into
oracle/_ref/cuda/libzfref_<variant>.so. It also compiles the reference's sampling and Adam kernels with the launchers of
oracle/ref_cuda/ref_sampling.cu into oracle/_ref/cuda/libzfref_sampling.so. Needs the reference sources (their root in the REFERENCE_ROOT environment
variable when not at the default mount); the built libraries are shipped with the rest of oracle/_ref.

    python oracle/ref_cuda/build.py [--jobs N]
"""
from __future__ import annotations

import argparse
import concurrent.futures
import json
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE.parent / '_ref' / 'cuda'
# the reference checkout: REFERENCE_ROOT, else a sibling directory 'reference' of this repository
REFERENCE_ROOT = Path(os.environ.get('REFERENCE_ROOT', str(HERE.parent.parent.parent / 'reference')))
BACKEND = REFERENCE_ROOT / 'ZipNeRFCudaBackend' / 'ZipNeRFCudaBackend'
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')
MIN_HALF_GRAD_ENTRIES = 1 << 20


def geometric(n_levels, log2_size, base, finest):
    scale = (finest / base) ** (1.0 / (n_levels - 1))
    sizes = [round(base * scale ** level) for level in range(n_levels)]
    return sizes, [min(s ** 3, 2 ** log2_size) for s in sizes]


def variants() -> dict:
    """name -> (level, sizes, entries, n_features, mlp_width): the layouts of the parity cases and of config 2."""
    out = {}
    for features in [1, 2, 3, 4]:
        out[f'grids_F{features}'] = (2, [2, 4, 128], [8, 64, 1 << 20], features, 0)
    for n_levels in [6, 8]:
        out[f'proposals_L{n_levels}'] = (0, [2 ** (i + 1) for i in range(n_levels)], [min(2 ** (3 * (i + 1)), 4096) for i in range(n_levels)], 1, 64)
    out['config1'] = (2, *geometric(10, 19, 16, 2048), 4, 0)
    out['config2_nerf'] = (2, *geometric(10, 21, 16, 8192), 4, 0)
    out['config2_prop0'] = (0, *geometric(10, 21, 16, 512), 1, 64)
    out['config2_prop1'] = (1, *geometric(10, 21, 16, 512), 1, 64)
    out['config5'] = (2, *geometric(12, 22, 16, 16384), 4, 0)
    return out


def preamble(level, sizes, entries, n_features, mlp_width) -> str:
    """The JIT preamble of featurizer.cu:157-184 for one layout (integer typedefs come from <cstdint> here; the switches'
    unreachable default case falls through to the final return instead of stopping the kernel)."""
    n_levels = len(sizes)
    offsets = [0]
    for e in entries:
        offsets.append(offsets[-1] + e)
    n_fp32 = 0
    while n_fp32 < n_levels and entries[n_fp32] < MIN_HALF_GRAD_ENTRIES:
        n_fp32 += 1
    lines = [f'#define JIT_N_LEVELS {n_levels}u', f'#define JIT_N_FEATURES {n_features}u', f'#define JIT_MLP_WIDTH {mlp_width}u',
             f'#define JIT_N_FP32_GRAD_LEVELS {n_fp32}u', '#define JIT_PRECONDITION_SCALING 10.000000000000000f', '#define JIT_BLOCK_SIZE 128u',
             f'#define JIT_PATTERN_STREAM {16 + level}ull', 'namespace zipnerf { namespace config {']

    def switch(name, type_, values):
        lines.append(f'__device__ inline {type_} {name}(const uint32_t level) {{')
        lines.append('    switch (level) {')
        for i, v in enumerate(values):
            lines.append(f'        case {i}: return {v};')
        lines.append('        default: break;')  # unreachable (every level index is below JIT_N_LEVELS)
        lines.append('    }')
        lines.append('    return 0;')
        lines.append('}')

    switch('level_size', 'uint32_t', [f'{s}u' for s in sizes])
    switch('level_entries', 'uint32_t', [f'{e}u' for e in entries])
    switch('level_offset', 'uint32_t', [f'{o}u' for o in offsets[:-1]])
    switch('level_hashed', 'bool', ['true' if s ** 3 > e else 'false' for s, e in zip(sizes, entries)])
    lines.append('} }')
    return '\n'.join(lines) + '\n'


def build_variant(name: str, layout) -> Path:
    directory = OUT / name
    directory.mkdir(parents=True, exist_ok=True)
    header = directory / 'preamble.cuh'
    header.write_text(preamble(*layout))
    target = OUT / f'libzfref_{name}.so'
    sources = [HERE / 'ref_cuda.cu', header] + sorted((BACKEND / 'featurization' / 'rtc').glob('*')) + [BACKEND / 'common' / 'include' / 'random.cuh']
    if target.exists() and all(s.stat().st_mtime <= target.stat().st_mtime for s in sources):
        return target
    cmd = [NVCC, '-gencode', 'arch=compute_100a,code=sm_100a', '-O3', '--use_fast_math', '-std=c++17', '-lineinfo', '-shared', '-Xcompiler', '-fPIC',
           '-Xcompiler', '-fvisibility=hidden', f'-DZF_REF_PREAMBLE="{header}"', f'-I{BACKEND / "featurization" / "rtc"}',
           f'-I{BACKEND / "common" / "include"}', str(HERE / 'ref_cuda.cu'), '-o', str(target)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        sys.stderr.write(result.stdout + result.stderr)
        raise RuntimeError(f'compiling the reference kernels of {name} failed')
    return target


def build_sampling() -> Path:
    """The reference's sampling and Adam kernels (sampling_api.cu, optimizer_api.cu) with the launchers of
    ref_sampling.cu, against the placeholder torch headers of torch_stub/, with the reference's nvcc options
    (setup.py:28-34) for sm_100a -> libzfref_sampling.so."""
    target = OUT / 'libzfref_sampling.so'
    sources = ([HERE / 'ref_sampling.cu'] + sorted((HERE / 'torch_stub').rglob('*.h')) + sorted((BACKEND / 'sampling').rglob('*'))
               + sorted((BACKEND / 'optimizer').rglob('*')) + sorted((BACKEND / 'common' / 'include').glob('*')))
    if target.exists() and all(s.stat().st_mtime <= target.stat().st_mtime for s in sources if s.is_file()):
        return target
    cmd = [NVCC, '-gencode', 'arch=compute_100a,code=sm_100a', '-O3', '--use_fast_math', '-std=c++17', '--expt-relaxed-constexpr', '-lineinfo',
           '-shared', '-Xcompiler', '-fPIC', '-Xcompiler', '-fvisibility=hidden', f'-I{HERE / "torch_stub"}',
           *[f'-I{BACKEND / sub}' for sub in ('sampling/include', 'sampling/src', 'optimizer/include', 'optimizer/src', 'common/include')],
           str(HERE / 'ref_sampling.cu'), '-o', str(target)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        sys.stderr.write(result.stdout + result.stderr)
        raise RuntimeError('compiling the reference sampling kernels failed')
    return target


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument('--jobs', type=int, default=os.cpu_count())
    args = parser.parse_args()
    if not BACKEND.exists():
        raise SystemExit(f'reference sources not found under {REFERENCE_ROOT}')
    OUT.mkdir(parents=True, exist_ok=True)
    layouts = variants()
    with concurrent.futures.ThreadPoolExecutor(max_workers=args.jobs) as pool:
        futures = [pool.submit(build_variant, name, layout) for name, layout in layouts.items()] + [pool.submit(build_sampling)]
        for future in futures:
            future.result()
    (OUT / 'variants.json').write_text(json.dumps({name: dict(zip(['level', 'sizes', 'entries', 'n_features', 'mlp_width'], layout))
                                                   for name, layout in layouts.items()}, indent=1))
    print(f'built {len(layouts)} reference featurization variants and the sampling kernels into {OUT}')


if __name__ == '__main__':
    main()

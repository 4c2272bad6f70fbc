"""Builds the B200 featurization library and its PyTorch binding in-tree.

    python fused-zipnerf_b200/build.py [--jobs N] [--force]

Outputs (next to the Python package that loads them, so they travel with the source tree):
  ZipNeRFCudaBackend/libzf_featurize.so  -- the sm_100a kernels and the C ABI of include/zf_featurize.h,
                                            include/zf_sampling.h, include/zf_optim.h and include/zf_mlp.h
  ZipNeRFCudaBackend/_C.<abi>.so         -- the PyTorch binding (ZipNeRFCudaBackend._C)

Kernels are compiled ahead of time for sm_100a only (nvcc -gencode arch=compute_100a,code=sm_100a), one object per
(features, padded MLP input width) instantiation so they compile in parallel; up-to-date objects are reused.
"""
from __future__ import annotations

import argparse
import concurrent.futures
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / 'csrc'
INCLUDE = REPO / 'include'
BUILD = HERE / '_build'
PACKAGE = HERE / 'ZipNeRFCudaBackend'
LIBRARY = PACKAGE / 'libzf_featurize.so'
MAX_LEVELS, MAX_FEATURES = 16, 4

NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')
NVCC_FLAGS = ['-gencode', 'arch=compute_100a,code=sm_100a', '-O3', '--use_fast_math', '-lineinfo', '-std=c++17',
              '-Xcompiler', '-fPIC', '-Xcompiler', '-fvisibility=hidden', f'-I{INCLUDE}', f'-I{CSRC}']
# extra nvcc flags for tuning builds (e.g. ZF_NVCC_EXTRA="-DZF_MIN_BLOCKS=6")
NVCC_FLAGS += os.environ.get('ZF_NVCC_EXTRA', '').split()


def _headers() -> list[Path]:
    return sorted(CSRC.glob('*.cuh')) + sorted(CSRC.glob('*.h')) + sorted(INCLUDE.glob('*.h'))


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(s.stat().st_mtime > mtime for s in sources)


def _run(cmd: list[str]) -> None:
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        sys.stderr.write(' '.join(cmd) + '\n' + result.stdout + result.stderr)
        raise RuntimeError(f'build step failed: {cmd[-1]}')


def build_library(jobs: int | None = None, force: bool = False, subset: set | None = None) -> Path:
    """Compiles the kernel instantiations and the C ABI into libzf_featurize.so. subset: (levels, features) pairs to
    compile as (features, padded MLP width or 0); (features, 0) selects all of that feature count; None compiles all."""
    BUILD.mkdir(parents=True, exist_ok=True)
    deps = _headers()
    steps = []
    inst = CSRC / 'fz_inst.cu'
    wanted = []
    for features in range(1, MAX_FEATURES + 1):
        # pad 0: the kernels without MLP; pads: the MLP kernels of padded input widths up to 16 (F + 1)
        for pad in [0] + list(range(4, 16 * (features + 1) + 1, 4)):
            if subset is not None and (features, pad) not in subset and (features, 0) not in subset:
                continue
            obj = BUILD / f'fz_inst_F{features}_P{pad}.o'
            wanted.append(obj)
            if force or _stale(obj, [inst, *deps]):
                steps.append([NVCC, *NVCC_FLAGS, f'-DZF_INST_F={features}', f'-DZF_INST_PAD={pad}', '-c', str(inst), '-o', str(obj)])
    # the C ABI translation units: featurizer objects, the sampling kernels, the Adam step, the MLP's ReLU backward, its
    # tensor-core forward and backward, and its pack and unfold
    abi_objects = []
    for name in ['fz_capi', 'fz_sampling', 'fz_optim', 'fz_mlp', 'fz_nerf_mlp', 'fz_nerf_mlp_backward', 'fz_nerf_mlp_pack']:
        source, obj = CSRC / f'{name}.cu', BUILD / f'{name}.o'
        abi_objects.append(obj)
        if force or _stale(obj, [source, *deps]):
            steps.append([NVCC, *NVCC_FLAGS, '-c', str(source), '-o', str(obj)])
    # the largest instantiations first, so the parallel build ends evenly
    steps.sort(key=lambda cmd: -int(next((a.split('=')[1] for a in cmd if a.startswith('-DZF_INST_PAD=')), '999')))
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as pool:
        for future in [pool.submit(_run, cmd) for cmd in steps]:
            future.result()
    objects = wanted + abi_objects
    if force or steps or _stale(LIBRARY, objects) or subset is not None:
        _run([NVCC, '-gencode', 'arch=compute_100a,code=sm_100a', '-shared', '-o', str(LIBRARY), *map(str, objects)])
    return LIBRARY


def build_torch_extension(force: bool = False) -> Path:
    """Compiles the PyTorch binding ZipNeRFCudaBackend._C, linked against libzf_featurize.so (rpath $ORIGIN)."""
    import torch
    from torch.utils import cpp_extension

    suffix = sysconfig.get_config_var('EXT_SUFFIX') or '.so'
    target = PACKAGE / f'_C{suffix}'
    source = CSRC / 'torch_ext.cpp'
    if not force and not _stale(target, [source, LIBRARY, *sorted(INCLUDE.glob('*.h'))]):
        return target
    includes = cpp_extension.include_paths(device_type='cuda')
    python_include = sysconfig.get_paths()['include']
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    torch_lib = Path(torch.__file__).resolve().parent / 'lib'
    cmd = ['g++', '-O2', '-std=c++17', '-shared', '-fPIC', f'-D_GLIBCXX_USE_CXX11_ABI={abi}', '-DTORCH_EXTENSION_NAME=_C',
           '-DTORCH_API_INCLUDE_EXTENSION_H', f'-I{INCLUDE}', f'-I{python_include}', *[f'-I{p}' for p in includes],
           str(source), '-o', str(target), f'-L{PACKAGE}', '-lzf_featurize', f'-L{torch_lib}', '-lc10', '-lc10_cuda', '-ltorch',
           '-ltorch_cpu', '-ltorch_python', "-Wl,-rpath,$ORIGIN", f'-Wl,-rpath,{torch_lib}']
    _run(cmd)
    return target


def build_all(jobs: int | None = None, force: bool = False, subset: set | None = None) -> None:
    build_library(jobs, force, subset)
    build_torch_extension(force)


if __name__ == '__main__':
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument('--jobs', type=int, default=None)
    parser.add_argument('--force', action='store_true')
    parser.add_argument('--subset', default=None, help='development build of some (features:mlp_pad) objects, e.g. 1:24,4:0')
    args = parser.parse_args()
    subset = {tuple(int(v) for v in pair.split(':')) for pair in args.subset.split(',')} if args.subset else None
    build_all(args.jobs, args.force, subset)
    print(f'built {LIBRARY} and the torch binding')

"""Compiles the reference's NerfMlp (mlp/src/nerf_mlp.cu, a chain of bf16 cuBLASLt GEMMs) for the GPU checks (TEST
INFRASTRUCTURE ONLY): the source from where it lies in the reference checkout (REFERENCE_ROOT, else a sibling directory
'reference' of this repository), with the reference's compile options (setup.py:24-33: -O3, -use_fast_math,
--expt-relaxed-constexpr, C++17) for sm_100a and its cuBLASLt link, plus the binding in this directory, into
oracle/_ref/ref_mlp/zf_ref_mlp.so (shipped with the rest of oracle/_ref; the GPU tests import it from there).

    python oracle/ref_mlp/build.py
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE.parent / '_ref' / 'ref_mlp'
REFERENCE_ROOT = Path(os.environ.get('REFERENCE_ROOT', str(HERE.parent.parent.parent / 'reference')))
BACKEND = REFERENCE_ROOT / 'ZipNeRFCudaBackend' / 'ZipNeRFCudaBackend'
NAME = 'zf_ref_mlp'


def build(verbose: bool = False) -> Path:
    from torch.utils import cpp_extension
    source = BACKEND / 'mlp' / 'src' / 'nerf_mlp.cu'
    if not source.exists():
        raise FileNotFoundError(f'the reference NeRF MLP source is not at {source}')
    OUT.mkdir(parents=True, exist_ok=True)
    # the architecture comes from the flags below only
    os.environ['TORCH_CUDA_ARCH_LIST'] = ''
    cpp_extension.load(
        name=NAME,
        sources=[str(HERE / 'binding.cpp'), str(source)],
        extra_include_paths=[str(BACKEND / 'mlp' / 'include'), str(BACKEND / 'common' / 'include')],
        extra_cflags=['-O3', '-std=c++17'],
        extra_cuda_cflags=['-O3', '-std=c++17', '-use_fast_math', '--expt-relaxed-constexpr', '-gencode', 'arch=compute_100a,code=sm_100a'],
        extra_ldflags=['-lcublasLt'],
        build_directory=str(OUT),
        is_python_module=True,
        verbose=verbose,
    )
    return OUT / f'{NAME}.so'


if __name__ == '__main__':
    print(build(verbose='-v' in sys.argv))

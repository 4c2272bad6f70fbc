"""Times the product's sampling, final-level and Adam kernels against the reference's own kernels on one B200, on identical
config-2-sized inputs (zipnerf_b200/rows.py), and counts the outputs that differ bit for bit at that size.

The reference kernels are the ones oracle/ref_cuda/build.py compiles from the reference sources
(oracle/_ref/cuda/libzfref_sampling.so). Each launch is timed alone with CUDA events after an L2 flush, with its
outputs allocated beforehand for both. Prints one JSON object; run on a GPU box:

    python tests/bench_rows_vs_reference_cuda.py [--iters 10] [--out path.json] [--impls b200,reference]
                                                 [--kernels resample,generate,final,adam]

(--impls / --kernels select a part, e.g. one kernel of one implementation for a profiler capture.)
"""
from __future__ import annotations

import argparse
import ctypes
import json
import sys
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent.parent
for path in (REPO, REPO / 'fused-zipnerf_b200'):
    sys.path.insert(0, str(path))

from oracle.zf_ref_sampling_cuda import RefAdamCuda, RefSamplingCuda  # noqa: E402
from zipnerf_b200 import capi, rows  # noqa: E402


def differing(a: torch.Tensor, b: torch.Tensor) -> int:
    view = torch.int16 if a.element_size() == 2 else torch.int32
    return int((a.contiguous().view(view) != b.contiguous().view(view)).sum())


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument('--iters', type=int, default=10)
    parser.add_argument('--out', default=None)
    parser.add_argument('--impls', default='b200,reference')
    parser.add_argument('--kernels', default='resample,generate,final,adam')
    args = parser.parse_args()
    impls, kernels = args.impls.split(','), args.kernels.split(',')
    device = torch.device('cuda', 0)
    lib, ref = capi.load(), RefSamplingCuda()
    timer = rows.LaunchTimer(device)
    stream = torch.cuda.current_stream().cuda_stream
    R = rows.N_RAYS
    warp = capi.make_ray_warp(rows.WARP)
    warp_host = torch.tensor(rows.WARP, dtype=torch.float32)
    result = {}

    inp = rows.resample_inputs(R, 64, device) if 'resample' in kernels else None
    for m, level in ((64, 1), (32, 2)) if 'resample' in kernels else ():
        outs = {impl: [torch.empty(R, 64, device=device), torch.empty(R, m + 1, device=device), torch.empty(R, m + 1, device=device)]
                for impl in ('b200', 'reference')}
        ours, theirs = outs['b200'], outs['reference']
        a = capi.zf_resample_args(inp['raw_density'].data_ptr(), inp['sdist'].data_ptr(), inp['tdist'].data_ptr(), inp['directions'].data_ptr(),
                                  R, 64, 0.5, m, 1234, level, warp, *[t.data_ptr() for t in ours])
        b200 = lambda: capi.check(lib.zf_composite_and_resample(ctypes.byref(a), stream))  # noqa: E731
        reference = lambda: ref.lib.ref_composite_and_resample(  # noqa: E731
            inp['raw_density'].data_ptr(), inp['sdist'].data_ptr(), inp['tdist'].data_ptr(), inp['directions'].data_ptr(), R, 64, 0.5, m, 1234,
            level, warp_host.data_ptr(), *[t.data_ptr() for t in theirs], stream)
        nbytes = R * rows.resample_bytes(64, m)
        entry = {'bytes': nbytes}
        time_impls(entry, timer, args.iters, impls, nbytes, b200, reference)
        if len(impls) == 2:
            entry['differing'] = {name: differing(x, y) for name, x, y in zip(['weights', 'sdist', 'tdist'], ours, theirs)}
        result[f'composite_and_resample_64_{m}'] = entry
    if 'generate' in kernels:
        result['generate_rays'] = generate(lib, ref, timer, stream, warp, warp_host, impls, args.iters, device)
    if 'final' in kernels:
        result['train_final'] = final(lib, ref, timer, stream, impls, args.iters, device)
    if 'adam' in kernels:
        result['adam'] = adam(ref, timer, impls, args.iters, device)

    text = json.dumps(result, indent=1)
    print(text)
    if args.out:
        Path(args.out).write_text(text + '\n')


def time_impls(entry: dict, timer, iters: int, impls, nbytes: int, b200, reference) -> None:
    for impl, fn in (('b200', b200), ('reference', reference)):
        if impl in impls:
            ms = timer(fn, iters)
            entry[impl] = {'ms': ms, 'gbs': nbytes / (ms * 1e-3) / 1e9}
    if len(impls) == 2:
        entry['speedup'] = entry['reference']['ms'] / entry['b200']['ms']


def generate(lib, ref, timer, stream, warp, warp_host, impls, iters: int, device) -> dict:
    R = rows.N_RAYS
    pool = rows.ray_pool(device)
    width = capi.direction_block_width(4)

    def new_outputs():
        return ([torch.empty(R, 3, device=device) for _ in range(2)] + [torch.empty(R, device=device), torch.empty(R, 3, device=device),
                torch.empty(R, width, dtype=torch.bfloat16, device=device), torch.empty(R, 65, device=device), torch.empty(R, 65, device=device)])
    ours, theirs = new_outputs(), new_outputs()
    pool_args = (pool['view_offsets'].data_ptr(), pool['view_cameras'].numel(), pool['view_cameras'].data_ptr(), pool['camera_offsets'].data_ptr(),
                 pool['local_directions'].data_ptr(), pool['c2w'].data_ptr(), pool['camera_radii'].data_ptr(), pool['pool_rgb'].data_ptr(),
                 pool['pool_rgb'].shape[0])
    ga = capi.zf_generate_rays_args(77, R, *pool_args, 4, 64, warp, *[t.data_ptr() for t in ours])
    b200 = lambda: capi.check(lib.zf_generate_rays(ctypes.byref(ga), stream))  # noqa: E731
    reference = lambda: ref.lib.ref_generate_rays(77, R, *pool_args, 4, 64, warp_host.data_ptr(), *[t.data_ptr() for t in theirs], stream)  # noqa: E731
    nbytes = R * rows.new_rays_bytes(64, width)
    entry = {'bytes': nbytes}
    time_impls(entry, timer, iters, impls, nbytes, b200, reference)
    if len(impls) == 2:
        entry['differing'] = {name: differing(x, y) for name, x, y in zip(['origins', 'directions', 'radii', 'rgb', 'encoded', 'sdist', 'tdist'], ours, theirs)}
    return entry


def final(lib, ref, timer, stream, impls, iters: int, device) -> dict:
    R = rows.N_RAYS
    fin = rows.final_inputs(device)
    props = fin['proposals']
    grads = {impl: [torch.empty_like(p['raw_density']) for p in props] for impl in ('b200', 'reference')}
    out_grads = {impl: torch.empty_like(fin['nerf_outputs']) for impl in ('b200', 'reference')}
    sums = {impl: torch.zeros(4, device=device) for impl in ('b200', 'reference')}
    levels = (capi.zf_proposal_level * 2)(*[capi.zf_proposal_level(p['raw_density'].shape[1], p['raw_density'].data_ptr(), p['sdist'].data_ptr(),
                                                                    p['tdist'].data_ptr(), p['weights'].data_ptr(), g.data_ptr(), p['interlevel_weight'],
                                                                    p['interlevel_blur']) for p, g in zip(props, grads['b200'])])
    fa = capi.zf_train_final_args(fin['nerf_outputs'].data_ptr(), fin['sdist'].data_ptr(), fin['tdist'].data_ptr(), R, 32, levels, 2,
                                  fin['directions'].data_ptr(), fin['seed'], fin['rgb_target'].data_ptr(), *rows.LOSS_ARGS,
                                  out_grads['b200'].data_ptr(), sums['b200'].data_ptr())
    arr = lambda ctype, values: (ctype * 2)(*values)  # noqa: E731
    ref_args = (fin['nerf_outputs'].data_ptr(), fin['sdist'].data_ptr(), fin['tdist'].data_ptr(), R, 32, 2, arr(ctypes.c_int, [64, 64]),
                arr(ctypes.c_void_p, [p['raw_density'].data_ptr() for p in props]), arr(ctypes.c_void_p, [p['sdist'].data_ptr() for p in props]),
                arr(ctypes.c_void_p, [p['tdist'].data_ptr() for p in props]), arr(ctypes.c_void_p, [p['weights'].data_ptr() for p in props]),
                arr(ctypes.c_void_p, [g.data_ptr() for g in grads['reference']]), arr(ctypes.c_float, [p['interlevel_weight'] for p in props]),
                arr(ctypes.c_float, [p['interlevel_blur'] for p in props]), fin['directions'].data_ptr(), fin['seed'], fin['rgb_target'].data_ptr(),
                *rows.LOSS_ARGS, out_grads['reference'].data_ptr(), sums['reference'].data_ptr(), stream)
    b200 = lambda: capi.check(lib.zf_train_final(ctypes.byref(fa), stream))  # noqa: E731
    reference = lambda: ref.lib.ref_train_final(*ref_args)  # noqa: E731
    nbytes = R * rows.final_bytes()
    entry = {'bytes': nbytes}
    time_impls(entry, timer, iters, impls, nbytes, b200, reference)
    if len(impls) == 2:
        entry['differing'] = {'nerf_outputs_grad': differing(out_grads['b200'], out_grads['reference']),
                              'proposal_grads': sum(differing(a, b) for a, b in zip(grads['b200'], grads['reference']))}
    return entry


def adam(ref, timer, impls, iters: int, device) -> dict:
    import ZipNeRFCudaBackend as backend
    layout, params, grads, n_levels = rows.adam_inputs(device)
    params_ref = [p.clone() for p in params] if 'reference' in impls else None
    grads_ref = [g.clone() for g in grads] if 'reference' in impls else None
    mags, mags_ref = torch.zeros(n_levels, device=device), torch.zeros(n_levels, device=device)
    hyper = (0.1, 1e-5, 0.9, 0.99, 1e-15)
    scales, offsets = [b['scale'] for b in layout], [b['offsets'] for b in layout]
    nbytes = rows.adam_bytes(layout)
    opt = backend.Adam(params, grads, scales, offsets, *hyper, mags) if 'b200' in impls else None
    opt_ref = RefAdamCuda(ref, params_ref, grads_ref, scales, offsets, *hyper, mags_ref) if 'reference' in impls else None
    entry = {'bytes': nbytes}
    if len(impls) == 2:
        opt.step(1e-2)  # one step from the same state: bit-exact check of parameters and moments
        opt_ref.step(1e-2)
        torch.cuda.synchronize()
        diff = sum(differing(a, b) for a, b in zip(params, params_ref))
        diff_m = sum(differing(opt.state(i)[0], opt_ref.exp_avgs[i]) + differing(opt.state(i)[1], opt_ref.exp_avg_sqs[i]) for i in range(len(params)))
        entry['differing'] = {'params': diff, 'moments': diff_m}
        entry['magnitudes_max_rel_diff'] = float(((mags - mags_ref).abs() / mags_ref.abs()).max())
    time_impls(entry, timer, iters, impls, nbytes, (lambda: opt.step(1e-3)) if opt else None, (lambda: opt_ref.step(1e-3)) if opt_ref else None)
    return entry


if __name__ == '__main__':
    main()

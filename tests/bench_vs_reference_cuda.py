"""Times the product kernels against the reference's own featurization kernels on one B200 (the primary comparison of
the north star: >= 2x the reference CUDA kernels' samples/s), on identical config-2 inputs.

The reference kernels are the ones oracle/ref_cuda/build.py compiles from the reference sources (variants
config2_prop0, config2_prop1, config2_nerf). Each kernel of a training-step featurization (2 proposal forwards,
NeRF forward, NeRF backward, 2 proposal backwards) is timed with CUDA events on the current stream; the inputs (~1.8 GB)
exceed the L2. Prints one JSON object (per-kernel medians and the step totals); run on a GPU box:

    python tests/bench_vs_reference_cuda.py [--rays 65536] [--steps 10] [--warmup 3] [--out path.json]
"""
from __future__ import annotations

import argparse
import json
import statistics
import sys
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent.parent
for path in (REPO, REPO / 'fused-zipnerf_b200'):
    sys.path.insert(0, str(path))

from oracle.zf_ref_cuda import RefCuda  # noqa: E402
from zipnerf_b200 import capi, workloads  # noqa: E402

KERNELS = ['forward_proposal0', 'forward_proposal1', 'forward_nerf', 'backward_nerf', 'backward_proposal0', 'backward_proposal1']


def make_step(impl: str, wl, device):
    props, nerf = wl.levels[:-1], wl.levels[-1]
    if impl == 'b200':
        fs = [capi.CFeaturizer(l.level, l.sizes, l.entries, l.n_features, l.mlp_width) for l in wl.levels]
    else:
        fs = [RefCuda(f'config2_prop{l.level}') for l in props] + [RefCuda('config2_nerf')]
    R = wl.n_rays
    g = torch.Generator().manual_seed(7)
    rays = (wl.origins, wl.directions, wl.radii)
    seed = wl.pattern_seed
    bufs = []
    for lvl in props:
        n = R * lvl.n_intervals
        bufs.append({'raw': torch.empty(R, lvl.n_intervals, device=device), 'feat': torch.empty(n, lvl.n_output_features, device=device),
                     'grad_raw': (torch.randn(R, lvl.n_intervals, generator=g) * 1e-3).to(device),
                     'gt': torch.zeros(lvl.table.numel(), device=device), 'gw0': torch.zeros(64, lvl.n_output_features, device=device),
                     'gb0': torch.zeros(64, device=device), 'gw1': torch.zeros(64, device=device), 'gb1': torch.zeros(1, device=device)})
    n = R * nerf.n_intervals
    split = sum(e for e in nerf.entries[:3])
    nb = {'feat': torch.empty(n, 56, device=device, dtype=torch.bfloat16), 'inputs': torch.zeros(n, 96, device=device, dtype=torch.bfloat16),
          'grad': (torch.randn(n, 56, generator=g) * 1e-6).bfloat16().to(device), 'g32': torch.zeros(split * 4, device=device),
          'g16': torch.zeros((sum(nerf.entries) - split) * 4, device=device, dtype=torch.float16)}

    def calls():
        out = []
        for lvl, f, b in zip(props, fs, bufs):
            out.append(lambda lvl=lvl, f=f, b=b: f.forward(*rays, lvl.tdist, seed, False, lvl.table, lvl.scale_magnitudes, *lvl.mlp,
                                                            raw_density=b['raw'], features_float=b['feat']))
        out.append(lambda: fs[-1].forward(*rays, nerf.tdist, seed, False, nerf.table, nerf.scale_magnitudes, features_bf16=nb['feat'],
                                          encoded_directions=wl.encoded_directions, nerf_inputs=nb['inputs']))
        out.append(lambda: fs[-1].backward(*rays, nerf.tdist, seed, nb['grad'][:, :50], nb['g32'], nb['g16']))
        for lvl, f, b in zip(props, fs, bufs):
            out.append(lambda lvl=lvl, f=f, b=b: f.backward_mlp(*rays, lvl.tdist, seed, b['feat'], b['grad_raw'], *lvl.mlp[:3], b['gt'], b['gw0'],
                                                                b['gb0'], b['gw1'], b['gb1']))
        return out

    return calls()


def time_impl(impl: str, wl, device, steps: int, warmup: int) -> dict:
    calls = make_step(impl, wl, device)
    for _ in range(warmup):
        for c in calls:
            c()
    torch.cuda.synchronize()
    times = {k: [] for k in KERNELS}
    totals = []
    for _ in range(steps):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in calls]
        for (a, b), c in zip(ev, calls):
            a.record()
            c()
            b.record()
        torch.cuda.synchronize()
        ms = [a.elapsed_time(b) for a, b in ev]
        for k, t in zip(KERNELS, ms):
            times[k].append(t)
        totals.append(sum(ms))
    return {'kernels_ms': {k: statistics.median(v) for k, v in times.items()}, 'step_ms': statistics.median(totals)}


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument('--rays', type=int, default=65536)
    parser.add_argument('--steps', type=int, default=10)
    parser.add_argument('--warmup', type=int, default=3)
    parser.add_argument('--out', type=Path, default=None)
    args = parser.parse_args()
    device = torch.device('cuda:0')
    wl = workloads.config2(n_rays=args.rays, seed=1).to(device)
    samples = wl.n_intervals_total * 6
    result = {'rays': args.rays, 'samples_per_step': samples, 'device': torch.cuda.get_device_name()}
    for impl in ['reference', 'b200']:
        r = time_impl(impl, wl, device, args.steps, args.warmup)
        r['msamples_per_s'] = samples / (r['step_ms'] * 1e-3) / 1e6
        result[impl] = r
    result['speedup'] = result['reference']['step_ms'] / result['b200']['step_ms']
    result['speedup_per_kernel'] = {k: result['reference']['kernels_ms'][k] / result['b200']['kernels_ms'][k] for k in KERNELS}
    text = json.dumps(result, indent=1)
    print(text)
    if args.out:
        args.out.parent.mkdir(parents=True, exist_ok=True)
        args.out.write_text(text + '\n')


if __name__ == '__main__':
    main()

"""Benchmark of the B200 featurization hot path (BASELINE.json metric: featurization fwd+bwd Msamples/s at 65536
rays; one sample = one interval x one of the 6 hexagonal multisamples).

A step is one training iteration's featurization of config 2 (paper shape): the forward of the two proposal levels
(64 intervals per ray, fused density MLP, fp32 features) and of the NeRF level (32 intervals, packed bf16 features and
NeRF-input tail), then the NeRF-level backward (bf16 upstream gradients -> fp32/fp16 grid gradients) and the two
proposal-level backwards (MLP recomputation, grid and MLP parameter gradients), in the order of the reference's
Renderer.render_rays_training / Trainer.compute_gradients. The three backwards are independent once their upstream
gradients exist (disjoint gradient buffers), so the timed steps run them on three streams, as a training step can; the
per-kernel times and the roofline come from further steps with the calls in sequence. Inputs are seeded synthetic data of config 2's shapes (the
reference's Mip-NeRF 360 scenes are not available). With --gpus N (one process per GPU, torchrun), every rank
featurizes its own 65536 rays (weak scaling) and the grid and MLP gradients are all-reduced over NCCL, the
data-parallel exchange of a training step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Prints one JSON line on rank 0. The line also carries "train_step": the full training step (rays, all levels'
featurization, resampling, the NeRF MLP, losses, backwards, the gradient all-reduce over the N GPUs and Adam) in ms,
max over ranks; and on one GPU "rows": the sampling, final-level and Adam kernels of that step, each timed alone
against the HBM roofline.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / 'fused-zipnerf_b200'))

import torch  # noqa: E402

N_MULTISAMPLES = 6
METRIC = 'featurization fwd+bwd Msamples/s at 65536 rays'
UNIT = 'Msamples/s'
GRAD_SCALE = 1048576.0


def algorithmic_bytes(kind: str, n_levels: int, n_features: int, n_out: int, n_fp32_levels: int = 0) -> int:
    """Algorithmic HBM bytes per interval of each kernel: every one of the 48 corner lookups (6 multisamples x 8
    corners, before merging) of every level reads (or atomically updates) one table row, plus the interval's own
    inputs and outputs."""
    row = 4 * n_features
    if kind == 'forward_proposal':
        return 48 * row * n_levels + 4 + 4 + 4 * n_out                # gathers, tdist, raw density, fp32 features
    if kind == 'forward_nerf':
        return 48 * row * n_levels + 4 + 2 * ((n_out + 7) // 8 * 8) + 2 * 32  # gathers, tdist, bf16 features, input tail
    if kind == 'backward_nerf':
        return 2 * n_out + 4 + 48 * (row * n_fp32_levels + 2 * n_features * (n_levels - n_fp32_levels))
    if kind == 'backward_proposal':
        return 4 * n_out + 4 + 4 + 48 * row * n_levels
    raise ValueError(kind)


def measured_peaks() -> dict:
    path = REPO / 'MEASURED_PEAKS.json'
    if path.exists():
        return json.loads(path.read_text()) | {'source': 'measured'}
    return {'hbm_gbs': 6650.0, 'bf16_tflops': 1590.0, 'source': 'fallback'}


def profiled_traffic() -> tuple[dict, str]:
    """DRAM bytes per call of each kernel kind from the committed ncu summary (profiles/traffic.txt: 'kernel bytes'
    lines; a '# commit' line names the source revision the capture ran). Not measured by this run: a committed figure
    that goes stale when a kernel changes."""
    path = REPO / 'profiles' / 'traffic.txt'
    out, commit = {}, 'unknown'
    if path.exists():
        for line in path.read_text().splitlines():
            parts = line.split()
            if line.startswith('# commit') and len(parts) >= 3:
                commit = parts[2]
            elif len(parts) == 2 and not line.startswith('#'):
                out[parts[0]] = float(parts[1])
    return out, commit


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    FIELDS = ['clocks.sm', 'clocks.max.sm', 'power.draw', 'clocks_event_reasons.active', 'clocks_event_reasons.hw_slowdown',
              'clocks_event_reasons.hw_thermal_slowdown', 'clocks_event_reasons.sw_thermal_slowdown', 'clocks_event_reasons.sw_power_cap']

    def __init__(self, device_index: int) -> None:
        self.device_index = device_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--id={self.device_index}', f'--query-gpu={",".join(self.FIELDS)}',
                                          '--format=csv,noheader,nounits', '-lms', '200'], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # nvidia-smi's first line can take longer than a short timed region: the region starts after it
            deadline = time.time() + 5.0
            while not self.lines and self.proc.poll() is None and time.time() < deadline:
                time.sleep(0.01)
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc) -> None:
        if self.proc is not None:
            # one more sample after the timed region's last work was queued (nvidia-smi samples every 200 ms)
            seen, deadline = len(self.lines), time.time() + 1.0
            while len(self.lines) == seen and self.proc.poll() is None and time.time() < deadline:
                time.sleep(0.01)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, sm_max, reasons = [], [], set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in self.lines:
            parts = [p.strip() for p in line.split(',')]
            if len(parts) != len(self.FIELDS):
                continue
            try:
                sm.append(float(parts[0]))
                sm_max.append(float(parts[1]))
            except ValueError:
                continue
            for name, value in zip(names, parts[4:]):
                if value.lower().startswith('active'):
                    reasons.add(name)
        if not sm:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': [], 'samples': 0}
        return {'sm_mhz': statistics.median(sm), 'sm_max_mhz': max(sm_max), 'reasons': sorted(reasons), 'samples': len(sm)}


class Step:
    """One featurization fwd+bwd step of a config 2 workload on one GPU, through the PyTorch binding (the
    reference's API). Buffers are allocated once; inputs can be refreshed from pinned host copies (e2e)."""

    def __init__(self, workload, device, rank: int = 0) -> None:
        import ZipNeRFCudaBackend as backend
        from zipnerf_b200 import sharding
        from zipnerf_b200 import workloads as wl_mod
        self.device = device
        self.wl = workload.to(device)
        wl = self.wl
        self.props, self.nerf = wl.levels[:-1], wl.levels[-1]
        self.featurizers = [backend.Featurizer(l.level, l.sizes, l.entries, l.n_features, l.mlp_width) for l in wl.levels]
        # this rank's rays follow the previous ranks' in the global batch (pattern random numbers of the whole batch)
        for lvl, f in zip(wl.levels, self.featurizers):
            f.sample_offset = sharding.sample_offset(rank * wl.n_rays, lvl.n_intervals)
        R = wl.n_rays
        g = torch.Generator(device='cpu').manual_seed(1234)
        self.empty = torch.empty(0, device=device)
        self.prop_out, self.prop_grads = [], []
        for lvl, f in zip(self.props, self.featurizers):
            n = R * lvl.n_intervals
            self.prop_out.append({'raw': torch.empty(R, lvl.n_intervals, device=device),
                                  'features': torch.empty(n, lvl.n_output_features, device=device),
                                  'grad_raw': (torch.randn(R, lvl.n_intervals, generator=g) * 1e-3).to(device)})
            W = lvl.mlp_width
            self.prop_grads.append({'table': torch.zeros(lvl.table.numel(), device=device), 'w0': torch.zeros(W, lvl.n_output_features, device=device),
                                    'b0': torch.zeros(W, device=device), 'w1': torch.zeros(W, device=device), 'b1': torch.zeros(1, device=device)})
        n = R * self.nerf.n_intervals
        width = wl_mod.nerf_feature_width(self.nerf.n_output_features)
        fn = self.featurizers[-1]
        split = fn.n_fp32_grad_rows
        F = self.nerf.n_features
        self.nerf_out = {'features': torch.empty(n, width, device=device, dtype=torch.bfloat16),
                         'inputs': torch.zeros(n, wl_mod.NERF_INPUTS_WIDTH, device=device, dtype=torch.bfloat16),
                         'grad': (torch.randn(n, width, generator=g) * 1e-6).bfloat16().to(device)}
        self.nerf_grads = {'g32': torch.zeros(split * F, device=device),
                           'g16': torch.zeros((sum(self.nerf.entries) - split) * F, device=device, dtype=torch.float16)}
        self.samples_per_step = wl.n_intervals_total * N_MULTISAMPLES
        self.kernel_names = ['forward_proposal', 'forward_proposal', 'forward_nerf', 'backward_nerf', 'backward_proposal', 'backward_proposal']
        # the streams of the concurrent backwards: NeRF level, proposal level 0, proposal level 1
        self.backward_streams = [torch.cuda.Stream(device=device) for _ in range(3)]
        self.calls_per_step = len(self.kernel_names)
        # kernel launches of the step's calls (level passes of the NeRF grid, two kernels per proposal backward)
        from zipnerf_b200 import capi
        counts = [capi.CFeaturizer(l.level, l.sizes, l.entries, l.n_features, l.mlp_width) for l in wl.levels]
        self.kernel_launches_per_step = (sum(c.launches('forward_mlp') + c.launches('backward_mlp') for c in counts[:-1]) +
                                         counts[-1].launches('forward') + counts[-1].launches('backward'))

    def input_buffers(self) -> list:
        wl = self.wl
        out = [wl.origins, wl.directions, wl.radii, wl.encoded_directions, self.nerf_out['grad']]
        for lvl, po in zip(wl.levels, self.prop_out + [None]):
            out.append(lvl.tdist)
            if po is not None:
                out.append(po['grad_raw'])
        return out

    def set_inputs(self, buffers: list) -> None:
        """Points the step at another set of input tensors (the order of input_buffers)."""
        wl = self.wl
        it = iter(buffers)
        wl.origins, wl.directions, wl.radii, wl.encoded_directions, self.nerf_out['grad'] = (next(it) for _ in range(5))
        for lvl, po in zip(wl.levels, self.prop_out + [None]):
            lvl.tdist = next(it)
            if po is not None:
                po['grad_raw'] = next(it)

    def run(self, events=None, after_backward=None, concurrent: bool = False) -> None:
        """One step; events (list of (start, end) CUDA event pairs per kernel) are recorded if given;
        after_backward(buffers) is called with each level's gradient buffers once its backward is enqueued, on that
        backward's stream (the data-parallel exchange of those buffers starts there). concurrent: the three levels'
        backwards on three streams after the forwards (not with events: those time each call alone)."""
        assert not (concurrent and events is not None)
        wl, seed, e = self.wl, self.wl.pattern_seed, self.empty
        rays = (wl.origins, wl.directions, wl.radii)
        k = 0

        def mark(i, which):
            if events is not None:
                events[i][which].record()

        for lvl, f, po in zip(self.props, self.featurizers, self.prop_out):
            mark(k, 0)
            f.forward(*rays, lvl.tdist, seed, False, lvl.table, lvl.scale_magnitudes, *lvl.mlp, po['raw'], po['features'], e, e, e)
            mark(k, 1)
            k += 1
        nerf, fn = self.nerf, self.featurizers[-1]
        mark(k, 0)
        fn.forward(*rays, nerf.tdist, seed, False, nerf.table, nerf.scale_magnitudes, e, e, e, e, e, e, self.nerf_out['features'],
                   wl.encoded_directions, self.nerf_out['inputs'])
        mark(k, 1)
        k += 1
        main = torch.cuda.current_stream()
        if concurrent:
            for s in self.backward_streams:
                s.wait_stream(main)
        with torch.cuda.stream(self.backward_streams[0] if concurrent else main):
            mark(k, 0)
            fn.backward(*rays, nerf.tdist, seed, self.nerf_out['grad'][:, :fn.n_output_features], self.nerf_grads['g32'], self.nerf_grads['g16'])
            mark(k, 1)
            k += 1
            if after_backward is not None:
                after_backward([self.nerf_grads['g32'], self.nerf_grads['g16']])
        for s, lvl, f, po, pg in zip(self.backward_streams[1:], self.props, self.featurizers, self.prop_out, self.prop_grads):
            with torch.cuda.stream(s if concurrent else main):
                mark(k, 0)
                f.backward_mlp(*rays, lvl.tdist, seed, po['features'], po['grad_raw'], *lvl.mlp[:3], pg['table'], pg['w0'], pg['b0'], pg['w1'], pg['b1'])
                mark(k, 1)
                k += 1
                if after_backward is not None:
                    after_backward([pg['table'], pg['w0'], pg['b0'], pg['w1'], pg['b1']])
        if concurrent:
            for s in self.backward_streams:
                main.wait_stream(s)

    def kernel_bytes(self) -> list:
        out = []
        for lvl in self.props:
            out.append(algorithmic_bytes('forward_proposal', lvl.n_levels, lvl.n_features, lvl.n_output_features) * self.wl.n_rays * lvl.n_intervals)
        nerf, fn = self.nerf, self.featurizers[-1]
        n_fp32 = sum(1 for e in nerf.entries if e < (1 << 20))
        n = self.wl.n_rays * nerf.n_intervals
        out.append(algorithmic_bytes('forward_nerf', nerf.n_levels, nerf.n_features, nerf.n_output_features) * n)
        out.append(algorithmic_bytes('backward_nerf', nerf.n_levels, nerf.n_features, nerf.n_output_features, n_fp32) * n)
        for lvl in self.props:
            out.append(algorithmic_bytes('backward_proposal', lvl.n_levels, lvl.n_features, lvl.n_output_features) * self.wl.n_rays * lvl.n_intervals)
        return out


class ReferenceStep:
    """The same step through the reference's own featurization kernels (a BASELINE leg, like cpu_baseline: the
    reference's four kernels compiled ahead of time from its sources by oracle/ref_cuda/build.py, launched as its
    featurizer.cu:188-355 launches them), on the inputs of a product Step and into buffers of its own. Outside every
    product timed region."""

    VARIANTS = ('config2_prop0', 'config2_prop1', 'config2_nerf')

    @staticmethod
    def unavailable() -> str | None:
        from oracle.zf_ref_cuda import available_variants
        missing = [v for v in ReferenceStep.VARIANTS if v not in available_variants()]
        return f'reference kernels not built ({", ".join(missing)}; python oracle/ref_cuda/build.py)' if missing else None

    def __init__(self, step: Step) -> None:
        from oracle.zf_ref_cuda import RefCuda
        self.step = step
        device, wl = step.device, step.wl
        self.featurizers = [RefCuda(f'config2_prop{l.level}') for l in step.props] + [RefCuda('config2_nerf')]
        self.prop_out = [{'raw': torch.empty_like(po['raw']), 'features': torch.empty_like(po['features'])} for po in step.prop_out]
        self.prop_grads = [{k: torch.zeros_like(v) for k, v in pg.items()} for pg in step.prop_grads]
        self.nerf_out = {'features': torch.empty_like(step.nerf_out['features']), 'inputs': torch.zeros_like(step.nerf_out['inputs'])}
        self.nerf_grads = {k: torch.zeros_like(v) for k, v in step.nerf_grads.items()}
        self.n_output_features = wl.levels[-1].n_output_features
        self.kernel_names = step.kernel_names

    def zero_grads(self) -> None:
        for g in [*self.prop_grads, self.nerf_grads]:
            for v in g.values():
                v.zero_()

    def run(self, events=None) -> None:
        """The reference kernels of one step, in the order of Step.run (per-call CUDA events if given)."""
        st, wl = self.step, self.step.wl
        rays, seed = (wl.origins, wl.directions, wl.radii), wl.pattern_seed
        k = 0

        def mark(i, which):
            if events is not None:
                events[i][which].record()

        for lvl, f, po in zip(st.props, self.featurizers, self.prop_out):
            mark(k, 0)
            f.forward(*rays, lvl.tdist, seed, False, lvl.table, lvl.scale_magnitudes, *lvl.mlp, raw_density=po['raw'], features_float=po['features'])
            mark(k, 1)
            k += 1
        nerf, fn = st.nerf, self.featurizers[-1]
        mark(k, 0)
        fn.forward(*rays, nerf.tdist, seed, False, nerf.table, nerf.scale_magnitudes, features_bf16=self.nerf_out['features'],
                   encoded_directions=wl.encoded_directions, nerf_inputs=self.nerf_out['inputs'])
        mark(k, 1)
        k += 1
        mark(k, 0)
        fn.backward(*rays, nerf.tdist, seed, st.nerf_out['grad'][:, :self.n_output_features], self.nerf_grads['g32'], self.nerf_grads['g16'])
        mark(k, 1)
        k += 1
        for lvl, f, po, spo, pg in zip(st.props, self.featurizers, self.prop_out, st.prop_out, self.prop_grads):
            mark(k, 0)
            f.backward_mlp(*rays, lvl.tdist, seed, po['features'], spo['grad_raw'], *lvl.mlp[:3], pg['table'], pg['w0'], pg['b0'], pg['w1'], pg['b1'])
            mark(k, 1)
            k += 1


def measure_reference_cuda(step: Step, args, physical: int, our_ms_per_step: float, our_kernels: dict) -> dict:
    """The north-star comparison: the reference's own CUDA kernels on the identical config-2 step and inputs, timed on
    this GPU right after the product's timed region, with the same protocol (CUDA events around the step on the
    current stream, warm-up first, inputs larger than L2) and its own clock record. ratio = reference ms per step / the
    product's ms per step (higher is better)."""
    why = ReferenceStep.unavailable()
    if why is not None:
        return {'unavailable': why}
    ref = ReferenceStep(step)
    for _ in range(args.warmup):
        ref.run()
    n_k = len(ref.kernel_names)
    events = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(n_k)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with ClockSampler(physical) as clocks:
        start.record()
        for i in range(args.steps):
            ref.run(events[i])
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    per_kernel: dict[str, list] = {}
    for i in range(args.steps):
        for name, (a, b) in zip(ref.kernel_names, events[i]):
            per_kernel.setdefault(name, []).append(a.elapsed_time(b))
    kernels_ms = {name: sum(t) / len(t) for name, t in per_kernel.items()}
    del ref
    torch.cuda.empty_cache()
    return {'what': "the reference's featurize_forward / featurize_forward_bf16 / featurize_backward / featurize_backward_mlp kernels, "
                    'compiled from its sources for sm_100a with its fast-math options, launched with its launch shapes, on the same '
                    'inputs as the product step (oracle/ref_cuda)',
            'ms_per_step': ms, 'msamples_per_s': step.samples_per_step / (ms * 1e-3) / 1e6, 'steps': args.steps, 'warmup': args.warmup,
            'kernels_avg_ms': kernels_ms, 'ours_ms_per_step': our_ms_per_step, 'ratio': ms / our_ms_per_step,
            'ratio_per_kernel': {name: kernels_ms[name] / our_kernels[name]['avg_ms'] for name in kernels_ms if name in our_kernels},
            'clocks': clocks.summary()}


def measure_contention(args, device, physical: int) -> dict:
    """Config 5 (atomic contention): the NeRF-level forward and backward of 65,536 rays x 160 intervals whose rays all
    pass through a 0.05-radius ball within a 5 degree cone (coarse rows receive ~10^5 contributions per step), 12 x 4
    features, table 2^22; the product's kernels through the PyTorch binding and, where built, the reference's kernels
    on the same inputs. Reported per call: ms, Msamples/s and the unmerged corner contributions per second of the
    backward (every interval's 6 x 8 x 12 corner updates)."""
    import ZipNeRFCudaBackend as backend
    from zipnerf_b200 import workloads as wl_mod
    wl = wl_mod.config5(n_rays=args.rays, seed=5).to(device)
    lvl = wl.levels[0]
    n = wl.n_rays * lvl.n_intervals
    width = wl_mod.nerf_feature_width(lvl.n_output_features)
    rays = (wl.origins, wl.directions, wl.radii, lvl.tdist)
    g = torch.Generator(device='cpu').manual_seed(55)
    grad = (torch.randn(n, width, generator=g) * 1e-6).bfloat16().to(device)
    feats = torch.empty(n, width, device=device, dtype=torch.bfloat16)
    ours = backend.Featurizer(lvl.level, lvl.sizes, lvl.entries, lvl.n_features, lvl.mlp_width)
    split = ours.n_fp32_grad_rows
    g32 = torch.zeros(split * lvl.n_features, device=device)
    g16 = torch.zeros((sum(lvl.entries) - split) * lvl.n_features, device=device, dtype=torch.float16)
    e = torch.empty(0, device=device)
    n_out = lvl.n_output_features

    def our_calls():
        return [lambda: ours.forward(*rays, wl.pattern_seed, False, lvl.table, lvl.scale_magnitudes, e, e, e, e, e, e, feats, e, e),
                lambda: ours.backward(*rays, wl.pattern_seed, grad[:, :n_out], g32, g16)]

    def ref_calls(ref):
        return [lambda: ref.forward(*rays, wl.pattern_seed, False, lvl.table, lvl.scale_magnitudes, features_bf16=feats),
                lambda: ref.backward(*rays, wl.pattern_seed, grad[:, :n_out], g32, g16)]

    def time_calls(calls):
        times = [[], []]
        for i in range(args.warmup + args.steps):
            g32.zero_()
            g16.zero_()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in calls]
            for (a, b), c in zip(ev, calls):
                a.record()
                c()
                b.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                for t, (a, b) in zip(times, ev):
                    t.append(a.elapsed_time(b))
        return [statistics.median(t) for t in times]

    contributions = n * N_MULTISAMPLES * 8 * lvl.n_levels
    samples = n * N_MULTISAMPLES
    n_fp32 = sum(1 for e in lvl.entries if e < (1 << 20))

    def entry(fwd_ms, bwd_ms):
        return {'forward_ms': fwd_ms, 'backward_ms': bwd_ms, 'forward_msamples_per_s': samples / (fwd_ms * 1e-3) / 1e6,
                'backward_msamples_per_s': samples / (bwd_ms * 1e-3) / 1e6,
                'backward_gcontributions_per_s': contributions / (bwd_ms * 1e-3) / 1e9}

    with ClockSampler(physical) as clocks:
        out = {'config': f'config5: {wl.n_rays} rays x {lvl.n_intervals} intervals x 6 multisamples, origins in a 0.05 ball, directions in a 5 degree '
                         f'cone; NeRF grid 12 x 4 features, table 2^22, 16 -> 16384 (fp32 gradients on the first {n_fp32} levels, fp16 above); '
                         'forward: packed bf16 features; backward: bf16 upstream gradients',
               'ours': entry(*time_calls(our_calls()))}
        from oracle.zf_ref_cuda import RefCuda, available_variants
        if 'config5' in available_variants():
            out['reference_cuda'] = entry(*time_calls(ref_calls(RefCuda('config5'))))
            out['ratio_backward'] = out['reference_cuda']['backward_ms'] / out['ours']['backward_ms']
            out['ratio_forward'] = out['reference_cuda']['forward_ms'] / out['ours']['forward_ms']
        else:
            out['reference_cuda'] = {'unavailable': 'reference kernel variant config5 not built'}
    out['clocks'] = clocks.summary()
    del wl, grad, feats, g32, g16
    torch.cuda.empty_cache()
    return out


def init_distributed(n_gpus: int):
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if world != n_gpus and world > 1:
        raise SystemExit(f'--gpus {n_gpus} but WORLD_SIZE={world}')
    return world, rank, local


class CpuBaseline:
    """The reference's own featurization code compiled for the host (oracle/_ref, where built), else the C oracle,
    on a bounded ray sample of config 2 (fwd+bwd of all three levels, gradient buffers allocated up front)."""

    def __init__(self, n_rays: int, threads: int) -> None:
        self.n_rays, self.threads = n_rays, threads
        self.prepared = None

    def run(self, repeats: int = 1) -> dict:
        """Times `repeats` passes; samples/s scaled to Msamples/s."""
        if self.prepared is None:
            self.prepared = _prepare_cpu_baseline(self.n_rays)
        return _time_cpu_baseline(self.prepared, self.n_rays, self.threads, repeats)


def _prepare_cpu_baseline(n_rays: int):
    import numpy as np
    from oracle.zf_oracle import GridSpec, Oracle, RefCpu
    from zipnerf_b200 import workloads
    kind = 'reference' if RefCpu.available() else 'port'
    checker = RefCpu() if kind == 'reference' else Oracle()
    wl = workloads.config2(n_rays=n_rays, seed=1)
    rays = [x.numpy() for x in (wl.origins, wl.directions, wl.radii)]
    g = np.random.default_rng(0)
    levels = []
    for lvl in wl.levels:
        grid = GridSpec(lvl.level, lvl.sizes, lvl.entries, lvl.n_features, lvl.mlp_width)
        n = n_rays * lvl.n_intervals
        entry = {'grid': grid, 'tdist': lvl.tdist.numpy(), 'table': lvl.table.numpy(), 'mags': lvl.scale_magnitudes.numpy()}
        if lvl.mlp_width > 0:
            W, n_out = lvl.mlp_width, lvl.n_output_features
            entry['mlp'] = [m.numpy() for m in lvl.mlp]
            entry['grad_raw'] = (g.standard_normal((n_rays, lvl.n_intervals)) * 1e-3).astype(np.float32)
            entry['grads'] = {'grad_table': np.zeros(grid.n_rows, np.float32), 'grad_w0': np.zeros((W, n_out), np.float32),
                              'grad_b0': np.zeros(W, np.float32), 'grad_w1': np.zeros(W, np.float32), 'grad_b1': np.zeros(1, np.float32)}
        else:
            entry['width'] = (lvl.n_output_features + 7) // 8 * 8
            entry['grad'] = (torch.randn(n, entry['width']) * 1e-6).bfloat16().view(torch.int16).numpy().view(np.uint16).copy()
            entry['g32'] = np.zeros(grid.n_fp32_grad_rows * grid.n_features, np.float32)
            entry['g16'] = np.zeros((grid.n_rows - grid.n_fp32_grad_rows) * grid.n_features, np.uint16)
        levels.append(entry)
    enc = wl.encoded_directions.view(torch.int16).numpy().view(np.uint16).copy()
    return kind, checker, wl, rays, levels, enc


def _time_cpu_baseline(prepared, n_rays: int, threads: int, repeats: int) -> dict:
    kind, checker, wl, rays, levels, enc = prepared
    n_threads = threads if kind == 'reference' else 1
    start = time.perf_counter()
    for _ in range(repeats):
        for e in levels:
            if 'mlp' in e:
                out = checker.forward(e['grid'], *rays, e['tdist'], wl.pattern_seed, e['table'], e['mags'], mlp=e['mlp'], raw_density=True,
                                      features_float=True, n_threads=n_threads)
                checker.backward_mlp(e['grid'], *rays, e['tdist'], wl.pattern_seed, out['features_float'], e['grad_raw'], *e['mlp'][:3],
                                     n_threads=n_threads, out=e['grads'])
            else:
                checker.forward(e['grid'], *rays, e['tdist'], wl.pattern_seed, e['table'], e['mags'], features_bf16_width=e['width'],
                                encoded_directions=enc, nerf_inputs_width=96, n_threads=n_threads)
                checker.backward(e['grid'], *rays, e['tdist'], wl.pattern_seed, e['grad'], e['g32'], e['g16'], n_threads=n_threads)
    elapsed = time.perf_counter() - start
    samples = n_rays * sum(l.n_intervals for l in wl.levels) * N_MULTISAMPLES * repeats
    return {'value': samples / elapsed / 1e6, 'unit': UNIT, 'cores': n_threads, 'kind': kind,
            'sample': f'{n_rays} rays of config 2 x (64 + 64 + 32) intervals x 6 multisamples, fwd+bwd of all three levels, '
                      f'{repeats} pass(es): {samples} samples in {elapsed:.2f} s'}


def bench_config(args, world: int, samples_per_step: int) -> dict:
    """The workload of both arms' lines."""
    return {'workload': 'config2: 65536 rays x (64 + 64 + 32) intervals x 6 multisamples, fwd+bwd of 2 proposal levels (10x1 features, '
                        'table 2^21, 16->512, fused MLP 64) and the NeRF level (10x4 features, table 2^21, 16->8192)',
            'rays_per_gpu': args.rays, 'samples_per_step_per_gpu': samples_per_step,
            'parallelism': f'dp{world} (rays sharded, gradients all-reduced)' if world > 1 else 'single GPU',
            'l2': 'inputs larger than L2 (step working set ~1.8 GB > 126 MB)',
            'schedule': 'forwards in sequence; the three backwards on three streams (independent given their upstream gradients); '
                        'per-kernel times from steps with every call in sequence'}


def run_reference_arm(args) -> None:
    world, rank, _ = init_distributed(args.gpus)
    if rank != 0:
        return
    from oracle.zf_oracle import build, n_threads_default
    build()
    baseline = CpuBaseline(args.reference_rays, n_threads_default())
    values = []
    for _ in range(args.warmup):
        baseline.run()
    for _ in range(args.steps):
        values.append(baseline.run())
    value = statistics.median(v['value'] for v in values)
    base = values[0]
    emit({'impl': 'reference', 'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': args.gpus, 'steps': args.steps,
                      'warmup': args.warmup, 'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32',
                      'data': 'synthetic (seeded config 2 shapes; Mip-NeRF 360 unavailable)',
                      'config': bench_config(args, 1, args.rays * (64 + 64 + 32) * N_MULTISAMPLES) |
                                {'timed_sample': f'each step times {args.reference_rays} of the {args.rays} rays (all three levels, fwd+bwd) on '
                                                 'the host cores and reports that sample\'s samples/s'},
                      'cpu_baseline': {'value': value, 'unit': UNIT, 'cores': base['cores'], 'kind': base['kind'], 'sample': base['sample']},
                      'e2e': {'value': value, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}})


def run_b200(args) -> None:
    import torch.distributed as dist
    from zipnerf_b200 import workloads
    world, rank, local = init_distributed(args.gpus)
    torch.cuda.set_device(local)
    device = torch.device('cuda', local)
    if world > 1:
        import datetime
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120), device_id=device)
    step = Step(workloads.config2(n_rays=args.rays, seed=1 + rank), device, rank)
    comm = torch.cuda.Stream() if world > 1 else None

    def start_exchange(buffers):
        # a level's gradients are final after its backward: average them on a communication stream while the next
        # levels' backwards run (every rank issues the same collectives in the same order)
        if world > 1:
            from zipnerf_b200 import sharding
            comm.wait_stream(torch.cuda.current_stream())  # the stream of the level's backward
            with torch.cuda.stream(comm):
                sharding.allreduce_gradients(buffers, half_wire=args.half_wire)

    tails = []

    def exchange():
        # the step ends when every level's exchange has finished; the events around the wait give the exchange tail
        # (the time the compute stream idles after its last backward)
        if world > 1:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            torch.cuda.current_stream().wait_stream(comm)
            b.record()
            tails.append((a, b))

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step.run(after_backward=start_exchange, concurrent=True)
        exchange()
    barrier()
    n_k = step.calls_per_step
    events = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(n_k)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    visible = os.environ.get('CUDA_VISIBLE_DEVICES')
    physical = int(visible.split(',')[local]) if visible and visible.split(',')[local].strip().isdigit() else local
    with ClockSampler(physical) as clocks:
        barrier()
        start.record()
        for i in range(args.steps):
            step.run(after_backward=start_exchange, concurrent=True)
            exchange()
        end.record()
        barrier()
    # the per-kernel times: the same steps with the calls in sequence (no exchange), each call between events, after
    # warm-up steps in sequence (the proposal backwards' workspaces come from the caching allocator, whose blocks
    # belong to the stream they were first used on)
    for _ in range(args.warmup):
        step.run()
    barrier()
    for i in range(args.steps):
        step.run(events[i])
    barrier()
    elapsed_ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([elapsed_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = t.item()
    ms_per_step = elapsed_ms / args.steps
    value = step.samples_per_step * world * args.steps / (elapsed_ms / 1e3) / 1e6
    exchange_tail_ms = statistics.mean(a.elapsed_time(b) for a, b in tails[-args.steps:]) if tails else 0.0
    # per-kernel durations and the roofline of the dominant kernel
    kernel_ms: dict[str, list] = {}
    for i in range(args.steps):
        for name, (a, b) in zip(step.kernel_names, events[i]):
            kernel_ms.setdefault(name, []).append(a.elapsed_time(b))
    bytes_per = {}
    for name, nbytes in zip(step.kernel_names, step.kernel_bytes()):
        bytes_per.setdefault(name, []).append(nbytes)
    peaks = measured_peaks()
    traffic, traffic_commit = profiled_traffic()
    kernels = {}
    for name, times in kernel_ms.items():
        launches_per_step = len(bytes_per[name])
        avg_ms = sum(times) / len(times)
        algo = sum(bytes_per[name]) / launches_per_step
        kernels[name] = {'calls': len(times), 'avg_ms': avg_ms, 'share': sum(times) / sum(sum(v) for v in kernel_ms.values()),
                         'algorithmic_bytes': algo, 'achieved_gbs': algo / (avg_ms * 1e-3) / 1e9}
    dominant = max(kernels, key=lambda k: kernels[k]['avg_ms'] * kernels[k]['calls'])
    dk = kernels[dominant]
    roofline = {'bound': 'hbm', 'kernel': dominant, 'achieved': dk['achieved_gbs'], 'peak': peaks['hbm_gbs'], 'unit': 'GB/s',
                'frac': dk['achieved_gbs'] / peaks['hbm_gbs'], 'peak_source': peaks['source'],
                'traffic': traffic.get(dominant),
                'traffic_source': f'committed ncu capture profiles/traffic.txt (DRAM read + write bytes per call, source revision {traffic_commit}); '
                                  'not measured by this run'}
    result = {'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup,
              'ms_per_step': ms_per_step, 'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32',
              'data': 'synthetic (seeded config 2 shapes; Mip-NeRF 360 unavailable)',
              'config': bench_config(args, world, step.samples_per_step),
              'roofline': roofline, 'kernels': kernels, 'gpu_launches': step.kernel_launches_per_step * args.steps, 'clocks': clocks.summary()}
    if world > 1:
        result['exchange'] = {'tail_ms_per_step': exchange_tail_ms, 'half_wire': args.half_wire,
                              'collectives': 'one coalesced NCCL group per level: NeRF grid (fp32 + fp16 gradients), then each proposal level '
                                             '(grid + MLP gradients), on a communication stream overlapping the later backwards'}
    if rank == 0 and world == 1 and not args.skip_reference_cuda:
        # baseline legs (test infrastructure, outside the product's timed regions): the reference's own CUDA kernels on
        # this step's inputs, and the config-5 contention case
        result['reference_cuda'] = measure_reference_cuda(step, args, physical, ms_per_step, kernels)
    if rank == 0 and world == 1 and not args.skip_contention:
        result['contention'] = measure_contention(args, device, physical)
    if rank == 0 and world == 1 and not args.skip_nerf_mlp:
        result['nerf_mlp'] = measure_nerf_mlp(device, physical, n=args.nerf_mlp_samples)
    if not args.skip_e2e:
        result['e2e'] = measure_e2e(step, args, world, start_exchange, exchange, barrier)
    if not args.skip_train_step:
        result['train_step'] = measure_train_step(args, world, rank, device, barrier)
    if not args.skip_render:
        result['render_frame'] = measure_render(args, world, rank, device, barrier)
    if rank == 0 and not args.skip_rows and world == 1:
        result['rows'] = measure_rows(device)
    if rank == 0 and not args.skip_cpu_baseline and world == 1:
        from oracle.zf_oracle import build, n_threads_default
        build()
        result['cpu_baseline'] = CpuBaseline(args.reference_rays, n_threads_default()).run(repeats=args.reference_repeats)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank == 0:
        emit(result)


def measure_rows(device, iters: int = 10) -> dict:
    """The per-step kernels around the featurization, each timed alone through the C ABI on config-2-sized inputs after
    an L2 flush (zipnerf_b200/rows.py): the two composite-and-resample calls of a training step (proposal level 0 -> 64
    intervals, level 1 -> 32), the training rays of a step drawn from a 185-view pool, the final level's losses and
    gradients, and the Adam step over the reference model's optimizer buffers (77.5 M parameters). Achieved bandwidth = algorithmic bytes / median time,
    against the measured HBM peak. Where the reference's own sampling and Adam kernels are built (oracle/ref_cuda, a
    baseline leg), each entry also carries their time on the same inputs (into outputs of their own) and the ratio."""
    import ctypes
    import ZipNeRFCudaBackend as backend
    from oracle import zf_ref_sampling_cuda as ref_mod
    from zipnerf_b200 import capi, rows
    lib = capi.load()
    ref = ref_mod.RefSamplingCuda() if ref_mod.available() else None
    peaks = measured_peaks()
    timer = rows.LaunchTimer(device)
    stream = torch.cuda.current_stream().cuda_stream
    R = rows.N_RAYS
    warp = capi.make_ray_warp(rows.WARP)
    warp_host = torch.tensor(rows.WARP, dtype=torch.float32)

    def entry(ms_list, nbytes, config, ref_list=None):
        ms = sum(ms_list)
        gbs = nbytes / (ms * 1e-3) / 1e9
        out = {'config': config, 'ms': ms, 'calls_ms': ms_list, 'algorithmic_bytes': nbytes, 'achieved_gbs': gbs, 'peak': peaks['hbm_gbs'],
               'frac': gbs / peaks['hbm_gbs']}
        if ref_list:
            out['reference_cuda_ms'] = sum(ref_list)
            out['ratio'] = sum(ref_list) / ms
        return out

    out = {}
    inp = rows.resample_inputs(R, 64, device)
    calls, ref_calls, nbytes = [], [], 0
    for m, level in ((64, 1), (32, 2)):
        s_next, t_next, weights = torch.empty(R, m + 1, device=device), torch.empty(R, m + 1, device=device), torch.empty(R, 64, device=device)
        a = capi.zf_resample_args(inp['raw_density'].data_ptr(), inp['sdist'].data_ptr(), inp['tdist'].data_ptr(), inp['directions'].data_ptr(), R,
                                  64, 0.5, m, 1234, level, warp, weights.data_ptr(), s_next.data_ptr(), t_next.data_ptr())
        calls.append(timer(lambda a=a: capi.check(lib.zf_composite_and_resample(ctypes.byref(a), stream)), iters))
        if ref is not None:
            theirs = [torch.empty_like(weights), torch.empty_like(s_next), torch.empty_like(t_next)]
            ref_calls.append(timer(lambda m=m, level=level, theirs=theirs: ref.lib.ref_composite_and_resample(
                inp['raw_density'].data_ptr(), inp['sdist'].data_ptr(), inp['tdist'].data_ptr(), inp['directions'].data_ptr(), R, 64, 0.5, m, 1234,
                level, warp_host.data_ptr(), *[t.data_ptr() for t in theirs], stream), iters))
        nbytes += R * rows.resample_bytes(64, m)
    out['composite_and_resample'] = entry(calls, nbytes, f'{R} rays: 64 -> 64 and 64 -> 32 intervals (training, jittered)', ref_calls)
    pool = rows.ray_pool(device)
    width = capi.direction_block_width(4)

    def new_ray_outputs():
        return ([torch.empty(R, 3, device=device) for _ in range(2)] + [torch.empty(R, device=device), torch.empty(R, 3, device=device),
                torch.empty(R, width, dtype=torch.bfloat16, device=device), torch.empty(R, 65, device=device), torch.empty(R, 65, device=device)])
    pool_args = (pool['view_offsets'].data_ptr(), pool['view_cameras'].numel(), pool['view_cameras'].data_ptr(), pool['camera_offsets'].data_ptr(),
                 pool['local_directions'].data_ptr(), pool['c2w'].data_ptr(), pool['camera_radii'].data_ptr(), pool['pool_rgb'].data_ptr(),
                 pool['pool_rgb'].shape[0])
    ours = new_ray_outputs()
    ga = capi.zf_generate_rays_args(77, R, *pool_args, 4, 64, warp, *[t.data_ptr() for t in ours])
    ms = timer(lambda: capi.check(lib.zf_generate_rays(ctypes.byref(ga), stream)), iters)
    ref_ms = []
    if ref is not None:
        theirs = new_ray_outputs()
        ref_ms.append(timer(lambda: ref.lib.ref_generate_rays(77, R, *pool_args, 4, 64, warp_host.data_ptr(), *[t.data_ptr() for t in theirs], stream),
                            iters))
    out['generate_rays'] = entry([ms], R * rows.new_rays_bytes(64, width), f'{R} rays from 185 views of 1296 x 840 pixels, 64 first-level intervals',
                                 ref_ms)
    del pool
    fin = rows.final_inputs(device)
    props = fin['proposals']
    proposal_grads = [torch.empty_like(p['raw_density']) for p in props]
    levels = (capi.zf_proposal_level * 2)(*[capi.zf_proposal_level(p['raw_density'].shape[1], p['raw_density'].data_ptr(), p['sdist'].data_ptr(),
                                                                    p['tdist'].data_ptr(), p['weights'].data_ptr(), g.data_ptr(), p['interlevel_weight'],
                                                                    p['interlevel_blur']) for p, g in zip(props, proposal_grads)])
    out_grad, loss_sums = torch.empty_like(fin['nerf_outputs']), torch.zeros(4, device=device)
    fa = capi.zf_train_final_args(fin['nerf_outputs'].data_ptr(), fin['sdist'].data_ptr(), fin['tdist'].data_ptr(), R, 32, levels, 2,
                                  fin['directions'].data_ptr(), fin['seed'], fin['rgb_target'].data_ptr(), *rows.LOSS_ARGS, out_grad.data_ptr(),
                                  loss_sums.data_ptr())
    ms = timer(lambda: capi.check(lib.zf_train_final(ctypes.byref(fa), stream)), iters)
    ref_ms = []
    if ref is not None:
        ref_grads = [torch.empty_like(g) for g in proposal_grads]
        ref_out_grad, ref_sums = torch.empty_like(out_grad), torch.zeros(4, device=device)

        def arr(ctype, values):
            return (ctype * 2)(*values)
        ref_args = (fin['nerf_outputs'].data_ptr(), fin['sdist'].data_ptr(), fin['tdist'].data_ptr(), R, 32, 2, arr(ctypes.c_int, [64, 64]),
                    arr(ctypes.c_void_p, [p['raw_density'].data_ptr() for p in props]), arr(ctypes.c_void_p, [p['sdist'].data_ptr() for p in props]),
                    arr(ctypes.c_void_p, [p['tdist'].data_ptr() for p in props]), arr(ctypes.c_void_p, [p['weights'].data_ptr() for p in props]),
                    arr(ctypes.c_void_p, [g.data_ptr() for g in ref_grads]), arr(ctypes.c_float, [p['interlevel_weight'] for p in props]),
                    arr(ctypes.c_float, [p['interlevel_blur'] for p in props]), fin['directions'].data_ptr(), fin['seed'], fin['rgb_target'].data_ptr(),
                    *rows.LOSS_ARGS, ref_out_grad.data_ptr(), ref_sums.data_ptr(), stream)
        ref_ms.append(timer(lambda: ref.lib.ref_train_final(*ref_args), iters))
    out['train_final'] = entry([ms], R * rows.final_bytes(), f'{R} rays: final level of 32 intervals, proposal levels of 64 and 64', ref_ms)
    del fin, proposal_grads
    layout, params, grads, n_levels = rows.adam_inputs(device)
    mags = torch.zeros(n_levels, device=device)
    hyper = (0.1, 1e-5, 0.9, 0.99, 1e-15)
    scales, offsets = [b['scale'] for b in layout], [b['offsets'] for b in layout]
    opt = backend.Adam(params, grads, scales, offsets, *hyper, mags)
    ms = timer(lambda: opt.step(1e-3), iters)
    ref_ms = []
    if ref is not None:
        opt_ref = ref_mod.RefAdamCuda(ref, [p.clone() for p in params], [g.clone() for g in grads], scales, offsets, *hyper,
                                      torch.zeros(n_levels, device=device))
        ref_ms.append(timer(lambda: opt_ref.step(1e-3), iters))
        del opt_ref
    n_params = sum(b['numel'] for b in layout)
    out['adam'] = entry([ms], rows.adam_bytes(layout), f'{n_params} parameters in {len(layout)} buffers ({n_levels} grid levels, '
                        'NeRF grid levels 3-9 with fp16 gradients)', ref_ms)
    return out


def measure_nerf_mlp(device, physical: int, iters: int = 10, n: int = 65536 * 32) -> dict:
    """The NeRF MLP over one training step's NeRF level (2,097,152 samples by default; the reference model's widths,
    nerf_mlp.cu:440-455), CUDA-event means over `iters` runs after 3 warm-ups under the clock sampler:

    * inference forward: the tcgen05 kernel (zf_nerf_mlp_forward_tc through the C ABI) against the folded layer chain
      as cuBLAS bf16 GEMMs with bias + ReLU epilogues (`NerfMlp._forward`), against the measured bf16 peak (burst);
    * training iteration (pack, training forward, backward with the packed-weight gradients unfolded into the
      reference's parameters) through `ZipNeRFCudaBackend.NerfMlp`: the tcgen05 kernels (forward keeping v0-v2 and
      their ReLU masks, data-gradient chain, TMA-fed weight-gradient GEMMs) against the cuBLAS chain with this
      backend's ReLU-backward kernel (`_forward` / `_backward`).

    Inputs (336 MB at the default size) are larger than L2."""
    import ZipNeRFCudaBackend as backend
    from zipnerf_b200 import capi, nerf_mlp as nm
    layout = nm.NerfMlpLayout()
    gen = torch.Generator().manual_seed(7)
    params = torch.zeros(layout.numel)
    layout.initialize(params, gen)
    features = torch.randn(n, 56, generator=gen).bfloat16().to(device)
    inputs = torch.zeros(n, 96, dtype=torch.bfloat16, device=device)
    inputs[:, 64:91] = (torch.rand(n, 27, generator=gen) * 2 - 1).bfloat16().to(device)
    inputs[:, 95] = 1.0
    grad_outputs = torch.zeros(n, 8, dtype=torch.bfloat16, device=device)
    grad_outputs[:, :4] = torch.randn(n, 4, generator=gen).bfloat16().to(device)
    outputs = torch.empty(n, 8, dtype=torch.bfloat16, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    packed = {k: v.to(device) for k, v in nm.pack(layout, params).items()}
    mlp = backend.NerfMlp(50, 64, 256, 256, 4)
    device_params = params.to(device)
    grad_params = torch.zeros_like(device_params)
    flat = mlp.pack(device_params)
    peaks = measured_peaks()
    flop = 2 * nm.MACS_PER_SAMPLE * n

    def time_ms(fn) -> float:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(iters):
            fn()
        end.record()
        torch.cuda.synchronize()
        return start.elapsed_time(end) / iters

    def train_tc():
        p = mlp.pack(device_params)
        _, context = mlp.forward(features, inputs, p, True)
        mlp.backward(grad_outputs, features, p, context, device_params, grad_params)

    def train_chain():
        p = mlp.pack(device_params)
        _, context = mlp._forward(features, inputs, p, True)
        mlp._backward(grad_outputs, features, p, context, device_params, grad_params, backend.relu_backward_)

    out = {'config': f'{n} samples; density 64 x 56, combined 256 x 96, skip 8 x 96, view 2 x 256 x 256, rgb 8 x 256; '
                     'bf16 operands, fp32 accumulation (fp32 weight gradients)', 'flop_per_sample': 2 * nm.MACS_PER_SAMPLE,
           'training_flop_per_sample': 3 * 2 * nm.MACS_PER_SAMPLE}
    with ClockSampler(physical) as clocks:
        for name, fn in (('tcgen05', lambda: capi.nerf_mlp_forward_tc(features, inputs, packed, outputs, status)),
                         ('cublas_chain', lambda: mlp._forward(features, inputs, flat, False))):
            ms = time_ms(fn)
            tflops = flop / (ms * 1e-3) / 1e12
            out[name] = {'ms': ms, 'tflops': tflops, 'frac_of_bf16_peak': tflops / peaks['bf16_tflops']}
        for name, fn in (('training_tcgen05', train_tc), ('training_cublas_chain', train_chain)):
            ms = time_ms(fn)
            tflops = 3 * flop / (ms * 1e-3) / 1e12
            out[name] = {'ms': ms, 'tflops': tflops, 'frac_of_bf16_peak': tflops / peaks['bf16_tflops']}
    out['clocks'] = clocks.summary()
    out['tcgen05_status'] = int(mlp.status(device).item()) | int(status.item())
    out['ratio'] = out['cublas_chain']['ms'] / out['tcgen05']['ms']
    out['training_ratio'] = out['training_cublas_chain']['ms'] / out['training_tcgen05']['ms']
    return out


def measure_render(args, world: int, rank: int, device, barrier, frames: int = 3) -> dict:
    """Config 3: the inference render of one 1296 x 840 frame (zipnerf_b200/render.py: Morton-ordered pixels, view rays,
    two proposal forwards writing raw densities, deterministic resampling, the NeRF forward, the NeRF MLP and the final
    compositing), sharded over the ranks by contiguous Morton ranges with no collective. Timed on the device over
    `frames` frames after 2 warm-up frames; ms per frame is the max over ranks."""
    import torch.distributed as dist
    from zipnerf_b200 import render
    r = render.FrameRenderer(device, rank=rank, world=world)
    for _ in range(2):
        r.render()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(frames):
        r.render()
    end.record()
    barrier()
    ms = start.elapsed_time(end) / frames
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    n_rays = r.n_pixels
    out = {'ms_per_frame': ms, 'frames': frames, 'rays_per_frame': n_rays, 'mrays_per_s': n_rays / (ms * 1e-3) / 1e6,
           'featurized_msamples_per_s': n_rays * sum(render.N_SAMPLES) * N_MULTISAMPLES / (ms * 1e-3) / 1e6,
           'rays_per_gpu': r.n_rays, 'batch_rays': r.batch_rays,
           'config': f'config3: 1296 x 840 frame, Morton order, {world} contiguous Morton shard(s), 64 + 64 + 32 intervals, pattern seed -1, '
                     'interleaved thread mapping, forward only; NeRF MLP through ZipNeRFCudaBackend.NerfMlp.forward (inference)'}
    del r
    torch.cuda.empty_cache()
    return out


def measure_train_step(args, world: int, rank: int, device, barrier, steps: int = 10) -> dict:
    """The full training step (zipnerf_b200/train_step.py, the reference model's default grids): every rank trains on
    its own rays (weak scaling), each gradient buffer is averaged over the ranks with NCCL on a communication stream as
    soon as its backward has finished, and the single-launch Adam step follows. Timed on the device over `steps`
    iterations after the warm-up, max over ranks."""
    import torch.distributed as dist
    from zipnerf_b200 import sharding, train_step
    step = train_step.TrainStep(device, n_rays=args.rays, rank=rank, world=world)
    comm = torch.cuda.Stream() if world > 1 else None

    def after_backward(buffers):
        if world > 1:
            comm.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(comm):
                sharding.allreduce_gradients([b for b in buffers if b is not None], half_wire=args.half_wire)

    tails = []

    def exchange():
        if world > 1:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            torch.cuda.current_stream().wait_stream(comm)
            b.record()
            tails.append((a, b))

    for i in range(args.warmup):
        step.run(i, after_backward=after_backward, exchange=exchange)
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(steps):
        step.run(args.warmup + i, after_backward=after_backward, exchange=exchange)
    end.record()
    barrier()
    elapsed_ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([elapsed_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = t.item()
    ms = elapsed_ms / steps
    losses = step.loss_sums.tolist()
    tail = statistics.mean(a.elapsed_time(b) for a, b in tails[-steps:]) if tails else 0.0
    return {'ms': ms, 'steps': steps, 'exchange_tail_ms': tail, 'half_wire': args.half_wire, 'rays_per_s': world * args.rays / (ms * 1e-3), 'featurized_msamples_per_s': world * step.samples_per_step / (ms * 1e-3) / 1e6,
            'loss_sums_last_step': losses,
            'config': f'{args.rays} rays per GPU x (64 + 64 + 32) intervals; grids of the reference model (6 and 8 levels x 1 feature, 10 x 4, '
                      f'scale 2, 2^21); rays from a 185-view 1296 x 840 pool; gradient all-reduce over {world} GPU(s) and Adam; the NeRF MLP '
                      'with the reference interface on the tcgen05 kernels: forward (keeping v0-v2 and their ReLU masks), data-gradient '
                      'chain and TMA-fed weight-gradient GEMMs'}


def measure_e2e(step: Step, args, world: int, start_exchange, exchange, barrier) -> dict:
    """The metric through the public API with host buffers: every step copies its inputs (rays, interval endpoints,
    encoded directions, upstream gradients) from pinned host memory and reads back the MLP bias gradients. As in a
    training loop, the inputs are double-buffered: a copy stream brings step i + 1's inputs over PCIe while step i
    computes; the copies of every timed step (the first two included) lie inside the timed region."""
    device_sets = [step.input_buffers()]
    device_sets.append([torch.empty_like(t) for t in device_sets[0]])
    host = [t.cpu().pin_memory() for t in device_sets[0]]
    result_dev = [g['b1'] for g in step.prop_grads]
    result_host = torch.empty(len(result_dev), pin_memory=True)
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = result_host.numel() * result_host.element_size()
    compute = torch.cuda.current_stream()
    copies = torch.cuda.Stream()
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    released = [torch.cuda.Event(), torch.cuda.Event()]

    def copy_inputs(k: int) -> None:
        # into input set k, once the step that last read it has finished
        copies.wait_event(released[k])
        with torch.cuda.stream(copies):
            for d, h in zip(device_sets[k], host):
                d.copy_(h, non_blocking=True)
        copied[k].record(copies)

    def run(n_steps: int) -> None:
        for k in range(min(2, n_steps)):
            copy_inputs(k)
        for i in range(n_steps):
            k = i % 2
            compute.wait_event(copied[k])
            step.set_inputs(device_sets[k])
            step.run(after_backward=start_exchange, concurrent=True)
            exchange()
            result_host.copy_(torch.cat(result_dev), non_blocking=True)
            released[k].record(compute)
            if i + 2 < n_steps:
                copy_inputs(k)

    for k in range(2):
        released[k].record(compute)
    run(max(1, args.warmup))
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for k in range(2):
        released[k].record(compute)  # the timed copies start after the start event
    run(args.steps)
    end.record()
    barrier()
    step.set_inputs(device_sets[0])
    elapsed = start.elapsed_time(end)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([elapsed], device=step.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = t.item()
    return {'value': step.samples_per_step * world * args.steps / (elapsed / 1e3) / 1e6, 'unit': UNIT, 'h2d_bytes_per_step': h2d,
            'd2h_bytes_per_step': d2h, 'api': 'ZipNeRFCudaBackend._C.Featurizer', 'overlap': 'inputs double-buffered on a copy stream'}


_RESULT_FD = None


def emit(result: dict) -> None:
    """Writes the one JSON line to the process's original standard output."""
    line = (json.dumps(result) + '\n').encode()
    os.write(_RESULT_FD if _RESULT_FD is not None else 1, line)


def main() -> None:
    global _RESULT_FD
    # everything else written to standard output (library banners, e.g. NCCL's version line) goes to standard error,
    # so that standard output carries exactly the result line
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument('--gpus', type=int, default=1)
    parser.add_argument('--steps', type=int, default=20)
    parser.add_argument('--warmup', type=int, default=3)
    parser.add_argument('--impl', choices=['b200', 'reference'], default='b200')
    parser.add_argument('--rays', type=int, default=65536)
    parser.add_argument('--reference-rays', type=int, default=16384, help='ray sample of the CPU reference / baseline')
    parser.add_argument('--reference-repeats', type=int, default=5, help='passes over the ray sample timed for cpu_baseline')
    parser.add_argument('--skip-e2e', action='store_true')
    parser.add_argument('--skip-cpu-baseline', action='store_true')
    parser.add_argument('--skip-rows', action='store_true', help='skip the timing of the sampling and Adam kernels')
    parser.add_argument('--skip-train-step', action='store_true', help='skip the timing of the full training step')
    parser.add_argument('--skip-reference-cuda', action='store_true', help="skip the timing of the reference's own CUDA kernels")
    parser.add_argument('--skip-contention', action='store_true', help='skip the config-5 contention timing')
    parser.add_argument('--skip-nerf-mlp', action='store_true', help='skip the timing of the NeRF MLP (inference forward and training iteration)')
    parser.add_argument('--nerf-mlp-samples', type=int, default=65536 * 32, help='samples of the NeRF MLP timing (one step\'s NeRF level by default)')
    parser.add_argument('--skip-render', action='store_true', help='skip the timing of the config-3 frame render')
    parser.add_argument('--half-wire', choices=['fp16', 'fp32'], default='fp16',
                        help='wire format of the NeRF grid\'s fp16 gradients in the all-reduce (fp16: pre-divided fp16 sums; fp32: fp32 copies)')
    args = parser.parse_args()
    args.warmup = max(args.warmup, 3)  # at least 3 untimed warm-up steps
    if args.impl == 'reference':
        run_reference_arm(args)
    else:
        run_b200(args)


if __name__ == '__main__':
    main()

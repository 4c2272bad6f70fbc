"""A complete training step of Fused Zip-NeRF on this backend, in the order of the reference trainer
(Trainer.compute_gradients / training_iteration, Trainer.py:92-141, with Renderer.render_rays_training,
Renderer.py:44-84): training rays of random pool pixels, the two proposal levels' featurization with their fused
density MLPs and the resampling of the next level's intervals, the NeRF level's featurization, the NeRF MLP, the
final level's losses and gradients, the NeRF MLP backward, the grid and MLP backwards of all levels, the data-parallel
gradient average (one NCCL all-reduce per gradient buffer, each started as soon as its buffer is final) and the
single-launch Adam step with the grid regularizer and scale-feature magnitudes.

Model: the reference model's defaults (Model.py:65-78): proposal grids of 6 and 8 levels x 1 feature and the NeRF grid
of 10 levels x 4 features (base resolution 16, per-level scale 2, 2^21 entries), density MLPs of width 64, 64 + 64 + 32
intervals per ray, the view-direction encoding of degree 4; the trainer's loss weights and Adam settings
(Trainer.py:17-57). Data: a synthetic pool of 185 views of 1296 x 840 pixels (uniform-noise colors).

The NeRF MLP is this backend's `NerfMlp` with the reference's interface and parameter layout (nerf_mlp.cu:440-620):
`pack` every step (one kernel launch), the forward on the tcgen05 kernel keeping the training record (v0-v2 and one
ReLU-mask bit per column), the backward on the tcgen05 data-gradient and weight-gradient kernels, and the unfold of the
packed-weight gradients into the fp32 parameters (one kernel launch).

The two proposal levels' backwards run on their own streams beside the NeRF grid's backward: all three are independent
once the NeRF MLP's backward has run.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

N_SAMPLES = (64, 64, 32)
GRID_LEVELS = (6, 8, 10)
GRID_FEATURES = (1, 1, 4)
MLP_WIDTH = 64
DEGREE = 4
NEAR, FAR = 0.2, 1000.0
LOSS = {'charbonnier_padding': 0.001, 'interlevel': 0.01, 'blurs': (0.03, 0.003), 'distortion': 0.01, 'distortion_power': -0.25,
        'distortion_premult': 10000.0, 'grid_regularization': 0.1}
ADAM = {'beta1': 0.9, 'beta2': 0.99, 'eps': 1e-15}


LR = {'init': 0.01, 'final': 0.001, 'delay_steps': 2500, 'delay_mult': 1e-8, 'max_steps': 25000}  # Trainer.py:17-26


def learning_rate(step: int) -> float:
    """The trainer's learning-rate policy (Trainer.py:22-26,58-61): the mip-NeRF schedule, a log-linear decay from
    init to final over max_steps, scaled during the first delay_steps by a sine ramp from delay_mult to 1."""
    t = min(max(step / LR['max_steps'], 0.0), 1.0)
    rate = math.exp(math.log(LR['init']) * (1 - t) + math.log(LR['final']) * t)
    ramp = min(max(step / LR['delay_steps'], 0.0), 1.0)
    return rate * (LR['delay_mult'] + (1 - LR['delay_mult']) * math.sin(0.5 * math.pi * ramp))


def grid_layout(n_levels: int):
    sizes = [16 * 2 ** level for level in range(n_levels)]
    return sizes, [min(s ** 3, 2 ** 21) for s in sizes]


@dataclass
class Level:
    featurizer: object
    table: torch.Tensor
    grad: torch.Tensor
    grad_half: torch.Tensor | None
    magnitudes: torch.Tensor


class TrainStep:
    """One rank's model, optimizer and ray pool; run() is one training iteration on n_rays rays, this rank's share of a
    global batch of world x n_rays random rays: each rank draws its rays, jitter, backgrounds and multisample patterns
    from the iteration's seed with the rank in bits 40-55 (the reference draws them by local ray index, so equal seeds
    would repeat the same rays on every rank)."""

    def __init__(self, device, n_rays: int = 65536, rank: int = 0, world: int = 1, seed: int = 0, pool_views: int = 185) -> None:
        import ZipNeRFCudaBackend as backend
        from zipnerf_b200 import rows
        self.backend, self.device, self.n_rays, self.rank, self.world = backend, device, n_rays, rank, world
        g = torch.Generator(device=device).manual_seed(seed)
        self.levels = []
        mags = []
        for level, (n_levels, f) in enumerate(zip(GRID_LEVELS, GRID_FEATURES)):
            sizes, entries = grid_layout(n_levels)
            feat = backend.Featurizer(level, sizes, entries, f, MLP_WIDTH if level < 2 else 0)
            table = (torch.rand(sum(entries), f, generator=g, device=device) * 2 - 1) * backend.grid_max_value
            if level < 2:
                grad, grad_half = torch.zeros(table.numel(), device=device), None
            else:
                split = feat.n_fp32_grad_rows * f
                grad, grad_half = torch.zeros(split, device=device), torch.zeros(table.numel() - split, device=device, dtype=torch.float16)
            offsets = np.cumsum([0] + entries)
            m = torch.stack([(backend.grid_max_value ** 2 + table[a:b].square().mean()).sqrt() for a, b in zip(offsets[:-1], offsets[1:])])
            mags.append(m)
            self.levels.append(Level(feat, table, grad, grad_half, m))
        self.magnitudes = torch.cat(mags).contiguous()
        for i, level in enumerate(self.levels):  # views into the optimizer's magnitudes
            a = sum(len(grid_layout(n)[1]) for n in GRID_LEVELS[:i])
            level.magnitudes = self.magnitudes[a:a + GRID_LEVELS[i]]
        # proposal MLPs: one flat buffer (w0 [64, n_out], b0 [64], w1 [64], b1 [1] per level), padded to 4
        self.prop_layout = []
        n = 0
        for level in range(2):
            n_out = GRID_LEVELS[level] * 2
            self.prop_layout.append((n, n_out))
            n += 64 * n_out + 64 + 64 + 1
        self.prop_params = torch.zeros((n + 3) // 4 * 4, device=device)
        for level, (a, n_out) in enumerate(self.prop_layout):
            w0, _, w1, _ = self.proposal_mlp(self.prop_params, level)
            w0.uniform_(-math.sqrt(6 / n_out), math.sqrt(6 / n_out), generator=g)
            w1.uniform_(-math.sqrt(6 / 64), math.sqrt(6 / 64), generator=g)
        self.prop_grads = torch.zeros_like(self.prop_params)
        # the NeRF MLP: the reference's parameter table (nerf_mlp_parameters of the model's widths, Model.py:96-105),
        # He-uniform over the fan-in columns, zero biases
        self.nerf_mlp = backend.NerfMlp(GRID_LEVELS[2] * (GRID_FEATURES[2] + 1), MLP_WIDTH, 256, 256, DEGREE)
        layout = self.nerf_mlp.layout
        self.nerf_params = torch.zeros(layout.numel, device=device)
        layout.initialize(self.nerf_params, g)
        self.nerf_grads = torch.zeros_like(self.nerf_params)
        # the optimizer over the trainer's buffers (Trainer.py:44-57)
        nerf = self.levels[2]
        sizes, entries = grid_layout(GRID_LEVELS[2])
        n_fp32 = sum(1 for e in entries if e < 2 ** 20)
        split = nerf.featurizer.n_fp32_grad_rows * 4
        params = [self.levels[0].table.view(-1), self.levels[1].table.view(-1), nerf.table.view(-1)[:split], nerf.table.view(-1)[split:],
                  self.prop_params, self.nerf_params]
        grads = [self.levels[0].grad, self.levels[1].grad, nerf.grad, nerf.grad_half, self.prop_grads, self.nerf_grads]
        scale = backend.nerf_grid_grad_scale
        offsets = [[int(o) for o in np.cumsum([0] + grid_layout(GRID_LEVELS[0])[1])], [int(o) for o in np.cumsum([0] + grid_layout(GRID_LEVELS[1])[1])],
                   [int(o) * 4 for o in np.cumsum([0] + entries[:n_fp32])], [int(o) * 4 for o in np.cumsum([0] + entries[n_fp32:])], [], []]
        self.grad_buffers = grads
        self.optimizer = backend.Adam(params, grads, [1.0, 1.0, scale, scale, 1.0, 1.0], offsets, LOSS['grid_regularization'], backend.grid_max_value,
                                      ADAM['beta1'], ADAM['beta2'], ADAM['eps'], self.magnitudes)
        # the proposal levels' backwards run on their own streams beside the NeRF grid's backward (their inputs are final
        # once the final level's kernel has run, and their gradient buffers are disjoint from the NeRF level's)
        self.backward_streams = [torch.cuda.Stream(device=device) for _ in range(2)]
        self.pool = rows.ray_pool(device, n_views=pool_views)
        self.warp = rows.ray_warp(NEAR, FAR)
        self.loss_sums = None

    def proposal_mlp(self, buffer: torch.Tensor, level: int):
        a, n_out = self.prop_layout[level]
        w0 = buffer[a:a + 64 * n_out].view(64, n_out)
        b0 = buffer[a + 64 * n_out:a + 64 * n_out + 64]
        w1 = buffer[a + 64 * n_out + 64:a + 64 * n_out + 128].view(1, 64)
        b1 = buffer[a + 64 * n_out + 128:a + 64 * n_out + 129]
        return w0, b0, w1, b1

    def run(self, iteration: int, lr: float | None = None, anneal: float | None = None, after_backward=None, exchange=None,
            concurrent: bool = True) -> None:
        """One training iteration (learning rate and resampling anneal from the trainer's schedules unless given).
        after_backward(buffers) is called with each group of gradient buffers as soon as they are final (the NeRF grid,
        then each proposal level with the MLP buffers last), on the stream of the backward that wrote them; exchange() is
        called before the optimizer step (the data-parallel average must have finished). concurrent=False runs the
        proposal levels' backwards on this stream after the NeRF grid's."""
        if lr is None:
            lr = learning_rate(iteration)
        if anneal is None:  # schlick_bias(iteration / NUM_ITERATIONS, ANNEAL_SLOPE) (utils.py:30-32, Trainer.py:135-136)
            x = iteration / LR['max_steps']
            anneal = 10.0 * x / (9.0 * x + 1.0)
        b = self.backend
        R, dev = self.n_rays, self.device
        seed = iteration + (self.rank << 40)  # below the stream bits (random.cuh:20)
        p = self.pool
        origins, directions, radii, rgb, encoded, sdist, tdist = b.generate_rays(
            seed, R, p['view_offsets'], p['view_cameras'], p['camera_offsets'], p['local_directions'], p['c2w'], p['camera_radii'], p['pool_rgb'],
            DEGREE, N_SAMPLES[0], self.warp)
        empty = torch.empty(0, device=dev)
        proposals = []
        for level in range(2):
            lv = self.levels[level]
            n = N_SAMPLES[level]
            raw = torch.empty(R, n, device=dev)
            feats = torch.empty(R * n, lv.featurizer.n_output_features, device=dev)
            lv.featurizer.forward(origins, directions, radii, tdist, seed, False, lv.table, lv.magnitudes, *self.proposal_mlp(self.prop_params, level),
                                  raw, feats, empty, empty, empty)
            weights, s_next, t_next = b.composite_and_resample(raw, sdist, tdist, directions, anneal, N_SAMPLES[level + 1], seed, level + 1, self.warp)
            proposals.append({'raw': raw, 'features': feats, 'sdist': sdist, 'tdist': tdist, 'weights': weights})
            sdist, tdist = s_next, t_next
        nerf = self.levels[2]
        n = N_SAMPLES[2]
        features = torch.empty(R * n, 56, device=dev, dtype=torch.bfloat16)
        inputs = torch.empty(R * n, 96, device=dev, dtype=torch.bfloat16)
        nerf.featurizer.forward(origins, directions, radii, tdist, seed, False, nerf.table, nerf.magnitudes, empty, empty, empty, empty, empty, empty,
                                features, encoded, inputs)
        packed = self.nerf_mlp.pack(self.nerf_params)
        outputs, context = self.nerf_mlp.forward(features, inputs, packed, True)
        grad_outputs, proposal_grads, self.loss_sums = b.train_final(
            outputs.view(R, n, 8), sdist, tdist, [q['raw'] for q in proposals], [q['sdist'] for q in proposals], [q['tdist'] for q in proposals],
            [q['weights'] for q in proposals], directions, seed, rgb, LOSS['charbonnier_padding'], [LOSS['interlevel']] * 2, list(LOSS['blurs']),
            LOSS['distortion'], LOSS['distortion_power'], LOSS['distortion_premult'], True)
        grad_features = self.nerf_mlp.backward(grad_outputs.view(R * n, 8), features, packed, context, self.nerf_params, self.nerf_grads)
        # the NeRF grid's backward on this stream, the proposal levels' beside it on theirs (they start after the NeRF
        # MLP's tensor-core kernels, which hold whole SMs); this stream waits for them before the exchange and Adam, so
        # the step's temporaries are not reused early
        main = torch.cuda.current_stream()
        streams = self.backward_streams if concurrent else [main, main]
        for s in streams:
            s.wait_stream(main)
        nerf.featurizer.backward(origins, directions, radii, tdist, seed, grad_features, nerf.grad, nerf.grad_half)
        if after_backward is not None:
            after_backward([nerf.grad, nerf.grad_half, self.nerf_grads])
        for level, s in enumerate(streams):
            lv, q = self.levels[level], proposals[level]
            gw0, gb0, gw1, gb1 = self.proposal_mlp(self.prop_grads, level)
            with torch.cuda.stream(s):
                lv.featurizer.backward_mlp(origins, directions, radii, q['tdist'], seed, q['features'], proposal_grads[level],
                                           *self.proposal_mlp(self.prop_params, level)[:3], lv.grad, gw0, gb0, gw1.view(-1), gb1)
                if after_backward is not None:
                    after_backward([lv.grad] + ([self.prop_grads] if level == 1 else []))
        for s in streams:
            main.wait_stream(s)
        if exchange is not None:
            exchange()
        self.optimizer.step(lr)

    @property
    def samples_per_step(self) -> int:
        """featurized samples (interval x multisample) of one step: the unit of the featurization metric"""
        return self.n_rays * sum(N_SAMPLES) * 6

"""Host-side pieces of the training-step driver (zipnerf_b200/train_step.py), on the CPU: the learning-rate policy
against the trainer's configuration (Trainer.py:15-24, the mip-NeRF decay of NeRFICG's LRDecayPolicy), the grid
layouts against Model.py:17-24 with the defaults of Model.py:66-73, and the optimizer buffers against the model's
layouts. The step's NeRF MLP is the reference-interface NerfMlp, checked in test_nerf_mlp_host.py and on the GPU."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from zipnerf_b200 import train_step as ts


def test_learning_rate_follows_the_trainer_configuration():
    assert ts.LR == {'init': 0.01, 'final': 0.001, 'delay_steps': 2500, 'delay_mult': 1e-8, 'max_steps': 25000}
    init, final, delay, mult, steps = 0.01, 0.001, 2500, 1e-8, 25000
    for step in (0, 1, 100, 1249, 2500, 2501, 12500, 24999, 25000, 40000):
        t = np.clip(step / steps, 0.0, 1.0)
        ramp = mult + (1.0 - mult) * np.sin(0.5 * np.pi * np.clip(step / delay, 0.0, 1.0))
        expected = ramp * init * (final / init) ** t  # geometric interpolation: the same log-linear decay
        assert math.isclose(ts.learning_rate(step), expected, rel_tol=1e-12), step
    assert ts.learning_rate(0) == pytest.approx(init * mult)
    assert ts.learning_rate(steps) == pytest.approx(final)
    after_delay = [ts.learning_rate(s) for s in range(delay, steps + 1, 500)]
    assert all(a > b for a, b in zip(after_delay, after_delay[1:]))  # decays once the ramp is over


@pytest.mark.parametrize('n_levels,entries', [
    (6, [16 ** 3, 32 ** 3, 64 ** 3, 2 ** 21, 2 ** 21, 2 ** 21]),
    (8, [16 ** 3, 32 ** 3, 64 ** 3] + [2 ** 21] * 5),
    (10, [16 ** 3, 32 ** 3, 64 ** 3] + [2 ** 21] * 7),
])
def test_grid_layout_matches_the_model_defaults(n_levels, entries):
    sizes, level_entries = ts.grid_layout(n_levels)
    assert sizes == [round(16 * 2.0 ** level) for level in range(n_levels)]
    assert level_entries == entries  # 128^3 = 2^21 exactly: level 3 is the first hashed-size level
    assert tuple(ts.GRID_LEVELS) == (6, 8, 10) and tuple(ts.GRID_FEATURES) == (1, 1, 4) and ts.MLP_WIDTH == 64


def test_adam_buffers_match_the_model_layout():
    """The benchmark's optimizer buffers (rows.adam_layout, Trainer.py:44-57) against the model's own layouts: the
    grids of grid_layout, the proposal MLPs' flat buffer (w0 [64, levels x 2], b0, w1, b1 per level, padded to 4) and
    the NeRF MLP's parameter table."""
    from zipnerf_b200 import nerf_mlp, rows
    layout = rows.adam_layout()
    assert [b['half'] for b in layout] == [False, False, False, True, False, False]
    for b, n_levels in zip(layout[:2], (6, 8)):
        _, entries = ts.grid_layout(n_levels)
        assert b['numel'] == sum(entries) and b['offsets'] == list(np.cumsum([0] + entries))
    _, entries = ts.grid_layout(10)
    split = sum(1 for e in entries if e < 2 ** 20)  # levels below 2^20 entries keep fp32 gradients (3 of 10)
    assert split == 3 and layout[2]['numel'] == 4 * sum(entries[:split]) and layout[3]['numel'] == 4 * sum(entries[split:])
    assert layout[2]['scale'] == layout[3]['scale'] == 2.0 ** 20
    proposal = sum(64 * 2 * n + 64 + 64 + 1 for n in (6, 8))
    assert layout[4]['numel'] == (proposal + 3) // 4 * 4 == 2052
    assert layout[5]['numel'] == nerf_mlp.NerfMlpLayout().numel
    assert round(sum(b['numel'] for b in layout) / 1e6, 1) == 77.5  # the parameter count of the Adam row's figures

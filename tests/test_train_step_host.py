"""Host-side pieces of the training-step driver (zipnerf_b200/train_step.py), on the CPU: the learning-rate policy
against the trainer's configuration (Trainer.py:15-24, the mip-NeRF decay of NeRFICG's LRDecayPolicy), the grid
layouts against Model.py:17-24 with the defaults of Model.py:66-73, and the chain rule of the NeRF MLP stand-in's
hand-written backward against autograd on the same bf16-rounded weights. The ReLU-backward kernel itself is checked
against PyTorch on the GPU (test_gpu_train_step.py); here a torch test double takes its place so that only the
stand-in's transposes, skip terms and accumulations are under test."""
from __future__ import annotations

import math
import sys
import types

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


def test_nerf_mlp_layout_is_one_padded_flat_buffer():
    mlp = ts.NerfMlp(torch.device('cpu'), torch.Generator().manual_seed(0))
    end = 0
    for name, shape in ts.NerfMlp.SHAPES:
        offset, stored = mlp.offsets[name]
        assert offset == end and stored == shape
        end += math.prod(shape)
        view = mlp.view(mlp.params, name)
        assert view.shape == shape and view.data_ptr() == mlp.params.data_ptr() + 4 * offset
        if len(shape) == 1:
            assert not view.any()  # biases start at zero
        else:
            bound = math.sqrt(6.0 / shape[1])  # He-uniform
            assert view.abs().max() <= bound and view.abs().max() > 0.5 * bound
    assert mlp.numel == (end + 3) // 4 * 4 and mlp.params.numel() == mlp.numel and mlp.grads.shape == mlp.params.shape


def _relu_backward_double(grad: torch.Tensor, activation: torch.Tensor, bias_grad: torch.Tensor) -> None:
    """The contract of relu_backward_ (zf_mlp.h) in torch: grad *= (activation > 0), NaN masking; bias_grad += the
    column sums of the masked gradient in fp32 when bias_grad is not empty."""
    grad.copy_(torch.where(activation > 0, grad, torch.zeros_like(grad)))
    if bias_grad.numel():
        bias_grad += grad.float().sum(0)


def test_nerf_mlp_backward_is_the_chain_rule_of_its_forward(monkeypatch):
    monkeypatch.setitem(sys.modules, 'ZipNeRFCudaBackend', types.SimpleNamespace(relu_backward_=_relu_backward_double))
    g = torch.Generator().manual_seed(5)
    mlp = ts.NerfMlp(torch.device('cpu'), g)
    for name, shape in ts.NerfMlp.SHAPES:  # nonzero biases so that every bias gradient path matters
        if len(shape) == 1:
            mlp.view(mlp.params, name).uniform_(-0.2, 0.2, generator=g)
    n = 384
    features = torch.randn(n, 56, generator=g).bfloat16()
    inputs = torch.zeros(n, 96).bfloat16()
    inputs[:, 64:] = torch.randn(n, 32, generator=g).bfloat16()
    direction_block = inputs[:, 64:].clone()
    outputs, context = mlp.forward(features, inputs)
    grad_outputs = torch.randn(n, 8, generator=g).bfloat16()
    grad_outputs[:, 4:] = 0  # padding columns carry no gradient, as train_final writes them
    grad_features = mlp.backward(grad_outputs, context)

    # the same network in fp32 on the bf16-rounded parameters, differentiated by autograd; each layer's output is
    # rounded to bf16 as the stand-in stores it (the rounding passes the gradient straight through), so both see the
    # same ReLU masks
    def stored(t):
        return t + (t.bfloat16().float() - t).detach()

    p = {name: mlp.view(mlp.params, name).bfloat16().float().requires_grad_() for name, _ in ts.NerfMlp.SHAPES}
    x = features.float().requires_grad_()
    hidden = stored(torch.relu(x @ p['density'].t() + p['density_b']))
    net_in = torch.cat([hidden, direction_block.float()], dim=1)
    v0 = stored(torch.relu(net_in @ p['combined'].t()))
    v1 = stored(torch.relu(v0 @ p['view_1'].t() + p['view_1_b']))
    v2 = stored(torch.relu(v1 @ p['view_2'].t() + p['view_2_b']))
    reference = net_in @ p['skip'].t() + v2 @ p['rgb'].t()
    assert torch.allclose(outputs.float(), reference, rtol=0.05, atol=0.05 * reference.abs().mean().item())
    (reference * grad_outputs.float()).sum().backward()

    def relative_error(a, b):
        return ((a.float() - b).norm() / b.norm().clamp_min(1e-30)).item()

    # bf16 intermediate gradients: relative errors near 3e-3; a wrong transpose or a lost term is O(1)
    errors = {name: relative_error(mlp.view(mlp.grads, name), p[name].grad) for name, _ in ts.NerfMlp.SHAPES}
    errors['features'] = relative_error(grad_features, x.grad)
    assert max(errors.values()) < 1e-2, errors
    assert not mlp.grads[mlp.params.numel() - (mlp.numel - sum(math.prod(s) for _, s in ts.NerfMlp.SHAPES)):].any()


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

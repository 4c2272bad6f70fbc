"""The full training step on one GPU (zipnerf_b200/train_step.py): every stage runs through this backend's kernels in
the reference trainer's order; after each step the losses are finite, every gradient buffer has been consumed and
zeroed by the Adam step, the parameters and scale-feature magnitudes moved, and repeated steps stay finite. Also the
NeRF MLP's ReLU backward with bias gradient (zf_mlp.h) against plain PyTorch."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_training_steps_run_and_update_the_model(cuda_device):
    from zipnerf_b200 import train_step
    step = train_step.TrainStep(cuda_device, n_rays=4096, pool_views=3)
    tables = [level.table.clone() for level in step.levels]
    mlp = (step.prop_params.clone(), step.nerf_params.clone())
    magnitudes = step.magnitudes.clone()
    losses = []
    for iteration in range(3):
        step.run(iteration)
        torch.cuda.synchronize()
        losses.append(step.loss_sums.clone())
        # all four terms present: data, mse, interlevel (the proposal weights against the final ones), distortion
        assert torch.isfinite(step.loss_sums).all() and (step.loss_sums > 0).all(), step.loss_sums
        for buffer in step.grad_buffers:
            assert not buffer.any(), 'the Adam step zeroes every gradient buffer'
    for before, level in zip(tables, step.levels):
        assert torch.isfinite(level.table).all() and not torch.equal(before, level.table)
    assert not torch.equal(mlp[0], step.prop_params) and not torch.equal(mlp[1], step.nerf_params)
    assert int(step.nerf_mlp.status(cuda_device).item()) == 0  # no wait of the tensor-core forward ran out
    assert torch.isfinite(step.magnitudes).all() and not torch.equal(magnitudes, step.magnitudes)
    assert float(step.optimizer.regularization()) > 0.0
    # the data term (charbonnier, per ray) is bounded by the colors' range
    assert all(0.0 < float(l[0]) < 2.0 for l in losses)


def test_concurrent_backwards_train_like_the_sequential_step(cuda_device):
    """The proposal levels' backwards on their own streams beside the NeRF grid's backward give the model of the
    sequential step: two models from the same initial state, trained three steps each way, have the same losses up to
    the gradient atomics' summation order (a backward that read a buffer before it was written would show here)."""
    from zipnerf_b200 import train_step
    losses = []
    for concurrent in (True, False):
        step = train_step.TrainStep(cuda_device, n_rays=4096, pool_views=3)
        out = []
        for iteration in range(3):
            step.run(iteration, concurrent=concurrent)
            out.append(step.loss_sums.clone())
        torch.cuda.synchronize()
        losses.append(torch.stack(out).double())
    torch.testing.assert_close(losses[0], losses[1], rtol=1e-3, atol=1e-7)


@pytest.mark.parametrize('cols,act_cols', [(256, 256), (64, 96), (8, 8), (24, 24)])
def test_relu_backward_matches_torch(cuda_device, cols, act_cols):
    """The masked gradient equals PyTorch's grad * (act > 0) exactly (NaN activations mask); the bias gradient (fp32
    column sums, atomics) to summation order. act_cols > cols: the activation is a column slice of a wider buffer."""
    import ZipNeRFCudaBackend as backend
    g = torch.Generator(device=cuda_device).manual_seed(cols)
    n = 10007
    grad = torch.randn(n, cols, generator=g, device=cuda_device).to(torch.bfloat16)
    act_full = torch.randn(n, act_cols, generator=g, device=cuda_device).relu().to(torch.bfloat16)
    act_full[::97, 0] = float('nan')
    act = act_full[:, :cols]
    expected = torch.where(act > 0, grad, torch.zeros_like(grad))
    bias = torch.full((cols,), 0.5, device=cuda_device)
    out = grad.clone()
    backend.relu_backward_(out, act, bias)
    torch.cuda.synchronize()
    assert torch.equal(out, expected)
    torch.testing.assert_close(bias, 0.5 + expected.float().sum(0), rtol=1e-4, atol=1e-3)
    out2 = grad.clone()
    backend.relu_backward_(out2, act, torch.empty(0, device=cuda_device))
    assert torch.equal(out2, expected)

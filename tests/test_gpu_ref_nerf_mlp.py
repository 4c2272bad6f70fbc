"""The NeRF MLP against the reference's own NerfMlp (mlp/src/nerf_mlp.cu: bf16 cuBLASLt GEMMs with fused epilogues),
compiled from its source by oracle/ref_mlp/build.py into oracle/_ref/ref_mlp: the same fp32 parameters, features,
direction inputs and output gradients through both, training forward and backward (nerf_mlp.cu:503-620). Both chains
round weights and activations to bf16 and accumulate in fp32 but in different GEMM orders, so outputs and gradients
agree within bf16 rounding (relative norm errors measured near 3e-3; bound 1e-2)."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

REF_MLP = Path(__file__).resolve().parent.parent / 'oracle' / '_ref' / 'ref_mlp'


@pytest.fixture(scope='module')
def ref_mlp():
    if not (REF_MLP / 'zf_ref_mlp.so').exists():
        pytest.skip('the reference NeRF MLP checker is not built (oracle/ref_mlp/build.py needs the reference sources)')
    sys.path.insert(0, str(REF_MLP))
    import zf_ref_mlp
    return zf_ref_mlp


def rel(a: torch.Tensor, b: torch.Tensor) -> float:
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def test_parameter_table_is_the_references(ref_mlp):
    """nerf_mlp_parameters gives the reference's names, shapes and fan-ins for the model's defaults and another width."""
    import ZipNeRFCudaBackend as backend
    for args in ((50, 64, 256, 256, 4), (50, 64, 128, 128, 4)):
        ours = [(name, list(shape), fan_in) for name, shape, fan_in in backend.nerf_mlp_parameters(*args)]
        assert ours == [(name, list(shape), fan_in) for name, shape, fan_in in ref_mlp.nerf_mlp_parameters(*args)]


@pytest.mark.parametrize('n', [4096, 57_003])
def test_nerf_mlp_matches_the_reference_nerf_mlp(ref_mlp, cuda_device, n):
    import ZipNeRFCudaBackend as backend
    from zipnerf_b200 import nerf_mlp as nm
    layout = nm.NerfMlpLayout()
    gen = torch.Generator().manual_seed(n + 1)
    params = torch.zeros(layout.numel)
    layout.initialize(params, gen)
    for name, _, fan_in in layout.parameters:  # nonzero biases, so that every bias fold matters
        if fan_in == 0:
            layout.view(params, name).uniform_(-0.3, 0.3, generator=gen)
    features = torch.zeros(n, 56)
    features[:, :50] = torch.randn(n, 50, generator=gen)
    inputs = torch.zeros(n, 96)
    inputs[:, 64:91] = torch.rand(n, 27, generator=gen) * 2 - 1
    inputs[:, 95] = 1.0
    grad_outputs = torch.zeros(n, 8)
    grad_outputs[:, :4] = torch.randn(n, 4, generator=gen)
    params = params.to(cuda_device)
    features = features.bfloat16().to(cuda_device)
    grad_outputs = grad_outputs.bfloat16().to(cuda_device)
    inputs_ref, inputs_ours = inputs.bfloat16().to(cuda_device), inputs.bfloat16().to(cuda_device)

    ref, ours = ref_mlp.NerfMlp(50, 64, 256, 256, 4), backend.NerfMlp(50, 64, 256, 256, 4)
    assert (ref.n_features, ref.n_inputs) == (ours.n_features, ours.n_inputs)
    ref_packed, ours_packed = ref.pack(params), ours.pack(params)
    ref_out, ref_context = ref.forward(features, inputs_ref, ref_packed, True)
    ours_out, ours_context = ours.forward(features, inputs_ours, ours_packed, True)
    grad_ref, grad_ours = torch.zeros_like(params), torch.zeros_like(params)
    ref_grad_features = ref.backward(grad_outputs, features, ref_packed, ref_context, params, grad_ref)
    ours_grad_features = ours.backward(grad_outputs, features, ours_packed, ours_context, params, grad_ours)
    torch.cuda.synchronize()
    assert int(ours.status(cuda_device).item()) == 0

    errors = {'outputs': rel(ours_out[:, :4], ref_out[:, :4]), 'hidden': rel(inputs_ours[:, :64], inputs_ref[:, :64]),
              'grad_features': rel(ours_grad_features[:, :50], ref_grad_features[:, :50])}
    # the direction block is the caller's and stays untouched by both
    assert torch.equal(inputs_ours[:, 64:].view(torch.int16), inputs_ref[:, 64:].view(torch.int16))
    for name, _, _ in layout.parameters:
        expected = layout.view(grad_ref, name)
        if expected.abs().max() > 0:
            errors[name] = rel(layout.view(grad_ours, name), expected)
    assert max(errors.values()) < 1e-2, errors

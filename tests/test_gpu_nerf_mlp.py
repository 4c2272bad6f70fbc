"""The NeRF MLP with the reference's interface (`ZipNeRFCudaBackend.NerfMlp`, zipnerf_b200/nerf_mlp.py) on the GPU:
pack, the training forward and the backward (cuBLAS bf16 GEMMs with bias + ReLU epilogues, this backend's ReLU
backward kernel, the unfold of the packed-weight gradients) against autograd of the fold and the same layer chain
with the same bf16 roundings (weights, activations), for the reference model's defaults (nerf_mlp.cu:440-620)."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _stored(t: torch.Tensor) -> torch.Tensor:
    """bf16 rounding that passes the gradient straight through"""
    return t + (t.bfloat16().float() - t).detach()


def test_nerf_mlp_matches_autograd(cuda_device):
    import ZipNeRFCudaBackend as backend
    from zipnerf_b200 import nerf_mlp as nm
    layout = nm.NerfMlpLayout()
    gen = torch.Generator().manual_seed(3)
    params = torch.zeros(layout.numel)
    layout.initialize(params, gen)
    for name, _, fan_in in layout.parameters:  # nonzero biases so that every bias fold matters
        if fan_in == 0:
            layout.view(params, name).uniform_(-0.3, 0.3, generator=gen)
    n = 4096
    features = torch.zeros(n, 56)
    features[:, :50] = torch.randn(n, 50, generator=gen)
    block = torch.zeros(n, 32)
    block[:, :27] = torch.rand(n, 27, generator=gen) * 2 - 1
    block[:, 31] = 1.0  # the bias lane
    grad_outputs = torch.randn(n, 8, generator=gen)
    grad_outputs[:, 4:] = 0
    params, features = params.to(cuda_device), features.bfloat16().to(cuda_device)
    block, grad_outputs = block.bfloat16().to(cuda_device), grad_outputs.bfloat16().to(cuda_device)

    mlp = backend.NerfMlp(50, 64, 256, 256, 4)
    assert (mlp.n_features, mlp.n_inputs) == (56, 96)
    packed = mlp.pack(params)
    inputs = torch.zeros(n, 96, dtype=torch.bfloat16, device=cuda_device)
    inputs[:, 64:] = block
    outputs, context = mlp.forward(features, inputs, packed, True)
    grad_params = torch.zeros_like(params)
    grad_features = mlp.backward(grad_outputs, features, packed, context, params, grad_params)
    torch.cuda.synchronize()

    p = params.clone().requires_grad_()
    x = features.float().requires_grad_()
    w = {k: _stored(v) for k, v in nm.fold(layout, p, 56, 8).items()}
    h = _stored(torch.relu(x @ w['density'].t() + w['density_bias']))
    net_in = torch.cat([h, block.float()], 1)
    v0 = _stored(torch.relu(net_in @ w['combined'].t()))
    v1 = _stored(torch.relu(v0 @ w['view_1'].t() + w['view_1_bias']))
    v2 = _stored(torch.relu(v1 @ w['view_2'].t() + w['view_2_bias']))
    expected = net_in @ w['skip'].t() + v2 @ w['rgb'].t()
    (expected * grad_outputs.float()).sum().backward()

    def rel(a, b):
        return ((a.float() - b).norm() / b.norm()).item()

    # bf16 intermediate gradients and cuBLAS accumulation order: relative errors of at most 3.4e-3 on a B200
    errors = {name: rel(layout.view(grad_params, name), layout.view(p.grad, name)) for name, _, _ in layout.parameters}
    errors['features'] = rel(grad_features, x.grad)
    errors['outputs'] = rel(outputs, expected)
    assert max(errors.values()) < 1e-2, errors
    assert rel(inputs[:, :64], h.detach()) < 1e-2  # the hidden layer is written into the inputs
    # inference: the same outputs, no context
    out_inference, no_context = mlp.forward(features, inputs.clone(), packed, False)
    assert no_context == [] and rel(out_inference, outputs.float()) < 1e-3


def test_nerf_mlp_parameters_is_the_reference_table():
    import ZipNeRFCudaBackend as backend
    table = backend.nerf_mlp_parameters(50, 64, 256, 256, 4)
    assert table[0] == ('density_0.weight', [64, 56], 50) and table[-1] == ('rgb.bias', [3], 0) and len(table) == 14


@pytest.mark.parametrize('n', [128, 4133, 57_003])
def test_tensor_core_forward_matches_the_layer_chain(cuda_device, n):
    """zf_nerf_mlp_forward_tc (one persistent tcgen05 kernel) against the same packed layer chain computed in fp32 from
    its bf16 operands with the kernel's roundings (bias + ReLU in fp32, then bf16): outputs within 1e-2 (1.7e-3
    measured), the hidden layer written into the inputs, zero padding outputs, no timed-out wait. n = 4133 leaves a
    ragged last tile; n = 57,003 gives every CTA of a B200 several tiles (446 tiles over 148 SMs)."""
    from zipnerf_b200 import capi, nerf_mlp as nm
    layout = nm.NerfMlpLayout()
    gen = torch.Generator().manual_seed(7)
    params = torch.zeros(layout.numel)
    layout.initialize(params, gen)
    for name, _, fan_in in layout.parameters:
        if fan_in == 0:
            layout.view(params, name).uniform_(-0.3, 0.3, generator=gen)
    packed = {k: v.to(cuda_device) for k, v in nm.pack(layout, params).items()}
    features = torch.zeros(n, 56)
    features[:, :50] = torch.randn(n, 50, generator=gen)
    block = torch.zeros(n, 32)
    block[:, :27] = torch.rand(n, 27, generator=gen) * 2 - 1
    block[:, 31] = 1.0
    features = features.bfloat16().to(cuda_device)
    inputs = torch.zeros(n, 96, dtype=torch.bfloat16, device=cuda_device)
    inputs[:, 64:] = block.bfloat16().to(cuda_device)
    outputs = torch.full((n, 8), float('nan'), dtype=torch.bfloat16, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    capi.nerf_mlp_forward_tc(features, inputs, packed, outputs, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0

    w = {k: (v if k.endswith('_bias') else nm.row_major(v, nm.K_SLICE[k])).float() for k, v in packed.items()}
    h = torch.relu(torch.nn.functional.pad(features.float(), (0, 8)) @ w['density'].t() + w['density_bias']).bfloat16().float()
    x = torch.cat([h, inputs[:, 64:].float()], 1)
    v0 = torch.relu(x @ w['combined'].t()).bfloat16().float()
    v1 = torch.relu(v0 @ w['view_1'].t() + w['view_1_bias']).bfloat16().float()
    v2 = torch.relu(v1 @ w['view_2'].t() + w['view_2_bias']).bfloat16().float()
    expected = (x @ w['skip'].t() + v2 @ w['rgb'].t())[:, :8]

    def rel(a, b):
        return ((a.float() - b).norm() / b.norm()).item()

    assert torch.isfinite(outputs.float()).all() and not outputs[:, 4:].any()
    assert rel(outputs, expected) < 1e-2 and rel(inputs[:, :64], h) < 1e-2


def test_tensor_core_forward_rows_are_independent_of_the_batch(cuda_device):
    """Each sample's outputs depend on its own row only: the first rows of a batch, run alone, equal the same rows of the
    whole batch bit for bit (what the sharded render relies on), and a second run of the batch repeats the first."""
    from zipnerf_b200 import capi, nerf_mlp as nm
    layout = nm.NerfMlpLayout()
    gen = torch.Generator().manual_seed(11)
    params = torch.zeros(layout.numel)
    layout.initialize(params, gen)
    packed = {k: v.to(cuda_device) for k, v in nm.pack(layout, params).items()}
    n = 30_001
    features = torch.randn(n, 56, generator=gen).bfloat16().to(cuda_device)
    inputs = torch.zeros(n, 96, dtype=torch.bfloat16, device=cuda_device)
    inputs[:, 64:91] = (torch.rand(n, 27, generator=gen) * 2 - 1).bfloat16().to(cuda_device)
    inputs[:, 95] = 1.0
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    whole, again = (torch.empty(n, 8, dtype=torch.bfloat16, device=cuda_device) for _ in range(2))
    capi.nerf_mlp_forward_tc(features, inputs, packed, whole, status)
    capi.nerf_mlp_forward_tc(features, inputs, packed, again, status)
    m = 1_000
    part_inputs = inputs[:m].clone()
    part = torch.empty(m, 8, dtype=torch.bfloat16, device=cuda_device)
    capi.nerf_mlp_forward_tc(features[:m].contiguous(), part_inputs, packed, part, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(whole.view(torch.int16), again.view(torch.int16))
    assert torch.equal(part.view(torch.int16), whole[:m].view(torch.int16))
    assert torch.equal(part_inputs.view(torch.int16), inputs[:m].view(torch.int16))


@pytest.mark.parametrize('n', [5, 8, 136, 4133, 57_003])
def test_tensor_core_backward_matches_the_gemm_chain(cuda_device, n):
    """NerfMlp.backward on the tensor cores (zf_nerf_mlp_backward_tc: the data-gradient kernel, then the weight-gradient
    GEMMs over the samples) against the same folded chain as bf16 GEMMs through torch (`_backward`, fp32 weight
    gradients) on the same forward context: feature and parameter gradients within 1e-2 relative (bf16 intermediate
    gradients, other summation orders), and no timed-out wait. n = 5 and 8 are less than one tile, 136 a partial second
    tile, 4,133 and 57,003 ragged last tiles; 57,003 gives every CTA several tiles."""
    import ZipNeRFCudaBackend as backend
    from zipnerf_b200 import nerf_mlp as nm
    layout = nm.NerfMlpLayout()
    gen = torch.Generator().manual_seed(n)
    params = torch.zeros(layout.numel)
    layout.initialize(params, gen)
    for name, _, fan_in in layout.parameters:
        if fan_in == 0:
            layout.view(params, name).uniform_(-0.3, 0.3, generator=gen)
    features = torch.zeros(n, 56)
    features[:, :50] = torch.randn(n, 50, generator=gen)
    inputs = torch.zeros(n, 96)
    inputs[:, 64:91] = torch.rand(n, 27, generator=gen) * 2 - 1
    inputs[:, 95] = 1.0
    grad_outputs = torch.zeros(n, 8)
    grad_outputs[:, :4] = torch.randn(n, 4, generator=gen)
    params, features = params.to(cuda_device), features.bfloat16().to(cuda_device)
    inputs, grad_outputs = inputs.bfloat16().to(cuda_device), grad_outputs.bfloat16().to(cuda_device)
    mlp = backend.NerfMlp(50, 64, 256, 256, 4)
    packed = mlp.pack(params)
    _, context = mlp.forward(features, inputs, packed, True)
    grad_tc, grad_chain = torch.zeros_like(params), torch.zeros_like(params)
    features_tc = mlp.backward(grad_outputs, features, packed, context, params, grad_tc)
    features_chain = mlp._backward(grad_outputs, features, packed, [t.clone() for t in context], params, grad_chain, backend.relu_backward_)
    torch.cuda.synchronize()
    assert int(mlp.status(cuda_device).item()) == 0

    def rel(a, b):
        return ((a.float() - b.float()).norm() / b.float().norm()).item()

    errors = {name: rel(layout.view(grad_tc, name), layout.view(grad_chain, name)) for name, _, _ in layout.parameters
              if layout.view(grad_chain, name).abs().max() > 0}
    errors['features'] = rel(features_tc, features_chain)
    assert max(errors.values()) < 1e-2, errors


def _backward_case(cuda_device, n, seed):
    import ZipNeRFCudaBackend as backend
    from zipnerf_b200 import nerf_mlp as nm
    layout = nm.NerfMlpLayout()
    gen = torch.Generator().manual_seed(seed)
    params = torch.zeros(layout.numel)
    layout.initialize(params, gen)
    for name, _, fan_in in layout.parameters:
        if fan_in == 0:
            layout.view(params, name).uniform_(-0.3, 0.3, generator=gen)
    features = torch.zeros(n, 56)
    features[:, :50] = torch.randn(n, 50, generator=gen)
    inputs = torch.zeros(n, 96)
    inputs[:, 64:91] = torch.rand(n, 27, generator=gen) * 2 - 1
    inputs[:, 95] = 1.0
    grad_outputs = torch.zeros(n, 8)
    grad_outputs[:, :4] = torch.randn(n, 4, generator=gen)
    mlp = backend.NerfMlp(50, 64, 256, 256, 4)
    params = params.to(cuda_device)
    return (mlp, layout, params, features.bfloat16().to(cuda_device), inputs.bfloat16().to(cuda_device),
            grad_outputs.bfloat16().to(cuda_device))


def test_training_record_masks_are_the_activations_signs(cuda_device):
    """The training forward's record holds v0, v1, v2 and, behind them, one bit per column set exactly where the stored
    bf16 value is positive (bit c % 32 of word c / 32), for v0-v2 and for the hidden layer h the forward writes into
    inputs[:, 0:64] (n = 5,003: a ragged last tile)."""
    mlp, _, params, features, inputs, _ = _backward_case(cuda_device, 5_003, 11)
    n = features.shape[0]
    packed = mlp.pack(params)
    _, context = mlp.forward(features, inputs, packed, True)
    torch.cuda.synchronize()
    record = context[1].as_strided((3 * n * 256 + 3 * n * 16 + 4 * n,), (1,))
    words = record[3 * n * 256:].view(torch.int32)
    bit = torch.arange(32, device=cuda_device)

    def expand(w, columns):
        return ((w.view(torch.int32).unsqueeze(-1) >> bit) & 1).reshape(n, columns).bool()

    for k in range(3):
        expected = context[1 + k].float() > 0
        assert torch.equal(expand(words[k * n * 8:(k + 1) * n * 8].view(n, 8), 256), expected), k
    assert torch.equal(expand(words[3 * n * 8:].view(n, 2), 64), inputs[:, :64].float() > 0)


def test_tensor_core_backward_reads_features_with_their_own_stride(cuda_device):
    """zf_nerf_mlp_backward_tc takes separate row strides for features and grad_features: features as the first 56
    columns of a [n, 64] buffer (stride 64) and grad_features as a [n, 72] buffer's give the same gradients bit for bit
    as the contiguous call."""
    from zipnerf_b200 import capi
    mlp, layout, params, features, inputs, grad_outputs = _backward_case(cuda_device, 9_001, 5)
    n = features.shape[0]
    packed = mlp.pack(params)
    _, context = mlp.forward(features, inputs, packed, True)
    record = context[1].as_strided((capi.nerf_mlp_record_size(n) // 2,), (1,))
    weights = mlp._tc_weights(packed, ('rgb_t', 'view_2_t', 'view_1_t', 'combined_t', 'skip_t', 'density_t'))
    workspace = torch.empty(capi.load().zf_nerf_mlp_backward_workspace_size(n), dtype=torch.uint8, device=cuda_device)
    results = []
    for feature_width, grad_width in ((56, 56), (64, 72)):
        wide = torch.zeros(n, feature_width, dtype=torch.bfloat16, device=cuda_device)
        wide[:, :56] = features
        grad_features = torch.zeros(n, grad_width, dtype=torch.bfloat16, device=cuda_device)
        grads = {name: torch.zeros(shape, device=cuda_device) for name, shape in capi.NERF_MLP_GRAD_SHAPES.items()}
        # one CTA's share of the weight gradients is summed by fp32 atomics in any order: compare up to that
        capi.nerf_mlp_backward_tc(grad_outputs, wide[:, :56], inputs, record, weights, grad_features[:, :56], grads, workspace,
                                  mlp.status(cuda_device))
        torch.cuda.synchronize()
        results.append((grad_features[:, :56].clone(), grads))
    assert int(mlp.status(cuda_device).item()) == 0
    assert torch.equal(results[0][0].view(torch.int16), results[1][0].view(torch.int16))
    for name in capi.NERF_MLP_GRAD_SHAPES:
        a, b = results[0][1][name], results[1][1][name]
        assert ((a - b).norm() <= 1e-5 * b.norm() + 1e-30).item(), name


def test_pack_kernel_matches_the_torch_fold(cuda_device):
    """zf_nerf_mlp_pack (one launch) against the fold computed with torch on the CPU (`NerfMlp.pack` of host
    parameters): every section of the packed buffer (row-major, the tensor-core forward's K-sliced weights and fp32
    biases, the transposed weights) holds the same values; the folded columns (fp32 sums over the 256 bottleneck
    outputs, in another order on each side) may differ by one bf16 step, everything copied is equal bit for bit."""
    import ZipNeRFCudaBackend as backend
    mlp, layout, params, _, _, _ = _backward_case(cuda_device, 8, 21)
    on_device = mlp.pack(params).cpu()
    on_host = mlp._pack(params.cpu())
    assert on_device.shape == on_host.shape
    a, b = on_device.float(), on_host.float()
    steps = (a - b).abs() / b.abs().clamp_min(1e-30)
    differing = (a != b)
    assert float(steps[differing].max()) <= 2 ** -7 if bool(differing.any()) else True
    # the copied tensors are equal bit for bit: view_1, view_2 and their biases in every section
    for name in ('view_1', 'view_2', 'view_1_bias', 'view_2_bias'):
        o, shape = mlp._offsets[name], mlp._shapes[name]
        size = shape[0] * (shape[1] if len(shape) > 1 else 1)
        assert torch.equal(on_device[o:o + size].view(torch.int16), on_host[o:o + size].view(torch.int16)), name
    assert int(differing.sum()) < 0.01 * on_device.numel()


def test_unfold_kernel_matches_autograd_of_the_fold(cuda_device):
    """zf_nerf_mlp_unfold_grads (one launch) against autograd of the fold on random packed-weight gradients: every
    parameter's gradient within 1e-5 relative (fp32 sums in other orders); it accumulates into the given buffer."""
    from zipnerf_b200 import capi, nerf_mlp as nm
    mlp, layout, params, _, _, _ = _backward_case(cuda_device, 8, 22)
    gen = torch.Generator().manual_seed(5)
    grads = {name: torch.randn(shape, generator=gen).to(cuda_device) for name, shape in capi.NERF_MLP_GRAD_SHAPES.items()}
    with torch.enable_grad():
        p = params.detach().double().requires_grad_()
        folded = nm.fold(layout, p)
        (expected,) = torch.autograd.grad([folded[name] for name in nm.PACKED_ORDER], p, [grads[name].double() for name in nm.PACKED_ORDER])
    start = torch.full_like(params, 0.25)
    got = start.clone()
    capi.nerf_mlp_unfold_grads(params, grads, got)
    torch.cuda.synchronize()
    for name, _, _ in layout.parameters:
        e, g = layout.view(expected, name), layout.view(got - start, name).double()
        assert float((g - e).norm()) <= 1e-5 * float(e.norm()) + 1e-6, name

"""The NeRF MLP's parameter layout and its fold into the packed weights of the tensor-core forward
(zipnerf_b200/nerf_mlp.py), on the CPU: the layout of `nerf_mlp_parameters` for the reference model's defaults
(nerf_mlp.cu:440-455 with Model.py:66-77,96-105), the He-uniform initialization over the fan-in columns, the packed
network's equality with the unfolded reference network in float64, and the packed weights' shapes and zero padding as
the kernel reads them (`PackedMlp` of csrc/fz_nerf_mlp.cu). Also that the kernel source compiles for sm_100a without
spills."""
from __future__ import annotations

import math
import re
import shutil
import subprocess
from pathlib import Path

import pytest
import torch

from zipnerf_b200 import nerf_mlp as nm

REPO = Path(__file__).resolve().parent.parent


def test_parameter_layout_of_the_reference_model():
    layout = nm.NerfMlpLayout()
    shapes = {name: (tuple(shape), fan_in) for name, shape, fan_in in layout.parameters}
    assert [name for name, _, _ in layout.parameters] == [
        'density_0.weight', 'density_0.bias', 'density_1.weight', 'density_1.bias', 'bottleneck.weight', 'bottleneck.bias',
        'view_0.weight', 'view_0.bias', 'view_1.weight', 'view_1.bias', 'view_2.weight', 'view_2.bias', 'rgb.weight', 'rgb.bias']
    assert shapes['density_0.weight'] == ((64, 56), 50)  # 50 features padded to 56 columns
    assert shapes['view_0.weight'] == ((256, 288), 283)  # bottleneck 256 + direction block 32 (27 used)
    assert shapes['rgb.weight'] == ((3, 544), 539)  # v2 256 + bottleneck 256 + direction block 32
    assert shapes['density_1.bias'] == ((1,), 0) and shapes['rgb.bias'] == ((3,), 0)
    assert layout.size == 227556 and layout.numel == 227556 and layout.n_inputs == 96 and layout.n_features == 56
    assert nm.direction_block_width(4) == 32 and nm.direction_block_width(0) == 8
    with pytest.raises(RuntimeError, match='ZipNeRF: nerf mlp widths must be multiples of 8'):
        nm.NerfMlpLayout(view_width=100)


def test_initialization_fills_the_fan_in_columns_only():
    layout = nm.NerfMlpLayout()
    params = torch.full((layout.numel,), 7.0)
    layout.initialize(params, torch.Generator().manual_seed(0))
    for name, shape, fan_in in layout.parameters:
        w = layout.view(params, name)
        if fan_in == 0:
            assert not w.any(), name
            continue
        bound = math.sqrt(6.0 / fan_in)
        assert w[:, :fan_in].abs().max() <= bound and w[:, :fan_in].abs().max() > 0.9 * bound, name
        assert not w[:, fan_in:].any(), name  # padding columns never hold values


def random_model(seed: int, dtype=torch.float64):
    layout = nm.NerfMlpLayout()
    g = torch.Generator().manual_seed(seed)
    params = torch.zeros(layout.numel, dtype=torch.float32)
    layout.initialize(params, g)
    for name, _, fan_in in layout.parameters:  # nonzero biases so that every bias fold matters
        if fan_in == 0:
            layout.view(params, name).uniform_(-0.3, 0.3, generator=g)
    return layout, params.to(dtype), g


def inputs(layout, n: int, g: torch.Generator, dtype=torch.float64):
    features = torch.zeros(n, layout.n_features, dtype=dtype)
    features[:, :50] = torch.randn(n, 50, generator=g, dtype=dtype)
    block = torch.zeros(n, 32, dtype=dtype)
    block[:, :layout.n_direction] = torch.rand(n, layout.n_direction, generator=g, dtype=dtype) * 2 - 1
    block[:, 31] = 1.0  # the bias lane
    return features, block


def test_folded_network_equals_the_reference_network():
    layout, params, g = random_model(1)
    features, block = inputs(layout, 257, g)
    expected = nm.unfolded_forward(layout, params, features, block)
    folded = nm.folded_forward(nm.fold(layout, params), features, block)
    assert expected.shape == folded.shape == (257, 8)
    assert not expected[:, 4:].any() and not folded[:, 4:].any()
    torch.testing.assert_close(folded, expected, rtol=1e-10, atol=1e-10)
    # and so are the gradients: autograd of the fold is the unfold of the packed weights' gradients
    grad_out = torch.randn(257, 8, generator=g, dtype=torch.float64)
    p1, p2 = params.clone().requires_grad_(), params.clone().requires_grad_()
    (nm.unfolded_forward(layout, p1, features, block) * grad_out).sum().backward()
    (nm.folded_forward(nm.fold(layout, p2), features, block) * grad_out).sum().backward()
    torch.testing.assert_close(p2.grad, p1.grad, rtol=1e-10, atol=1e-10)
    # the bias lane carries the folded biases: without it the outputs change
    no_lane = block.clone()
    no_lane[:, 31] = 0.0
    assert not torch.allclose(nm.folded_forward(nm.fold(layout, params), features, no_lane), expected)


def test_packed_weights_have_the_kernel_shapes_and_padding():
    layout, params, g = random_model(2, torch.float32)
    stored = nm.pack(layout, params)
    # the weights are stored in the tensor cores' order; row_major undoes it, and the values are the fold's in bf16
    packed = {k: (v if k.endswith('_bias') else nm.row_major(v, nm.K_SLICE[k])) for k, v in stored.items()}
    folded = nm.fold(layout, params)
    for k, v in packed.items():
        assert torch.equal(v, folded[k].to(torch.bfloat16).float() if k.endswith('_bias') else folded[k].to(torch.bfloat16)), k
    shapes = {'density': (64, 64), 'density_bias': (64,), 'combined': (256, 96), 'skip': (16, 96), 'view_1': (256, 256),
              'view_1_bias': (256,), 'view_2': (256, 256), 'view_2_bias': (256,), 'rgb': (16, 256)}
    assert {k: tuple(v.shape) for k, v in packed.items()} == shapes
    for name, t in stored.items():
        assert t.is_contiguous() and t.dtype == (torch.float32 if name.endswith('_bias') else torch.bfloat16), name
    assert not packed['density'][:, 50:].any()  # 6 padding feature columns + 8 columns of the MMA K step
    assert not packed['combined'][:, 91:95].any()  # direction padding between the 27 encoded values and the bias lane
    assert not packed['skip'][4:].any() and not packed['skip'][:, 91:95].any() and not packed['skip'][0, 64:95].any()
    assert not packed['rgb'][0].any() and not packed['rgb'][4:].any()
    # bf16 operands: the packed network stays within bf16 rounding of the reference network
    features, block = inputs(layout, 512, g, torch.float32)
    expected = nm.unfolded_forward(layout, params, features, block)
    bf16 = {k: v.float() for k, v in packed.items()}
    actual = nm.folded_forward(bf16, features.bfloat16().float(), block)
    err = ((actual - expected).norm() / expected.norm()).item()
    assert err < 1e-2, err  # about 3e-3


@pytest.mark.skipif(shutil.which('nvcc') is None, reason='nvcc is not on PATH')
@pytest.mark.parametrize('source', ['fz_nerf_mlp.cu', 'fz_nerf_mlp_backward.cu'])
def test_tensor_core_kernels_compile_for_sm100a(tmp_path, source):
    run = subprocess.run(['nvcc', '-gencode', 'arch=compute_100a,code=sm_100a', '-O3', '--use_fast_math', '-std=c++17', '-Xptxas', '-v', '-c',
                          '-I', str(REPO / 'include'), str(REPO / 'fused-zipnerf_b200' / 'csrc' / source), '-o', str(tmp_path / 'kernel.o')],
                         capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stderr[-2000:]
    spills = re.findall(r'(\d+) bytes spill stores, (\d+) bytes spill loads', run.stderr)
    assert spills and all(s == ('0', '0') for s in spills), run.stderr


def _relu_backward_double(grad: torch.Tensor, activation: torch.Tensor, bias_grad: torch.Tensor) -> None:
    """The contract of relu_backward_ (zf_mlp.h) in torch: grad *= (activation > 0); bias_grad += the fp32 column sums
    of the masked gradient when bias_grad is not empty. The kernel itself is checked against torch on the GPU."""
    grad.copy_(torch.where(activation > 0, grad, torch.zeros_like(grad)))
    if bias_grad.numel():
        bias_grad += grad.float().sum(0)


def test_reference_interface_forward_and_backward_match_autograd():
    """NerfMlp's layer chain (`_forward`, `_backward`) on CPU tensors against autograd of the fold and the folded
    chain with the same bf16 roundings (weights, activations), and against the unfolded reference network in fp32."""
    layout, params32, g = random_model(3, torch.float32)
    mlp = nm.NerfMlp(50, 64, 256, 256, 4)
    n = 320
    features32, block = inputs(layout, n, g, torch.float32)
    features = features32.bfloat16()
    net_inputs = torch.zeros(n, mlp.n_inputs, dtype=torch.bfloat16)
    net_inputs[:, 64:] = block.bfloat16()
    packed = mlp._pack(params32)
    assert packed.dtype == torch.bfloat16 and packed.numel() == mlp.packed_size
    outputs, context = mlp._forward(features, net_inputs, packed, True)
    assert outputs.shape == (n, 8) and len(context) == 4 and not outputs[:, 4:].any()
    assert mlp._forward(features, net_inputs.clone(), packed, False)[1] == []
    grad_outputs = torch.randn(n, 8, generator=g).bfloat16()
    grad_outputs[:, 4:] = 0
    grad_params = torch.full_like(params32, 0.25)  # accumulates (+=)
    grad_features = mlp._backward(grad_outputs, features, packed, context, params32, grad_params, _relu_backward_double)
    grad_params -= 0.25

    def stored(t):  # bf16 rounding that passes the gradient straight through
        return t + (t.bfloat16().float() - t).detach()

    p = params32.clone().requires_grad_()
    x = features.float().requires_grad_()
    w = {k: stored(v) for k, v in nm.fold(layout, p, 56, 8).items()}
    h = stored(torch.relu(x @ w['density'].t() + w['density_bias']))
    net_in = torch.cat([h, block.bfloat16().float()], dim=1)
    v0 = stored(torch.relu(net_in @ w['combined'].t()))
    v1 = stored(torch.relu(v0 @ w['view_1'].t() + w['view_1_bias']))
    v2 = stored(torch.relu(v1 @ w['view_2'].t() + w['view_2_bias']))
    expected = net_in @ w['skip'].t() + v2 @ w['rgb'].t()
    torch.testing.assert_close(outputs.float(), expected, rtol=2e-2, atol=2e-2 * expected.abs().mean().item())
    (expected * grad_outputs.float()).sum().backward()

    def rel(a, b):
        return ((a.float() - b).norm() / b.norm()).item()

    errors = {name: rel(layout.view(grad_params, name), layout.view(p.grad, name)) for name, _, fan_in in layout.parameters}
    errors['features'] = rel(grad_features, x.grad)
    assert max(errors.values()) < 1e-2, errors
    for name, _, fan_in in layout.parameters:  # padding columns of the parameters receive no gradient
        if name in ('view_0.weight', 'rgb.weight'):
            assert not layout.view(grad_params, name)[:, fan_in:].any(), name
    # the same parameters in the unfolded reference network, fp32 throughout
    q = params32.clone().requires_grad_()
    reference = nm.unfolded_forward(layout, q, features.float(), block)
    (reference * grad_outputs.float()).sum().backward()
    # bf16 weights and activations move this chain's parameter gradients by 4-8 % from fp32 (the fold itself is exact,
    # test_folded_network_equals_the_reference_network); outputs by 3e-3
    assert rel(grad_params, q.grad) < 0.1 and rel(outputs, reference) < 1e-2


def test_reference_interface_checks_its_arguments():
    mlp = nm.NerfMlp(50, 64, 256, 256, 4)
    assert (mlp.n_features, mlp.n_inputs) == (56, 96)
    with pytest.raises(RuntimeError, match='ZipNeRF: params must be a contiguous cuda tensor of the expected type'):
        mlp.pack(torch.zeros(mlp.layout.numel))  # a CPU tensor: the product path is CUDA only
    with pytest.raises(RuntimeError, match='ZipNeRF: invalid nerf mlp parameters'):
        mlp._pack(torch.zeros(100))
    with pytest.raises(RuntimeError, match='ZipNeRF: invalid nerf mlp inputs'):
        mlp._forward(torch.zeros(4, 50, dtype=torch.bfloat16), torch.zeros(4, 96, dtype=torch.bfloat16), torch.zeros(mlp.packed_size, dtype=torch.bfloat16), True)
    with pytest.raises(RuntimeError, match='ZipNeRF: invalid nerf mlp backward inputs'):
        mlp._backward(None, None, torch.zeros(mlp.packed_size, dtype=torch.bfloat16), [], None, None, _relu_backward_double)
    with pytest.raises(RuntimeError, match='ZipNeRF: nerf mlp widths must be multiples of 8'):
        nm.NerfMlp(50, 60, 256, 256, 4)


def canonical_offset(row: int, k: int, k_total: int) -> int:
    """csrc/fz_nerf_mlp.cu canonical_offset: the byte offset of element (row, k) of a K-major operand."""
    return ((row >> 3) * (k_total >> 3) + (k >> 3)) * 128 + (row & 7) * 16 + (k & 7) * 2


def mma_operand(image, start: int, leading: int, stride: int, rows: int):
    """The [rows x 16] operand one kind::f16 MMA reads through a no-swizzle K-major descriptor: the canonical layout
    ((8, rows / 8), (8, 2)) : ((16 B, stride), (2 B, leading)) of the tcgen05 shared-memory descriptor."""
    import numpy as np
    out = np.empty((rows, 16), dtype=image.dtype)
    for r in range(rows):
        for k in range(16):
            address = start + 16 * (r % 8) + stride * (r // 8) + 2 * (k % 8) + leading * (k // 8)
            out[r, k] = image[address // 2]
    return out


@pytest.mark.parametrize('n,k', [(64, 64), (256, 96), (128, 96), (16, 96), (256, 256), (128, 256), (16, 256)])
def test_tensor_core_operand_layout_is_consistent(n, k):
    """The kernel's staging (canonical_offset) and its MMA descriptors (start + 256 B per K step, leading offset 128 B,
    stride offset k / 8 * 128 B) address the same elements: emulating the operand reads of the documented canonical
    layout over all K steps reproduces A @ B^T for each layer shape of the kernel."""
    import numpy as np
    rng = np.random.default_rng(n + k)
    a, b = rng.integers(-8, 8, size=(128, k)).astype(np.float64), rng.integers(-8, 8, size=(n, k)).astype(np.float64)
    a_image, b_image = np.zeros(128 * k), np.zeros(n * k)
    for r in range(128):
        for c in range(k):
            a_image[canonical_offset(r, c, k) // 2] = a[r, c]
    for r in range(n):
        for c in range(k):
            b_image[canonical_offset(r, c, k) // 2] = b[r, c]
    d = np.zeros((128, n))
    for s in range(k // 16):
        step = 2 * s * 128
        d += mma_operand(a_image, step, 128, k // 8 * 128, 128) @ mma_operand(b_image, step, 128, k // 8 * 128, n).T
    np.testing.assert_array_equal(d, a @ b.T)


def _cutlass_include():
    import importlib.util
    spec = importlib.util.find_spec('flashinfer')
    if spec is None or spec.origin is None:
        return None
    path = Path(spec.origin).parent / 'data' / 'cutlass' / 'include'
    return path if (path / 'cute' / 'arch' / 'mma_sm100_desc.hpp').exists() else None


DESCRIPTOR_CHECK = r'''
#include <cstdio>
#include <cute/arch/mma_sm100_desc.hpp>
#include <cute/numeric/numeric_types.hpp>
#include "fz_nerf_mlp.cu"
namespace zf {  // the library's error recording, not linked into this check
int set_error(int code, const std::string&) { return code; }
int set_cuda_error(cudaError_t, const char*) { return 3; }
}
template <int N> int check_instr() {
    const uint32_t theirs = uint32_t(cute::UMMA::make_instr_desc<cute::bfloat16_t, cute::bfloat16_t, float, 128, N, cute::UMMA::Major::K, cute::UMMA::Major::K>());
    const uint32_t ours = zf::nerf_mlp::instr_descriptor(128, N);
    if (theirs != ours) std::printf("instr N=%d: cute %08x ours %08x\n", N, theirs, ours);
    return theirs != ours;
}
int main() {
    int bad = check_instr<16>() + check_instr<64>() + check_instr<128>() + check_instr<256>();
    for (uint32_t address : {0u, 0x4000u, 0x1a300u, 0x36000u}) {
        for (uint32_t k : {64u, 96u, 256u}) {
            cute::UMMA::SmemDescriptor d;
            d.version_ = 1; d.lbo_mode_ = 0; d.layout_type_ = uint8_t(cute::UMMA::LayoutType::SWIZZLE_NONE); d.base_offset_ = 0;
            d.start_address_ = uint16_t(address >> 4); d.leading_byte_offset_ = 128 >> 4; d.stride_byte_offset_ = uint16_t(k / 8 * 128 >> 4);
            const uint64_t ours = zf::nerf_mlp::smem_descriptor(address, 128, k / 8 * 128);
            if (uint64_t(d) != ours) { std::printf("smem %x k=%u: cute %llx ours %llx\n", address, k, (unsigned long long)uint64_t(d), (unsigned long long)ours); bad++; }
        }
    }
    std::printf("%d mismatches\n", bad);
    return bad;
}
'''


@pytest.mark.skipif(shutil.which('nvcc') is None or _cutlass_include() is None, reason='nvcc or the CUTLASS headers are absent')
def test_tensor_core_descriptors_match_cutlass(tmp_path):
    """The kernel's instruction descriptors (bf16 x bf16 -> fp32, M = 128, N = 16 / 64 / 128 / 256, K-major) and its
    no-swizzle shared-memory descriptors equal the ones CUTLASS's CuTe sm100 code builds (cute/arch/mma_sm100_desc.hpp:
    make_instr_desc, SmemDescriptor with version 1 as make_umma_desc sets it)."""
    source = tmp_path / 'check.cu'
    source.write_text(DESCRIPTOR_CHECK)
    binary = tmp_path / 'check'
    build = subprocess.run(['nvcc', '-std=c++17', '-gencode', 'arch=compute_100a,code=sm_100a', '-I', str(_cutlass_include()),
                            '-I', str(REPO / 'fused-zipnerf_b200' / 'csrc'), '-I', str(REPO / 'include'), str(source), '-o', str(binary)],
                           capture_output=True, text=True, timeout=300)
    assert build.returncode == 0, build.stderr[-3000:]
    run = subprocess.run([str(binary)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and '0 mismatches' in run.stdout, run.stdout


MN_DESCRIPTOR_CHECK = r"""
#include <cstdio>
#include <cute/tensor.hpp>
#include <cute/atom/mma_traits_sm100.hpp>
#include "fz_tcgen05.cuh"
using namespace cute;
// the backward's weight-gradient tiles: a [rows (K) x width (MN)] bf16 tile in the canonical order, element (k, m) at
// ((k / 8) (width / 8) + m / 8) 64 + (k % 8) 8 + m % 8, read as an MN-major operand
template <int Width, int Rows> int check_mn() {
    auto layout = make_layout(make_shape(make_shape(Int<8>{}, Int<Width / 8>{}), make_shape(Int<8>{}, Int<Rows / 8>{})),
                              make_stride(make_stride(Int<1>{}, Int<64>{}), make_stride(Int<8>{}, Int<Width / 8 * 64>{})));
    auto tensor = make_tensor(make_smem_ptr(reinterpret_cast<bfloat16_t*>(uintptr_t(0))), layout);
    const uint64_t theirs = uint64_t(UMMA::make_umma_desc<UMMA::Major::MN>(tensor)) & ~uint64_t(0x3FFF);  // start address: device only
    const uint64_t ours = zf::nerf_mlp::smem_descriptor(0, Width / 8 * 128, 128);
    if (theirs != ours) std::printf("MN width %d: cute %llx ours %llx\n", Width, (unsigned long long)theirs, (unsigned long long)ours);
    return theirs != ours;
}
template <int N> int check_instr_mn() {
    const uint32_t theirs = uint32_t(UMMA::make_instr_desc<bfloat16_t, bfloat16_t, float, 128, N, UMMA::Major::MN, UMMA::Major::MN>());
    const uint32_t ours = zf::nerf_mlp::instr_descriptor(128, N, true, true);
    if (theirs != ours) std::printf("instr MN N=%d: cute %08x ours %08x\n", N, theirs, ours);
    return theirs != ours;
}
// the TMA-written weight-gradient tiles: K-major tiling of CuTe's MN-major swizzle atoms (8-row K groups adjacent)
template <class Atom, int Width, int Rows> uint64_t cute_swizzled() {
    auto layout = tile_to_shape(Atom{}, make_shape(Int<Width>{}, Int<Rows>{}), Step<_2, _1>{});
    auto tensor = make_tensor(make_smem_ptr(reinterpret_cast<bfloat16_t*>(uintptr_t(0))), layout);
    return uint64_t(UMMA::make_umma_desc<UMMA::Major::MN>(tensor)) & ~uint64_t(0x3FFF);
}
template <int Width, int Rows> int check_sw128() {
    const uint64_t theirs = cute_swizzled<UMMA::Layout_MN_SW128_Atom<bfloat16_t>, Width, Rows>();
    const uint64_t ours = zf::nerf_mlp::mn_sw128_descriptor(0, Rows);
    if (theirs != ours) std::printf("SW128 width %d rows %d: cute %llx ours %llx\n", Width, Rows, (unsigned long long)theirs, (unsigned long long)ours);
    return theirs != ours;
}
int check_sw32() {
    const uint64_t theirs = cute_swizzled<UMMA::Layout_MN_SW32_Atom<bfloat16_t>, 16, 32>();
    const uint64_t ours = zf::nerf_mlp::mn_sw32_descriptor(0);
    if (theirs != ours) std::printf("SW32: cute %llx ours %llx\n", (unsigned long long)theirs, (unsigned long long)ours);
    return theirs != ours;
}
int main() {
    int bad = check_mn<256, 64>() + check_mn<128, 64>() + check_mn<16, 64>() + check_mn<96, 64>() + check_mn<64, 64>();
    bad += check_sw128<256, 32>() + check_sw128<128, 32>() + check_sw32();
    bad += check_instr_mn<16>() + check_instr_mn<64>() + check_instr_mn<96>() + check_instr_mn<256>();
    std::printf("%d mismatches\n", bad);
    return bad;
}
"""


@pytest.mark.skipif(shutil.which('nvcc') is None or _cutlass_include() is None, reason='nvcc or the CUTLASS headers are absent')
def test_weight_gradient_descriptors_match_cutlass(tmp_path):
    """The backward's weight-gradient GEMMs read their operands MN-major (the samples are K): the shared-memory
    descriptors of canonical tiles (leading byte offset = the K-atom stride, stride byte offset = 128), of the
    TMA-written tiles with the 128-byte swizzle (leading offset = the 64-column atom stride, stride offset = 1024)
    and the 32-byte swizzle, and the MN-major instruction descriptors equal the ones CuTe builds for the same layouts
    (make_umma_desc<Major::MN>, make_instr_desc with Major::MN)."""
    source = tmp_path / 'check_mn.cu'
    source.write_text(MN_DESCRIPTOR_CHECK)
    binary = tmp_path / 'check_mn'
    build = subprocess.run(['nvcc', '-std=c++17', '-gencode', 'arch=compute_100a,code=sm_100a', '-I', str(_cutlass_include()),
                            '-I', str(REPO / 'fused-zipnerf_b200' / 'csrc'), '-I', str(REPO / 'include'), str(source), '-o', str(binary)],
                           capture_output=True, text=True, timeout=300)
    assert build.returncode == 0, build.stderr[-3000:]
    run = subprocess.run([str(binary)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and '0 mismatches' in run.stdout, run.stdout


@pytest.mark.parametrize('rows,k,k_slice', [(64, 64, 64), (256, 96, 64), (16, 96, 96), (256, 256, 64), (16, 256, 256)])
def test_packed_order_is_the_kernels_sliced_canonical_layout(rows, k, k_slice):
    """Element (r, c) of a packed weight sits in K-slice s = c // k_slice at the slice's start plus the kernel's
    canonical_offset(r, c - s k_slice, width) / 2, where each slice is rows x width elements; so a single bulk copy
    lands a slice where the MMA descriptors read it. row_major inverts the order."""
    order = nm.sliced_order(rows, k, k_slice)
    assert sorted(order.tolist()) == list(range(rows * k))
    position = torch.empty(rows * k, dtype=torch.long)
    position[order] = torch.arange(rows * k)
    for r in range(rows):
        for c in range(0, k, 3):
            s = c // k_slice
            width = min(k_slice, k - s * k_slice)
            assert position[r * k + c].item() == rows * s * k_slice + canonical_offset(r, c - s * k_slice, width) // 2
    w = torch.randn(rows, k).bfloat16()
    assert torch.equal(nm.row_major(w.reshape(-1)[order].view(rows, k), k_slice), w)


def test_tensor_core_forward_wrapper_rejects_mismatched_tensors():
    """The C ABI of the tensor-core forward sees only pointers and row strides, so the wrapper checks shapes, dtypes and
    layouts first: every mismatch below raises ValueError before anything reaches the device."""
    from zipnerf_b200 import capi
    layout = nm.NerfMlpLayout()
    params = torch.zeros(layout.numel)
    layout.initialize(params, torch.Generator().manual_seed(1))
    packed = nm.pack(layout, params)
    n = 40

    def good():
        return {'features': torch.zeros(n, 56, dtype=torch.bfloat16), 'inputs': torch.zeros(n, 96, dtype=torch.bfloat16),
                'packed': dict(packed), 'outputs': torch.zeros(n, 8, dtype=torch.bfloat16), 'status': torch.zeros(1, dtype=torch.int32)}

    def call(a, require_cuda=False):
        capi.check_nerf_mlp_forward_tc(a['features'], a['inputs'], a['packed'], a['outputs'], a['status'], require_cuda=require_cuda)

    call(good())  # the shapes nerf_mlp.pack and the kernel agree on
    with pytest.raises(ValueError):
        call(good(), require_cuda=True)  # host tensors
    bad = []
    for key, value in [('features', torch.zeros(n, 48, dtype=torch.bfloat16)), ('features', torch.zeros(n, 56)),
                       ('inputs', torch.zeros(n, 64, dtype=torch.bfloat16)), ('inputs', torch.zeros(n + 1, 96, dtype=torch.bfloat16)),
                       ('outputs', torch.zeros(n, 4, dtype=torch.bfloat16)), ('outputs', torch.zeros(n - 1, 8, dtype=torch.bfloat16)),
                       ('outputs', torch.zeros(8, n, dtype=torch.bfloat16).t()), ('outputs', torch.zeros(n, 8)),
                       ('features', torch.zeros(56, n, dtype=torch.bfloat16).t()), ('status', torch.zeros(1, dtype=torch.int64))]:
        a = good()
        a[key] = value
        bad.append(a)
    for name in packed:
        for wrong in (packed[name][:-1].clone() if packed[name].dim() == 1 else packed[name][:-1].clone(), packed[name].double()):
            a = good()
            a['packed'] = dict(packed) | {name: wrong}
            bad.append(a)
    a = good()
    del a['packed']['rgb']
    bad.append(a)
    for a in bad:
        with pytest.raises(ValueError):
            call(a)

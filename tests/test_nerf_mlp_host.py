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
    # the bias lane carries the folded biases: without it the outputs change
    no_lane = block.clone()
    no_lane[:, 31] = 0.0
    assert not torch.allclose(nm.folded_forward(nm.fold(layout, params), features, no_lane), expected)


def test_packed_weights_have_the_kernel_shapes_and_padding():
    layout, params, g = random_model(2, torch.float32)
    packed = nm.pack(layout, params)
    shapes = {'density': (64, 64), 'density_bias': (64,), 'combined': (256, 96), 'skip': (16, 96), 'view_1': (256, 256),
              'view_1_bias': (256,), 'view_2': (256, 256), 'view_2_bias': (256,), 'rgb': (16, 256)}
    assert {k: tuple(v.shape) for k, v in packed.items()} == shapes
    for name, t in packed.items():
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
def test_tensor_core_forward_compiles_for_sm100a(tmp_path):
    run = subprocess.run(['nvcc', '-gencode', 'arch=compute_100a,code=sm_100a', '-O3', '--use_fast_math', '-std=c++17', '-Xptxas', '-v', '-c',
                          str(REPO / 'fused-zipnerf_b200' / 'csrc' / 'fz_nerf_mlp.cu'), '-o', str(tmp_path / 'fz_nerf_mlp.o')],
                         capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stderr[-2000:]
    spills = re.findall(r'(\d+) bytes spill stores, (\d+) bytes spill loads', run.stderr)
    assert spills and all(s == ('0', '0') for s in spills), run.stderr

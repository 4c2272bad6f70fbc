"""The NeRF MLP's fp32 parameter layout and its fold into the packed weights of the tensor-core forward
(csrc/fz_nerf_mlp.cu, `PackedMlp`), restated from the reference: the layout of `nerf_mlp_parameters`
(B/mlp/src/nerf_mlp.cu:440-455, the buffer Model.py:96-105 builds from it) and the fold of `pack_kernel`
(nerf_mlp.cu:186-234).

The reference network (unfolded, `unfolded_forward`):
    h = relu(features @ density_0^T + b)               density = h @ density_1^T + b
    bottleneck = h @ bottleneck^T + b                   (no activation)
    v0 = relu([bottleneck | direction] @ view_0^T + b)  v1, v2 = relu(... view_1 / view_2 ...)
    rgb = [v2 | bottleneck | direction] @ rgb^T + b
Because the bottleneck only feeds linear maps, the fold multiplies it into the first view layer and the rgb layer's
skip columns, and moves every bias of a layer that reads the inputs [h | direction block] into the block's last
column (the bias lane, 1.0): the packed network (`folded_forward`) has one GEMM fewer and no bottleneck activation.
The direction block holds 3 + 6 * degree encoded values, zero padding and the bias lane, padded to a multiple of 8.
"""
from __future__ import annotations

import math

import torch


# multiply-adds per sample of the packed network at the reference model's widths: density 64 x 56, combined 256 x 96,
# skip 8 x 96, view_1 and view_2 256 x 256, rgb 8 x 256
MACS_PER_SAMPLE = 64 * 56 + 256 * 96 + 8 * 96 + 2 * 256 * 256 + 8 * 256


def direction_block_width(degree: int) -> int:
    """zipnerf_config.h:18: identity, sines and cosines of 3 axes and `degree` octaves, a bias lane, padded to 8."""
    return (3 + 6 * degree + 1 + 7) // 8 * 8


def nerf_mlp_parameters(n_features: int, density_width: int, bottleneck_width: int, view_width: int, direction_degree: int):
    """(name, shape, fan-in) of every tensor of the flat fp32 parameter buffer in layout order, fan-in 0 for biases;
    input columns padded to multiples of 8, the padding columns last (nerf_mlp.cu:440-455)."""
    n_direction = 3 + 6 * direction_degree
    n_view_inputs = bottleneck_width + direction_block_width(direction_degree)
    return [
        ('density_0.weight', [density_width, (n_features + 7) // 8 * 8], n_features), ('density_0.bias', [density_width], 0),
        ('density_1.weight', [1, density_width], density_width), ('density_1.bias', [1], 0),
        ('bottleneck.weight', [bottleneck_width, density_width], density_width), ('bottleneck.bias', [bottleneck_width], 0),
        ('view_0.weight', [view_width, n_view_inputs], bottleneck_width + n_direction), ('view_0.bias', [view_width], 0),
        ('view_1.weight', [view_width, view_width], view_width), ('view_1.bias', [view_width], 0),
        ('view_2.weight', [view_width, view_width], view_width), ('view_2.bias', [view_width], 0),
        ('rgb.weight', [3, view_width + n_view_inputs], view_width + bottleneck_width + n_direction), ('rgb.bias', [3], 0),
    ]


class NerfMlpLayout:
    """Views of the flat parameter buffer (tensors back to back in `nerf_mlp_parameters` order; the buffer is padded to
    a multiple of 4 for the vectorized optimizer, Model.py:105). The defaults are the reference model's: 50 NeRF grid
    features (10 levels x (4 + 1)), padded to 56 columns; widths 64 / 256 / 256; direction degree 4 (Model.py:66-77)."""

    def __init__(self, n_features: int = 50, density_width: int = 64, bottleneck_width: int = 256, view_width: int = 256,
                 direction_degree: int = 4) -> None:
        if density_width % 8 or bottleneck_width % 8 or view_width % 8:
            raise RuntimeError('ZipNeRF: nerf mlp widths must be multiples of 8')  # nerf_mlp.cu:458
        self.parameters = nerf_mlp_parameters(n_features, density_width, bottleneck_width, view_width, direction_degree)
        self.density_width, self.bottleneck_width, self.view_width = density_width, bottleneck_width, view_width
        self.n_features = self.parameters[0][1][1]
        self.n_direction = 3 + 6 * direction_degree
        self.n_inputs = density_width + direction_block_width(direction_degree)
        self.offsets, n = {}, 0
        for name, shape, _ in self.parameters:
            self.offsets[name] = (n, tuple(shape))
            n += math.prod(shape)
        self.size = n
        self.numel = (n + 3) // 4 * 4

    def view(self, buffer: torch.Tensor, name: str) -> torch.Tensor:
        offset, shape = self.offsets[name]
        return buffer[offset:offset + math.prod(shape)].view(shape)

    def initialize(self, buffer: torch.Tensor, generator: torch.Generator) -> None:
        """He-uniform over the first fan-in columns of each weight; the padding columns (last) and biases stay zero
        (Model.py:59-62,110-113)."""
        buffer.zero_()
        for name, _, fan_in in self.parameters:
            if fan_in > 0:
                bound = math.sqrt(6.0 / fan_in)
                self.view(buffer, name)[:, :fan_in].uniform_(-bound, bound, generator=generator)


def unfolded_forward(layout: NerfMlpLayout, params: torch.Tensor, features: torch.Tensor, direction_block: torch.Tensor) -> torch.Tensor:
    """The reference network on its fp32 parameters: [n, 8] outputs (raw density, 3 rgb logits, 4 zeros). Only the
    encoded values of the direction block are inputs: its padding and bias-lane columns meet the weights' padding
    columns, which hold zeros and receive no gradient (nerf_mlp.cu:442)."""
    p = {name: layout.view(params, name) for name, _, _ in layout.parameters}
    direction_block = torch.nn.functional.pad(direction_block[:, :layout.n_direction], (0, direction_block.shape[1] - layout.n_direction))
    h = torch.relu(features @ p['density_0.weight'].t() + p['density_0.bias'])
    density = h @ p['density_1.weight'].t() + p['density_1.bias']
    bottleneck = h @ p['bottleneck.weight'].t() + p['bottleneck.bias']
    view_inputs = torch.cat([bottleneck, direction_block], dim=1)
    v0 = torch.relu(view_inputs @ p['view_0.weight'].t() + p['view_0.bias'])
    v1 = torch.relu(v0 @ p['view_1.weight'].t() + p['view_1.bias'])
    v2 = torch.relu(v1 @ p['view_2.weight'].t() + p['view_2.bias'])
    rgb = torch.cat([v2, view_inputs], dim=1) @ p['rgb.weight'].t() + p['rgb.bias']
    return torch.cat([density, rgb, torch.zeros_like(rgb[:, :1]).expand(-1, 4)], dim=1)


def fold(layout: NerfMlpLayout, params: torch.Tensor, k_features: int = 64, out_rows: int = 16) -> dict:
    """The packed network in the parameters' dtype, by default in the tensor-core kernel's shapes (`PackedMlp`):
    density [density_width, k_features] (features zero padded to the MMA K step), combined [view_width, n_inputs], skip
    [out_rows, n_inputs], view_1 / view_2, rgb [out_rows, view_width] (out_rows >= 8: the smallest N of an M = 128 MMA
    is 16), and the biases of the density and view layers. Differentiable: autograd of the fold is the unfold of the
    packed weights' gradients into the parameters' (nerf_mlp.cu:236-284)."""
    p = {name: layout.view(params, name) for name, _, _ in layout.parameters}
    dw, bw, vw, nd, ni = layout.density_width, layout.bottleneck_width, layout.view_width, layout.n_direction, layout.n_inputs
    bias_lane = ni - 1
    density = params.new_zeros(dw, k_features)
    density[:, :layout.n_features] = p['density_0.weight']
    view_0 = p['view_0.weight']
    combined = params.new_zeros(vw, ni)
    combined[:, :dw] = view_0[:, :bw] @ p['bottleneck.weight']
    combined[:, dw:dw + nd] = view_0[:, bw:bw + nd]
    combined[:, bias_lane] = view_0[:, :bw] @ p['bottleneck.bias'] + p['view_0.bias']
    rgb_w = p['rgb.weight']
    skip = params.new_zeros(out_rows, ni)
    skip[0, :dw] = p['density_1.weight'][0]
    skip[0, bias_lane] = p['density_1.bias'][0]
    skip[1:4, :dw] = rgb_w[:, vw:vw + bw] @ p['bottleneck.weight']
    skip[1:4, dw:dw + nd] = rgb_w[:, vw + bw:vw + bw + nd]
    skip[1:4, bias_lane] = rgb_w[:, vw:vw + bw] @ p['bottleneck.bias'] + p['rgb.bias']
    rgb = params.new_zeros(out_rows, vw)
    rgb[1:4] = rgb_w[:, :vw]
    return {'density': density, 'density_bias': p['density_0.bias'].clone(), 'combined': combined, 'skip': skip,
            'view_1': p['view_1.weight'].clone(), 'view_1_bias': p['view_1.bias'].clone(), 'view_2': p['view_2.weight'].clone(),
            'view_2_bias': p['view_2.bias'].clone(), 'rgb': rgb}


def canonical_order(rows: int, k: int) -> torch.Tensor:
    """Row-major element indices of a [rows x k] operand in the tensor cores' no-swizzle K-major layout: 8-row x 8-column
    core matrices (128 bytes of bf16) stored contiguously, K-adjacent core matrices next, then the next 8 rows; the same
    order as the kernel's canonical_offset (csrc/fz_nerf_mlp.cu), so one bulk copy lands a weight ready for the MMAs."""
    r = torch.arange(rows).view(rows // 8, 1, 8, 1)
    c = torch.arange(k).view(1, k // 8, 1, 8)
    return (r * k + c).expand(rows // 8, k // 8, 8, 8).reshape(-1)


# K-slice width of each packed weight: the tensor-core kernel streams a layer's weights as consecutive slices of this
# many input columns (all output rows each), and every slice is one contiguous block in the canonical order
K_SLICE = {'density': 64, 'combined': 64, 'skip': 96, 'view_1': 64, 'view_2': 64, 'rgb': 256}


def sliced_order(rows: int, k: int, k_slice: int) -> torch.Tensor:
    """Row-major element indices of a [rows x k] weight stored as consecutive K-slices of k_slice columns (the last one
    narrower when k_slice does not divide k), each slice a [rows x width] block in `canonical_order`."""
    parts = []
    for c0 in range(0, k, k_slice):
        width = min(k_slice, k - c0)
        local = canonical_order(rows, width)
        parts.append(local // width * k + c0 + local % width)
    return torch.cat(parts)


def row_major(weight: torch.Tensor, k_slice: int | None = None) -> torch.Tensor:
    """The row-major [rows x k] matrix of a weight stored in `sliced_order` (k_slice columns per slice; one slice by
    default), the inverse permutation."""
    rows, k = weight.shape
    out = torch.empty_like(weight).reshape(-1)
    out[sliced_order(rows, k, k_slice or k).to(weight.device)] = weight.reshape(-1)
    return out.view(rows, k)


_ORDERS: dict = {}


def _device_order(rows: int, k: int, k_slice: int, device) -> torch.Tensor:
    """sliced_order on the device, computed once per shape and device"""
    key = (rows, k, k_slice, str(device))
    if key not in _ORDERS:
        _ORDERS[key] = sliced_order(rows, k, k_slice).to(device)
    return _ORDERS[key]


def pack_folded(folded: dict) -> dict:
    """The folded network (`fold` in the kernel's shapes) as the operands of zf_nerf_mlp_forward_tc: the weights
    rounded to bf16 and stored as the tensor-core kernel streams them (`sliced_order` with the K-slices of K_SLICE),
    the biases rounded to bf16 but stored as fp32 (the reference adds bf16 biases in its fp32 GEMM epilogues,
    nerf_mlp.cu:31,355-363)."""
    out = {}
    for name, t in folded.items():
        if name.endswith('_bias'):
            out[name] = t.to(torch.bfloat16).float().contiguous()
        else:
            order = _device_order(*t.shape, K_SLICE[name], t.device)
            out[name] = t.to(torch.bfloat16).reshape(-1)[order].view(t.shape).contiguous()
    return out


def pack(layout: NerfMlpLayout, params: torch.Tensor) -> dict:
    """`fold` in the kernel's shapes, packed as the operands of zf_nerf_mlp_forward_tc (`pack_folded`)."""
    return pack_folded(fold(layout, params))


# the transposed weights of the backward's data-gradient chain (B operands [inputs x outputs] of dX = dY W), their
# K-slice widths over the outputs, and their stored shapes
K_SLICE_T = {'rgb_t': 16, 'view_2_t': 64, 'view_1_t': 64, 'combined_t': 64, 'skip_t': 16, 'density_t': 64}
TRANSPOSED_OF = {'rgb_t': 'rgb', 'view_2_t': 'view_2', 'view_1_t': 'view_1', 'combined_t': 'combined', 'skip_t': 'skip', 'density_t': 'density'}


def pack_transposed(folded: dict) -> dict:
    """The folded weights transposed ([inputs x outputs]: rgb_t [256, 16], view_2_t / view_1_t [256, 256], combined_t
    [96, 256], skip_t [96, 16], density_t [64, 64]), rounded to bf16 and stored as the backward kernel streams them
    (`sliced_order` with the K-slices of K_SLICE_T): the B operands of zf_nerf_mlp_backward_tc."""
    out = {}
    for name, source in TRANSPOSED_OF.items():
        t = folded[source].t().contiguous()
        order = _device_order(*t.shape, K_SLICE_T[name], t.device)
        out[name] = t.to(torch.bfloat16).reshape(-1)[order].view(t.shape).contiguous()
    return out


def folded_forward(packed: dict, features: torch.Tensor, direction_block: torch.Tensor) -> torch.Tensor:
    """The packed network's layer chain as the kernel runs it (in the packed tensors' dtype, fp32 accumulation when
    they are fp32): [n, 8] outputs. The hidden layer h is the first columns of the inputs [h | direction block]."""
    dtype = packed['density'].dtype
    f = torch.nn.functional.pad(features, (0, packed['density'].shape[1] - features.shape[1])).to(dtype)
    h = torch.relu(f @ packed['density'].t() + packed['density_bias'].to(dtype))
    inputs = torch.cat([h, direction_block.to(dtype)], dim=1)
    v0 = torch.relu(inputs @ packed['combined'].t())
    out = inputs @ packed['skip'].t()
    v1 = torch.relu(v0 @ packed['view_1'].t() + packed['view_1_bias'].to(dtype))
    v2 = torch.relu(v1 @ packed['view_2'].t() + packed['view_2_bias'].to(dtype))
    out = out + v2 @ packed['rgb'].t()
    return out[:, :8]


PACKED_ORDER = ('density', 'density_bias', 'combined', 'skip', 'view_1', 'view_1_bias', 'view_2', 'view_2_bias', 'rgb')
TRANSPOSED_ORDER = tuple(K_SLICE_T)


def _weight_grad(grad: torch.Tensor, activation: torch.Tensor) -> torch.Tensor:
    """grad^T activation of bf16 operands in fp32 (the reference's weight gradients are fp32 GEMM outputs,
    nerf_mlp.cu:581-582)."""
    if grad.is_cuda:
        return torch.mm(grad.t(), activation, out_dtype=torch.float32)
    return grad.t().float() @ activation.float()


class NerfMlp:
    """The reference's `NerfMlp` interface (nerf_mlp.h:47-73: `n_features`, `n_inputs`, `pack`, `forward`,
    `backward`). `pack` returns one flat bf16 tensor (its layout private to this class, as the reference's packed
    buffer is): the folded weights and biases row-major, and, for the reference model's widths, the same fold in the
    tensor-core kernel's order (`pack`, K-sliced canonical bf16 weights and fp32 biases stored bit for bit).

    For the reference model's widths every step runs on this backend's kernels (zf_mlp.h): `pack` is one launch of
    zf_nerf_mlp_pack (the fold in the reference's fp32 order); `forward` the tcgen05 kernel zf_nerf_mlp_forward_tc (one
    persistent kernel for all layers; training keeps v0, v1, v2 and their ReLU masks for the backward); `backward` the
    tcgen05 data-gradient and weight-gradient kernels (zf_nerf_mlp_backward_tc), then the unfold of the packed-weight
    gradients into the fp32 parameters (zf_nerf_mlp_unfold_grads). Other widths run the folded bf16 layer chain as GEMMs
    with bias + ReLU epilogues (cuBLASLt through torch), this backend's ReLU backward and bias gradient
    (`relu_backward_`), and the unfold as autograd of the fold.

    `_forward` and `_backward` hold the GEMM layer chain for any device with `relu_backward` given (the CPU tests pass a
    torch restatement of the kernel's contract); the public methods take CUDA tensors only, as the reference's
    checks (nerf_mlp.cu:286-290,493-496,570-574)."""

    def __init__(self, n_features: int, density_width: int, bottleneck_width: int, view_width: int, direction_degree: int) -> None:
        self.layout = NerfMlpLayout(n_features, density_width, bottleneck_width, view_width, direction_degree)
        self._shapes = {name: tuple(t.shape) for name, t in fold(self.layout, torch.zeros(self.layout.numel), self.layout.n_features, 8).items()}
        self._offsets, n = {}, 0
        for name in PACKED_ORDER:
            self._offsets[name] = n
            n += math.prod(self._shapes[name])
        # the tensor-core section: the kernel's widths only (features padded to 56, 64 / 256 / 256, direction degree 4)
        self.tensor_cores = (self.layout.n_features == 56 and density_width == 64 and view_width == 256 and self.layout.n_inputs == 96)
        self._tc_shapes, self._tc_offsets = {}, {}
        if self.tensor_cores:
            folded = fold(self.layout, torch.zeros(self.layout.numel))
            self._tc_shapes = {name: tuple(t.shape) for name, t in folded.items()}
            for name in PACKED_ORDER:
                self._tc_offsets[name] = n
                n += math.prod(self._tc_shapes[name]) * (2 if name.endswith('_bias') else 1)  # fp32 biases: two bf16 slots
            # the transposed weights of the tensor-core backward
            for name in TRANSPOSED_ORDER:
                self._tc_shapes[name] = tuple(reversed(self._tc_shapes[TRANSPOSED_OF[name]]))
                self._tc_offsets[name] = n
                n += math.prod(self._tc_shapes[name])
        self.packed_size = n
        self._status = {}
        if self.tensor_cores:
            # zf_nerf_mlp_pack's targets: element offsets in the packed buffer (the row-major section, the tensor-core
            # forward's, the transposed weights), and the packed-weight gradients as views of one flat fp32 buffer
            self._pack_targets = {name: self._offsets[name] for name in PACKED_ORDER}
            self._pack_targets |= {'tc_' + name: self._tc_offsets[name] for name in PACKED_ORDER}
            self._pack_targets |= {name: self._tc_offsets[name] for name in TRANSPOSED_ORDER}
            self._grad_offsets, g = {}, 0
            for name in PACKED_ORDER:
                self._grad_offsets[name] = g
                g += math.prod(self._tc_shapes[name])
            self._grad_numel = g

    @property
    def n_features(self) -> int:
        return self.layout.n_features

    @property
    def n_inputs(self) -> int:
        return self.layout.n_inputs

    @staticmethod
    def _check(tensor: torch.Tensor, name: str, dtype: torch.dtype) -> None:
        if not tensor.is_cuda or not tensor.is_contiguous() or tensor.dtype != dtype:
            raise RuntimeError(f'ZipNeRF: {name} must be a contiguous cuda tensor of the expected type')

    def _fold(self, params: torch.Tensor) -> dict:
        return fold(self.layout, params[:self.layout.numel], self.layout.n_features, 8)

    def _pack(self, params: torch.Tensor) -> torch.Tensor:
        if params.numel() < self.layout.size:
            raise RuntimeError('ZipNeRF: invalid nerf mlp parameters')
        if not self.tensor_cores:
            folded = self._fold(params)
            return torch.cat([folded[name].reshape(-1).to(torch.bfloat16) for name in PACKED_ORDER])
        if params.is_cuda:
            # one launch: zf_nerf_mlp_pack writes every section of the packed buffer
            from zipnerf_b200 import capi
            packed = torch.empty(self.packed_size, dtype=torch.bfloat16, device=params.device)
            base = packed.data_ptr()
            capi.nerf_mlp_pack(params, {name: base + 2 * offset for name, offset in self._pack_targets.items()})
            return packed
        # on the CPU: one fold in the kernel's shapes; the row-major section is its leading rows and columns
        folded = fold(self.layout, params[:self.layout.numel])
        parts = [folded[name][tuple(slice(0, d) for d in self._shapes[name])].reshape(-1).to(torch.bfloat16) for name in PACKED_ORDER]
        tc = pack_folded(folded)
        parts += [tc[name].reshape(-1).view(torch.bfloat16) if name.endswith('_bias') else tc[name].reshape(-1) for name in PACKED_ORDER]
        transposed = pack_transposed(folded)
        parts += [transposed[name].reshape(-1) for name in TRANSPOSED_ORDER]
        return torch.cat(parts)

    def _weights(self, packed: torch.Tensor) -> dict:
        return {name: packed[self._offsets[name]:self._offsets[name] + math.prod(self._shapes[name])].view(self._shapes[name]) for name in PACKED_ORDER}

    def _tc_weights(self, packed: torch.Tensor, names=PACKED_ORDER) -> dict:
        """Views of the tensor-core section: bf16 weights in the kernels' order, fp32 biases."""
        out = {}
        for name in names:
            a, shape = self._tc_offsets[name], self._tc_shapes[name]
            if name.endswith('_bias'):
                out[name] = packed[a:a + 2 * math.prod(shape)].view(torch.float32)
            else:
                out[name] = packed[a:a + math.prod(shape)].view(shape)
        return out

    def status(self, device) -> torch.Tensor:
        """The device int32 the tensor-core forward sets to 1 if one of its bounded waits ran out (outputs undefined)."""
        key = str(device)
        if key not in self._status:
            self._status[key] = torch.zeros(1, dtype=torch.int32, device=device)
        return self._status[key]

    def _forward_tc(self, features: torch.Tensor, inputs: torch.Tensor, packed: torch.Tensor, training: bool):
        from zipnerf_b200 import capi
        if features.shape[1] != self.n_features or inputs.shape[1] != self.n_inputs or packed.numel() != self.packed_size:
            raise RuntimeError('ZipNeRF: invalid nerf mlp inputs')
        n = features.shape[0]
        outputs = torch.empty(n, 8, dtype=torch.bfloat16, device=features.device)
        if not training:
            capi.nerf_mlp_forward_tc(features, inputs, self._tc_weights(packed), outputs, self.status(features.device))
            return outputs, []
        # the training record: v0, v1, v2 ([3, n, 256] bf16, the context's views), then their ReLU masks for the backward
        record = torch.empty(capi.nerf_mlp_record_size(n) // 2, dtype=torch.bfloat16, device=features.device)
        capi.nerf_mlp_forward_tc(features, inputs, self._tc_weights(packed), outputs, self.status(features.device), activations=record)
        planes = record[:3 * n * self.layout.view_width].view(3, n, self.layout.view_width)
        return outputs, [inputs, planes[0], planes[1], planes[2]]

    def _forward(self, features: torch.Tensor, inputs: torch.Tensor, packed: torch.Tensor, training: bool):
        if features.shape[1] != self.n_features or inputs.shape[1] != self.n_inputs or packed.numel() != self.packed_size:
            raise RuntimeError('ZipNeRF: invalid nerf mlp inputs')
        w = self._weights(packed)
        dw = self.layout.density_width
        zero_bias = packed.new_zeros(self.layout.view_width)
        inputs[:, :dw] = torch._addmm_activation(w['density_bias'], features, w['density'].t())
        v0 = torch._addmm_activation(zero_bias, inputs, w['combined'].t())
        outputs = inputs @ w['skip'].t()
        v1 = torch._addmm_activation(w['view_1_bias'], v0, w['view_1'].t())
        v2 = torch._addmm_activation(w['view_2_bias'], v1, w['view_2'].t())
        outputs += v2 @ w['rgb'].t()
        return outputs, ([inputs, v0, v1, v2] if training else [])

    def _backward(self, grad_outputs, features, packed, context, params, grad_params, relu_backward) -> torch.Tensor:
        if len(context) != 4 or packed.numel() != self.packed_size:
            raise RuntimeError('ZipNeRF: invalid nerf mlp backward inputs')
        inputs, v0, v1, v2 = context
        w = self._weights(packed)
        dw = self.layout.density_width
        bias_grads = {name: torch.zeros(self._shapes[name], device=packed.device) for name in ('density_bias', 'view_1_bias', 'view_2_bias')}
        no_bias = bias_grads['density_bias'][:0]
        g = {'rgb': _weight_grad(grad_outputs, v2)}
        g_v2 = grad_outputs @ w['rgb']
        relu_backward(g_v2, v2, bias_grads['view_2_bias'])
        g['view_2'] = _weight_grad(g_v2, v1)
        g_v1 = g_v2 @ w['view_2']
        relu_backward(g_v1, v1, bias_grads['view_1_bias'])
        g['view_1'] = _weight_grad(g_v1, v0)
        g_v0 = g_v1 @ w['view_1']
        relu_backward(g_v0, v0, no_bias)
        g['combined'] = _weight_grad(g_v0, inputs)
        g['skip'] = _weight_grad(grad_outputs, inputs)
        g_hidden = torch.addmm(grad_outputs @ w['skip'][:, :dw], g_v0, w['combined'][:, :dw])
        relu_backward(g_hidden, inputs[:, :dw], bias_grads['density_bias'])
        g['density'] = _weight_grad(g_hidden, features)
        g.update(bias_grads)
        with torch.enable_grad():
            p = params[:self.layout.numel].detach().float().requires_grad_()
            folded = self._fold(p)
            (grad,) = torch.autograd.grad([folded[name] for name in PACKED_ORDER], p, [g[name].to(p.dtype) for name in PACKED_ORDER])
        grad_params[:self.layout.numel] += grad.to(grad_params.dtype)
        return g_hidden @ w['density']

    def pack(self, params: torch.Tensor) -> torch.Tensor:
        self._check(params, 'params', torch.float32)
        return self._pack(params)

    def forward(self, features: torch.Tensor, inputs: torch.Tensor, packed: torch.Tensor, training: bool):
        for tensor, name in ((features, 'features'), (inputs, 'inputs'), (packed, 'packed')):
            self._check(tensor, name, torch.bfloat16)
        if self.tensor_cores:
            return self._forward_tc(features, inputs, packed, training)
        return self._forward(features, inputs, packed, training)

    def _backward_tc(self, grad_outputs, features, packed, context, params, grad_params) -> torch.Tensor:
        """The backward on the tensor cores (zf_nerf_mlp_backward_tc: the data-gradient chain and the packed-weight
        gradients in fp32), then the unfold of the packed-weight gradients into the parameters (zf_nerf_mlp_unfold_grads)."""
        from zipnerf_b200 import capi
        if len(context) != 4 or packed.numel() != self.packed_size:
            raise RuntimeError('ZipNeRF: invalid nerf mlp backward inputs')
        inputs, base = context[0], context[1]
        n = features.shape[0]
        # the training forward's record: v0, v1, v2 are its first three planes, the ReLU masks follow them
        record_elements = capi.nerf_mlp_record_size(n) // 2
        plane = base.numel()
        if (base.dtype != torch.bfloat16 or not base.is_contiguous() or context[2].data_ptr() != base.data_ptr() + 2 * plane
                or context[3].data_ptr() != base.data_ptr() + 4 * plane
                or base.untyped_storage().nbytes() < 2 * (base.storage_offset() + record_elements)):
            raise RuntimeError('ZipNeRF: nerf mlp backward needs the context of the tensor-core forward')
        activations = base.as_strided((record_elements,), (1,))
        grad_features = torch.empty(n, self.n_features, dtype=torch.bfloat16, device=features.device)
        flat = torch.zeros(self._grad_numel, device=features.device)
        grads = {name: flat[self._grad_offsets[name]:self._grad_offsets[name] + math.prod(shape)].view(shape)
                 for name, shape in capi.NERF_MLP_GRAD_SHAPES.items()}
        workspace = torch.empty(max(capi.load().zf_nerf_mlp_backward_workspace_size(n), 16), dtype=torch.uint8, device=features.device)
        capi.nerf_mlp_backward_tc(grad_outputs, features, inputs, activations, self._tc_weights(packed, TRANSPOSED_ORDER), grad_features, grads,
                                  workspace, self.status(features.device))
        # the unfold into the reference's parameters, one launch (zf_nerf_mlp_unfold_grads)
        capi.nerf_mlp_unfold_grads(params, grads, grad_params)
        return grad_features

    def backward(self, grad_outputs, features, packed, context, params, grad_params) -> torch.Tensor:
        import ZipNeRFCudaBackend as backend
        self._check(params, 'params', torch.float32)
        self._check(grad_params, 'grad_params', torch.float32)
        if self.tensor_cores:
            return self._backward_tc(grad_outputs, features, packed, context, params, grad_params)
        return self._backward(grad_outputs, features, packed, context, params, grad_params, backend.relu_backward_)

// fz_nerf_mlp_pack.cu -- the NeRF MLP's pack (fp32 parameters -> the packed bf16 operands of the layer chain and of the
// tensor-core kernels) and unfold (packed-weight gradients -> parameter gradients), one launch each, for the reference
// model's widths (56 features (50 used), density 64, bottleneck 256, view 256, direction degree 4).
//
// The fold moves the bottleneck into the first view layer and the rgb layer's skip columns and the biases of layers
// reading the inputs into the direction block's last column (the bias lane), as the reference's pack_kernel does
// (nerf_mlp.cu:186-234); a folded column is the fp32 multiply-add chain over the 256 bottleneck outputs in their order,
// so the packed values are the reference's. The unfold is the chain rule of the same fold (unpack_kernel,
// nerf_mlp.cu:236-284), one thread per parameter (no atomics), accumulated into the gradient buffer.
#include <cuda_runtime.h>

#include <cstdint>

#include "zf_mlp.h"
#include "fz_status.h"
#include "fz_tcgen05.cuh"

namespace zf::nerf_mlp::pack {

constexpr int kF = 56;            // density_0.weight columns (features padded to 56)
constexpr int kFK = 64;           // the tensor-core density weight's K (features padded to the MMA K step)
constexpr int kD = 64;            // density width (the hidden layer h)
constexpr int kB = 256;           // bottleneck width
constexpr int kV = 256;           // view width
constexpr int kDir = 27;          // encoded direction features
constexpr int kIn = 96;           // inputs: h, the direction block, the bias lane (last column)
constexpr int kBias = kIn - 1;
constexpr int kViewIn = 288;      // view_0.weight columns: bottleneck, direction block (27 + 5 padding)
constexpr int kRgbIn = kV + kViewIn;  // rgb.weight columns: v2, then the view inputs
constexpr int kOut = 8;           // the row-major chain's output rows (skip, rgb)
constexpr int kOutTc = 16;        // the tensor-core kernels' output rows (the smallest N of an M = 128 MMA)

// offsets of the parameter tensors in the flat fp32 buffer (nerf_mlp_parameters order)
constexpr int64_t kDensity0W = 0, kDensity0B = kDensity0W + kD * kF, kDensity1W = kDensity0B + kD, kDensity1B = kDensity1W + kD;
constexpr int64_t kBottleneckW = kDensity1B + 1, kBottleneckB = kBottleneckW + kB * kD, kView0W = kBottleneckB + kB;
constexpr int64_t kView0B = kView0W + kV * kViewIn, kView1W = kView0B + kV, kView1B = kView1W + kV * kV, kView2W = kView1B + kV;
constexpr int64_t kView2B = kView2W + kV * kV, kRgbW = kView2B + kV, kRgbB = kRgbW + 3 * kRgbIn, kParams = kRgbB + 3;
static_assert(kParams == 227556, "the parameter table of the reference model's widths");

// the folded tensors in the tensor-core kernels' shapes, back to back (one thread per element)
enum Tensor { kTDensity, kTDensityBias, kTCombined, kTSkip, kTView1, kTView1Bias, kTView2, kTView2Bias, kTRgb, kTensors };
__host__ __device__ constexpr int rows_of(const int t) {
    return t == kTDensity || t == kTDensityBias ? kD : t == kTSkip || t == kTRgb ? kOutTc : t == kTCombined || t == kTView1 || t == kTView2 || t == kTView1Bias || t == kTView2Bias ? kV : 0;
}
__host__ __device__ constexpr int cols_of(const int t) {
    return t == kTDensity ? kFK : t == kTCombined || t == kTSkip ? kIn : t == kTView1 || t == kTView2 || t == kTRgb ? kV : 1;
}
__host__ __device__ constexpr int64_t elements_before(const int t) { return t == 0 ? 0 : elements_before(t - 1) + int64_t{rows_of(t - 1)} * cols_of(t - 1); }
constexpr int64_t kFolded = elements_before(kTensors);

// K-slice widths of the forward's weights and of the backward's transposed weights
__host__ __device__ constexpr int k_slice_of(const int t) { return t == kTSkip ? kIn : t == kTRgb ? kV : 64; }
__host__ __device__ constexpr int k_slice_t_of(const int t) { return t == kTSkip || t == kTRgb ? kOutTc : 64; }

// element (r, c) of a [rows x k] weight stored as K-slices of k_slice columns, each in the no-swizzle K-major order
__device__ __forceinline__ int64_t sliced_position(const int r, const int c, const int rows, const int k, const int k_slice) {
    const int s = c / k_slice, width = min(k_slice, k - s * k_slice);
    return int64_t{rows} * s * k_slice + canonical_offset(r, c - s * k_slice, width) / 2;
}

// a folded column: sum over the bottleneck outputs k of row[k] times the bottleneck weight (bias column: its bias),
// the fp32 multiply-add chain in k order
__device__ __forceinline__ float fold_column(const float* __restrict__ params, const float* __restrict__ row, const int column) {
    float sum = 0.0f;
    if (column == kBias) {
        for (int k = 0; k < kB; k++) sum = __fmaf_rn(row[k], __ldg(params + kBottleneckB + k), sum);
    }
    else {
        for (int k = 0; k < kB; k++) sum = __fmaf_rn(row[k], __ldg(params + kBottleneckW + k * kD + column), sum);
    }
    return sum;
}

__device__ __forceinline__ uint16_t to_bf16_bits(const float v) {
    uint32_t out;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(out) : "f"(0.0f), "f"(v));
    return static_cast<uint16_t>(out & 0xFFFFu);
}

// the folded value of element (r, c) of tensor t (the tensor-core shapes; zeros where the shape pads)
__device__ __forceinline__ float folded_value(const float* __restrict__ params, const int t, const int r, const int c) {
    switch (t) {
        case kTDensity: return c < kF ? __ldg(params + kDensity0W + r * kF + c) : 0.0f;
        case kTDensityBias: return __ldg(params + kDensity0B + r);
        case kTCombined: {
            const float* view_0 = params + kView0W + int64_t{r} * kViewIn;
            if (c < kD) return fold_column(params, view_0, c);
            if (c == kBias) return __fadd_rn(fold_column(params, view_0, c), __ldg(params + kView0B + r));
            if (c < kD + kDir) return __ldg(view_0 + kB + c - kD);
            return 0.0f;
        }
        case kTSkip: {
            if (r == 0) return c < kD ? __ldg(params + kDensity1W + c) : c == kBias ? __ldg(params + kDensity1B) : 0.0f;
            if (r > 3) return 0.0f;
            const float* rgb = params + kRgbW + int64_t{r - 1} * kRgbIn + kV;  // the rgb row's weights of the view inputs
            if (c < kD) return fold_column(params, rgb, c);
            if (c == kBias) return __fadd_rn(fold_column(params, rgb, c), __ldg(params + kRgbB + r - 1));
            if (c < kD + kDir) return __ldg(rgb + kB + c - kD);
            return 0.0f;
        }
        case kTView1: return __ldg(params + kView1W + r * kV + c);
        case kTView1Bias: return __ldg(params + kView1B + r);
        case kTView2: return __ldg(params + kView2W + r * kV + c);
        case kTView2Bias: return __ldg(params + kView2B + r);
        case kTRgb: return r >= 1 && r <= 3 ? __ldg(params + kRgbW + int64_t{r - 1} * kRgbIn + c) : 0.0f;
        default: return 0.0f;
    }
}

struct PackTargets {
    uint16_t* row_major[kTensors];   // bf16, the reference chain's shapes (density [64, 56], skip and rgb 8 rows)
    uint16_t* tc[kTensors];          // bf16 K-sliced weights; the biases as fp32 (two bf16 slots each)
    uint16_t* transposed[kTensors];  // bf16 K-sliced transposed weights (none for the biases)
};

__global__ void fz_nerf_mlp_pack_kernel(const float* __restrict__ params, const PackTargets out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= kFolded) return;
    int t = 0;
    int64_t e = i;  // the element within tensor t
    while (t + 1 < kTensors && e >= int64_t{rows_of(t)} * cols_of(t)) {
        e -= int64_t{rows_of(t)} * cols_of(t);
        t++;
    }
    const int rows = rows_of(t), cols = cols_of(t);
    const int r = static_cast<int>(e / cols), c = static_cast<int>(e % cols);
    const float v = folded_value(params, t, r, c);
    const uint16_t bits = to_bf16_bits(v);
    const bool bias = cols == 1;
    // the layer chain's row-major operands
    const int rm_cols = t == kTDensity ? kF : cols, rm_rows = t == kTSkip || t == kTRgb ? kOut : rows;
    if (out.row_major[t] != nullptr && r < rm_rows && c < rm_cols) out.row_major[t][int64_t{r} * rm_cols + c] = bits;
    // the tensor-core forward's operands: K-sliced weights, bf16-rounded biases stored as fp32
    if (out.tc[t] != nullptr) {
        if (bias) reinterpret_cast<float*>(out.tc[t])[r] = __uint_as_float(static_cast<uint32_t>(bits) << 16);
        else out.tc[t][sliced_position(r, c, rows, cols, k_slice_of(t))] = bits;
    }
    // the backward's transposed operands: element (c, r) of the [cols x rows] transpose
    if (!bias && out.transposed[t] != nullptr) out.transposed[t][sliced_position(c, r, cols, rows, k_slice_t_of(t))] = bits;
}

// gradient of a weight over the bottleneck outputs, column k, from the gradient row of its folded weights (the bias
// lane's term first, then the 64 hidden columns in order)
__device__ __forceinline__ float unfold_row(const float* __restrict__ params, const float* __restrict__ grad_row, const int k) {
    float sum = __fmul_rn(__ldg(grad_row + kBias), __ldg(params + kBottleneckB + k));
    for (int j = 0; j < kD; j++) sum = __fmaf_rn(__ldg(grad_row + j), __ldg(params + kBottleneckW + k * kD + j), sum);
    return sum;
}

// gradient of bottleneck weight (k, column) (column kBias: of bottleneck bias k) from the folded columns that used it:
// the first view layer's and the rgb skip rows'
__device__ __forceinline__ float unfold_bottleneck(const float* __restrict__ params, const zf_nerf_mlp_grads& g, const int k, const int column) {
    float sum = 0.0f;
    for (int o = 0; o < kV; o++) sum = __fmaf_rn(__ldg(params + kView0W + int64_t{o} * kViewIn + k), __ldg(g.combined + o * kIn + column), sum);
    for (int r = 0; r < 3; r++) sum = __fmaf_rn(__ldg(params + kRgbW + int64_t{r} * kRgbIn + kV + k), __ldg(g.skip + (r + 1) * kIn + column), sum);
    return sum;
}

__global__ void fz_nerf_mlp_unfold_kernel(const float* __restrict__ params, const zf_nerf_mlp_grads g, float* __restrict__ grad_params) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= kParams) return;
    float grad = 0.0f;
    if (i < kDensity0B) {
        grad = __ldg(g.density + (i / kF) * kFK + i % kF);
    }
    else if (i < kDensity1W) {
        grad = __ldg(g.density_bias + (i - kDensity0B));
    }
    else if (i < kDensity1B) {
        grad = __ldg(g.skip + (i - kDensity1W));                   // row 0, the hidden columns
    }
    else if (i < kBottleneckW) {
        grad = __ldg(g.skip + kBias);                              // row 0, the bias lane
    }
    else if (i < kBottleneckB) {
        const int e = static_cast<int>(i - kBottleneckW);
        grad = unfold_bottleneck(params, g, e / kD, e % kD);
    }
    else if (i < kView0W) {
        grad = unfold_bottleneck(params, g, static_cast<int>(i - kBottleneckB), kBias);
    }
    else if (i < kView0B) {
        const int e = static_cast<int>(i - kView0W), o = e / kViewIn, column = e % kViewIn;
        if (column < kB) grad = unfold_row(params, g.combined + o * kIn, column);
        else if (column < kB + kDir) grad = __ldg(g.combined + o * kIn + kD + column - kB);
    }
    else if (i < kView1W) {
        grad = __ldg(g.combined + (i - kView0B) * kIn + kBias);
    }
    else if (i < kView1B) {
        grad = __ldg(g.view_1 + (i - kView1W));
    }
    else if (i < kView2W) {
        grad = __ldg(g.view_1_bias + (i - kView1B));
    }
    else if (i < kView2B) {
        grad = __ldg(g.view_2 + (i - kView2W));
    }
    else if (i < kRgbW) {
        grad = __ldg(g.view_2_bias + (i - kView2B));
    }
    else if (i < kRgbB) {
        const int e = static_cast<int>(i - kRgbW), r = e / kRgbIn, column = e % kRgbIn;
        const float* skip_row = g.skip + (r + 1) * kIn;
        if (column < kV) grad = __ldg(g.rgb + (r + 1) * kV + column);
        else if (column < kV + kB) grad = unfold_row(params, skip_row, column - kV);
        else if (column < kV + kB + kDir) grad = __ldg(skip_row + kD + column - kV - kB);
    }
    else {
        grad = __ldg(g.skip + (i - kRgbB + 1) * kIn + kBias);
    }
    if (grad != 0.0f) grad_params[i] += grad;
}

}  // namespace zf::nerf_mlp::pack

int64_t zf_nerf_mlp_parameter_count(void) { return zf::nerf_mlp::pack::kParams; }

int zf_nerf_mlp_pack(const float* params, const zf_nerf_mlp_packed* out, cudaStream_t stream) {
    using namespace zf::nerf_mlp::pack;
    if (params == nullptr || out == nullptr) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "invalid nerf mlp pack arguments");
    PackTargets t{};
    uint16_t* const row_major[kTensors] = {out->density, out->density_bias, out->combined, out->skip, out->view_1, out->view_1_bias, out->view_2,
                                           out->view_2_bias, out->rgb};
    uint16_t* const tc[kTensors] = {out->tc_density, reinterpret_cast<uint16_t*>(out->tc_density_bias), out->tc_combined, out->tc_skip, out->tc_view_1,
                                    reinterpret_cast<uint16_t*>(out->tc_view_1_bias), out->tc_view_2, reinterpret_cast<uint16_t*>(out->tc_view_2_bias),
                                    out->tc_rgb};
    uint16_t* const transposed[kTensors] = {out->density_t, nullptr, out->combined_t, out->skip_t, out->view_1_t, nullptr, out->view_2_t, nullptr, out->rgb_t};
    for (int i = 0; i < kTensors; i++) {
        t.row_major[i] = row_major[i];
        t.tc[i] = tc[i];
        t.transposed[i] = transposed[i];
        if (reinterpret_cast<uintptr_t>(tc[i]) % 4 != 0) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "nerf mlp pack: misaligned target");
    }
    constexpr int kThreadsPerBlock = 256;
    const unsigned blocks = static_cast<unsigned>((kFolded + kThreadsPerBlock - 1) / kThreadsPerBlock);
    fz_nerf_mlp_pack_kernel<<<blocks, kThreadsPerBlock, 0, stream>>>(params, t);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ZF_OK : zf::set_cuda_error(e, "nerf mlp pack");
}

int zf_nerf_mlp_unfold_grads(const float* params, const zf_nerf_mlp_grads* grads, float* grad_params, cudaStream_t stream) {
    using namespace zf::nerf_mlp::pack;
    if (params == nullptr || grads == nullptr || grad_params == nullptr) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "invalid nerf mlp unfold arguments");
    const float* pointers[] = {grads->density, grads->density_bias, grads->combined, grads->skip, grads->view_1, grads->view_1_bias,
                               grads->view_2, grads->view_2_bias, grads->rgb};
    for (const float* p : pointers) {
        if (p == nullptr) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "nerf mlp gradients must be given");
    }
    constexpr int kThreadsPerBlock = 256;
    const unsigned blocks = static_cast<unsigned>((kParams + kThreadsPerBlock - 1) / kThreadsPerBlock);
    fz_nerf_mlp_unfold_kernel<<<blocks, kThreadsPerBlock, 0, stream>>>(params, *grads, grad_params);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ZF_OK : zf::set_cuda_error(e, "nerf mlp unfold");
}

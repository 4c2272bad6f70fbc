// fz_optim.cuh -- the fused Adam step of the hash grids and MLP parameters for sm_100a: one launch over all optimized
// buffers that unscales and sanitizes the gradients (fp32, or fp16 as accumulated by the NeRF-level backward), adds
// the per-level grid regularizer's gradient, updates the moments and parameters, zeroes the gradients, and reduces the
// per-level sums of squared parameters into the scale-feature magnitudes and the regularizer value.
//
// The per-element update is the reference's operation for operation (B/optimizer/src/optimizer_api.cu:43-53,
// B/ = ZipNeRFCudaBackend/ZipNeRFCudaBackend/; the library is compiled with --use_fast_math like the reference), so
// parameters, moments and zeroed gradients equal the reference kernel's bit for bit. The work split is this build's:
// the host cuts every buffer's level ranges into block-sized chunks, so a block lies inside one range (one buffer, one
// level or none) and its loop needs no per-element range search; each thread streams two 16-byte groups of each of the
// four arrays per iteration. The per-level sums are reduced in a fixed order (thread partials, a warp tree, the block's
// warps in order, then the blocks of a level in order by the last block), so the magnitudes and the regularizer are
// deterministic, where the reference sums them with floating-point atomics.
#pragma once

#include <cfloat>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace zf {

constexpr int kAdamMaxBuffers = 8;                               // optimizer_api.cu:15
constexpr int kAdamMaxLevels = 32;                               // optimizer_api.cu:16
constexpr int kAdamMaxRanges = kAdamMaxLevels + kAdamMaxBuffers;  // optimizer_api.cu:17
constexpr int kAdamBlock = 256;
constexpr int kAdamBlocksPerSm = 4;  // 64 registers: two groups of the four arrays in flight per thread

struct AdamBuffer {
    float4* param;
    float4* grad;       // fp32 gradient, or null
    uint2* grad_half;   // four fp16 gradients per group (instead of grad), or null
    float4* exp_avg;
    float4* exp_avg_sq;
    float inv_grad_scale;
};

// consecutive groups (four parameters) of one buffer that form a regularized grid level (level >= 0) or an
// unregularized span (level -1), and the blocks that process them: block first_block + k takes groups
// [begin + k chunk, min(begin + (k + 1) chunk, end))
struct AdamRange {
    int64_t begin, end, chunk;
    int buffer, level, first_block;
};

struct AdamParams {
    AdamBuffer buffers[kAdamMaxBuffers];
    AdamRange ranges[kAdamMaxRanges];
    float level_reg_weights[kAdamMaxLevels];   // reg_weight / level size
    double level_inv_sizes[kAdamMaxLevels];
    int n_ranges, n_levels, n_blocks;
    float lr, beta1, beta2, eps, bias_correction1, bias_correction2;
    double max_value_sq;
    double* block_sums;      // [n_blocks] sum of squared updated parameters of each block (its range's level)
    unsigned* counter;       // finished blocks (zero between steps)
    float* magnitudes;       // [n_levels] sqrt(max_value^2 + mean(p^2)) per level
    float* regularization;   // 0.5 reg_weight sum_levels mean(p^2)
};

// one parameter (optimizer_api.cu:43-53): the gradient unscaled plus the regularizer's gradient, nan_to_num-ed, the
// moment and parameter update; returns the updated parameter squared
__device__ __forceinline__ float adam_update(float& p, float g, float& m, float& v, const float inv_grad_scale, const float reg_weight,
                                             const AdamParams& a) {
    g = g * inv_grad_scale + reg_weight * p;
    g = isnan(g) ? 0.0f : fminf(fmaxf(g, -FLT_MAX), FLT_MAX);
    m = a.beta1 * m + (1.0f - a.beta1) * g;
    v = a.beta2 * v + (1.0f - a.beta2) * g * g;
    p -= a.lr * (m / a.bias_correction1) / (sqrtf(v / a.bias_correction2) + a.eps);
    return p * p;
}

// four fp16 gradients, clamped to the fp16 range so that an overflow cannot reach the moments (optimizer_api.cu:83-86)
__device__ __forceinline__ float4 half_gradients(const uint2 h) {
    const float2 xy = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
    const float2 zw = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
    return make_float4(fminf(fmaxf(xy.x, -65504.0f), 65504.0f), fminf(fmaxf(xy.y, -65504.0f), 65504.0f), fminf(fmaxf(zw.x, -65504.0f), 65504.0f),
                       fminf(fmaxf(zw.y, -65504.0f), 65504.0f));
}

__device__ __forceinline__ float adam_group(float4& p, const float4 g, float4& m, float4& v, const float inv_grad_scale, const float reg_weight,
                                            const AdamParams& a) {
    float sum = adam_update(p.x, g.x, m.x, v.x, inv_grad_scale, reg_weight, a);
    sum += adam_update(p.y, g.y, m.y, v.y, inv_grad_scale, reg_weight, a);
    sum += adam_update(p.z, g.z, m.z, v.z, inv_grad_scale, reg_weight, a);
    sum += adam_update(p.w, g.w, m.w, v.w, inv_grad_scale, reg_weight, a);
    return sum;
}

template <bool HALF>
__device__ __forceinline__ float adam_chunk(const AdamBuffer& buffer, const int64_t begin, const int64_t end, const float reg_weight, const AdamParams& a) {
    float4* __restrict__ param = buffer.param;
    float4* __restrict__ grad = buffer.grad;
    uint2* __restrict__ grad_half = buffer.grad_half;
    float4* __restrict__ exp_avg = buffer.exp_avg;
    float4* __restrict__ exp_avg_sq = buffer.exp_avg_sq;
    const float inv = buffer.inv_grad_scale;
    float sum = 0.0f;
    int64_t i = begin + threadIdx.x;
    // two groups per thread and iteration: eight independent 16-byte loads in flight
    for (; i + kAdamBlock < end; i += 2 * kAdamBlock) {
        const int64_t j = i + kAdamBlock;
        float4 p0 = param[i], p1 = param[j], m0 = exp_avg[i], m1 = exp_avg[j], v0 = exp_avg_sq[i], v1 = exp_avg_sq[j];
        const float4 g0 = HALF ? half_gradients(grad_half[i]) : grad[i];
        const float4 g1 = HALF ? half_gradients(grad_half[j]) : grad[j];
        sum += adam_group(p0, g0, m0, v0, inv, reg_weight, a);
        sum += adam_group(p1, g1, m1, v1, inv, reg_weight, a);
        param[i] = p0;
        param[j] = p1;
        exp_avg[i] = m0;
        exp_avg[j] = m1;
        exp_avg_sq[i] = v0;
        exp_avg_sq[j] = v1;
        if (HALF) {
            grad_half[i] = make_uint2(0u, 0u);
            grad_half[j] = make_uint2(0u, 0u);
        } else {
            grad[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            grad[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
    }
    if (i < end) {
        float4 p = param[i], m = exp_avg[i], v = exp_avg_sq[i];
        const float4 g = HALF ? half_gradients(grad_half[i]) : grad[i];
        sum += adam_group(p, g, m, v, inv, reg_weight, a);
        param[i] = p;
        exp_avg[i] = m;
        exp_avg_sq[i] = v;
        if (HALF) grad_half[i] = make_uint2(0u, 0u);
        else grad[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    return sum;
}

__global__ void __launch_bounds__(kAdamBlock, kAdamBlocksPerSm) fz_adam_kernel(const __grid_constant__ AdamParams a) {
    __shared__ float warp_sums[kAdamBlock / 32];
    __shared__ bool last_block;
    int r = 0;
    while (r + 1 < a.n_ranges && a.ranges[r + 1].first_block <= static_cast<int>(blockIdx.x)) r++;
    const AdamRange& range = a.ranges[r];
    const AdamBuffer& buffer = a.buffers[range.buffer];
    const int64_t begin = range.begin + static_cast<int64_t>(blockIdx.x - range.first_block) * range.chunk;
    const int64_t end = min(begin + range.chunk, range.end);
    const float reg_weight = range.level >= 0 ? a.level_reg_weights[range.level] : 0.0f;
    float sum = buffer.grad_half != nullptr ? adam_chunk<true>(buffer, begin, end, reg_weight, a) : adam_chunk<false>(buffer, begin, end, reg_weight, a);
    // the block's sum of squares in a fixed order: a warp tree, then the warps in order
    for (int offset = 16; offset > 0; offset /= 2) sum += __shfl_xor_sync(0xffffffffu, sum, offset);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (lane == 0) warp_sums[warp] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        float block_sum = 0.0f;
        for (int w = 0; w < kAdamBlock / 32; w++) block_sum += warp_sums[w];
        a.block_sums[blockIdx.x] = static_cast<double>(block_sum);
        __threadfence();
        last_block = atomicAdd(a.counter, 1u) == static_cast<unsigned>(a.n_blocks) - 1;
    }
    __syncthreads();
    if (!last_block || warp != 0) return;
    // the last block: each level's blocks in order (one lane per level), then the regularizer over the levels in order
    __threadfence();
    double value = 0.0;
    for (int rr = 0; rr < a.n_ranges; rr++) {
        const AdamRange& q = a.ranges[rr];
        if (q.level < 0 || q.level % 32 != lane) continue;
        const int next = rr + 1 < a.n_ranges ? a.ranges[rr + 1].first_block : a.n_blocks;
        double level_sum = 0.0;
        for (int b = q.first_block; b < next; b++) level_sum += __ldcg(&a.block_sums[b]);
        a.magnitudes[q.level] = static_cast<float>(sqrt(a.max_value_sq + level_sum * a.level_inv_sizes[q.level]));
        value = 0.5 * a.level_reg_weights[q.level] * level_sum;
    }
    // levels < 32: lane l holds level l's term; sum them in level order
    double regularization = 0.0;
    for (int l = 0; l < a.n_levels; l++) regularization += __shfl_sync(0xffffffffu, value, l);
    if (lane == 0) {
        *a.regularization = static_cast<float>(regularization);
        *a.counter = 0u;
    }
}

}  // namespace zf

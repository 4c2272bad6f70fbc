// fz_final.cuh -- sm_100a kernels of the final sampling level: the training losses with their gradients w.r.t. the raw
// outputs of all levels (charbonnier data loss of the composited color against the target over a random background,
// distortion loss on the curved distances, interlevel losses of the proposal weights against the blurred final
// weights), and the inference compositing of color, opacity and depth.
//
// Per ray the arithmetic is the reference's, operation for operation (B/sampling/include/ray_ops.cuh:20-24,91-166 and
// B/sampling/src/sampling_api.cu:203-424, B/ = ZipNeRFCudaBackend/ZipNeRFCudaBackend/), in the same fast-math build, so
// gradients and images equal the reference kernels' bit for bit (the loss sums are accumulated with atomics across
// warps, in an order that varies). One ray per thread and one warp per block, as the per-ray recurrences (optical
// depth, composite backward, the blurred-histogram spline) are sequential; the NeRF outputs of an interval are read as
// one 8-byte load and its output-gradient row leaves as one 16-byte store, instead of per-value 2-byte accesses.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "fz_sampling.cuh"

namespace zf {

constexpr int kMaxProposalLevels = 4;  // ray_ops.cuh:11
constexpr int kNerfOutputs = 8;        // raw density, rgb logits, zero padding (sampling_api.cu:15)
constexpr float kRgbPadding = 0.001f;  // sampling_api.cu:14

struct ProposalLevelsArgs {
    int n_levels;
    int n_intervals[kMaxProposalLevels];
    const float* raw_density[kMaxProposalLevels];
    const float* sdist[kMaxProposalLevels];
    const float* tdist[kMaxProposalLevels];
    const float* weights[kMaxProposalLevels];
    float* raw_density_grad[kMaxProposalLevels];
    float interlevel_weight[kMaxProposalLevels];
    float interlevel_blur[kMaxProposalLevels];
};

struct TrainFinalArgs {
    const uint16_t* nerf_outputs;   // bf16 [n_rays, n, 8]
    const float* sdist;             // [n_rays, n + 1]
    const float* tdist;
    ProposalLevelsArgs proposals;
    const float* directions;        // [n_rays, 3]
    unsigned long long seed;
    const float* rgb_target;        // [n_rays, 3]
    uint16_t* nerf_outputs_grad;    // bf16 [n_rays, n, 8]
    float* loss_sums;               // [4] or null
    int n;
    float charbonnier_padding, distortion_weight, distortion_power, distortion_premult;
    int n_rays;
    int vectors;                    // nonzero: nerf_outputs 8-byte and nerf_outputs_grad 16-byte aligned
};

struct CompositeFinalArgs {
    const uint16_t* nerf_outputs;   // bf16 [n_rays, n, 8]
    const float* tdist;
    const float* directions;
    const float* background;        // [3]
    const int64_t* pixel_indices;   // [n_rays]
    float* rgb;                     // [pixels, 3]
    float* alpha;                   // [pixels] or null
    float* depth;                   // [pixels] or null
    int n, n_rays;
    int use_median_depth;
    int vectors;                    // nonzero: nerf_outputs 8-byte aligned
};

// signed power ladder of the distortion loss's curved distances (ray_ops.cuh:20-24)
__device__ __forceinline__ float power_ladder(const float x, const float p, const float premult) {
    const float xp = fabsf(x * premult);
    const float y = fabsf(p - 1.0f) / p * (powf(xp / fabsf(p - 1.0f) + 1.0f, p) - 1.0f);
    return copysignf(y, x);
}

// alpha compositing of n intervals with their optical depths sigma dt |d| (ray_ops.cuh:91-99)
__device__ __forceinline__ void composite_depths(const float* density, const float* t, const int n, const float direction_norm, float* w_out, float* x_out) {
    float optical_depth = 0.0f;
    for (int i = 0; i < n; i++) {
        const float x = density[i] * (t[i + 1] - t[i]) * direction_norm;
        w_out[i] = -expm1f(-x) * expf(-optical_depth);
        optical_depth += x;
        x_out[i] = x;
    }
}

// dL/dx_k = g_k T_k exp(-x_k) - sum_{i>k} g_i w_i, in place (ray_ops.cuh:102-117)
__device__ __forceinline__ void composite_backward(float* grad, const float* x, const float* w, const int n) {
    float transmittance[kMaxSamplingIntervals];
    float optical_depth = 0.0f;
    for (int i = 0; i < n; i++) {
        optical_depth += x[i];
        transmittance[i] = expf(-optical_depth);
    }
    float suffix = 0.0f;
    for (int i = n - 1; i >= 0; i--) {
        const float g = grad[i];
        grad[i] = g * transmittance[i] - suffix;
        suffix += g * w[i];
    }
}

__device__ __forceinline__ float plus_eps(const float x) { return fabsf(x) < kSamplingTiny ? kSamplingTiny : nextafterf(x, INFINITY); }
__device__ __forceinline__ float minus_eps(const float x) { return fabsf(x) < kSamplingTiny ? -kSamplingTiny : nextafterf(x, -INFINITY); }

// the histogram (t, w) of n bins blurred by a box of the given half width, resampled into the nq - 1 bins of the sorted
// edges tq (ray_ops.cuh:121-166): the blurred pdf is a piecewise-linear spline whose knots are the merged box edges;
// its integral at the query edges gives the resampled weights
__device__ __forceinline__ void blur_and_resample(const float* tq, const int nq, const float* t, const float* w, const int n, const float halfwidth,
                                                  float* wq_out) {
    float edge_lo[kMaxSamplingIntervals + 1], edge_hi[kMaxSamplingIntervals + 1], slope_change[kMaxSamplingIntervals + 1];
    float pdf_previous = 0.0f;
    for (int i = 0; i <= n; i++) {
        const float dt = i < n ? t[i + 1] - t[i] : 0.0f;
        const float pdf = i < n && dt >= kSamplingTiny ? w[i] / dt : 0.0f;
        edge_lo[i] = t[i] - halfwidth;
        edge_hi[i] = fmaxf(plus_eps(t[i]), t[i] + halfwidth);
        slope_change[i] = (pdf - pdf_previous) / (edge_hi[i] - edge_lo[i]);
        pdf_previous = pdf;
    }
    constexpr int kMaxKnots = 2 * (kMaxSamplingIntervals + 1);
    float tp[kMaxKnots], yp[kMaxKnots];
    const int n_knots = 2 * (n + 1);
    int i_lo = 0, i_hi = 0;
    float slope = 0.0f;
    for (int k = 0; k < n_knots; k++) {
        const bool take_lo = i_hi > n || (i_lo <= n && edge_lo[i_lo] <= edge_hi[i_hi]);
        const float knot = take_lo ? edge_lo[i_lo] : edge_hi[i_hi];
        yp[k] = k == 0 || k == n_knots - 1 ? 0.0f : yp[k - 1] + (knot - tp[k - 1]) * slope;
        tp[k] = knot;
        if (k < n_knots - 2) slope += take_lo ? slope_change[i_lo] : -slope_change[i_hi];
        if (take_lo) i_lo++;
        else i_hi++;
    }
    const float t_min = tp[0], t_max = minus_eps(tp[n_knots - 1]);
    int k = 0;
    float integral = 0.0f, previous = 0.0f;
    for (int j = 0; j < nq; j++) {
        const float q = fminf(fmaxf(tq[j], t_min), t_max);
        while (k + 2 < n_knots && tp[k + 1] <= q) {
            integral += 0.5f * (tp[k + 1] - tp[k]) * (yp[k] + yp[k + 1]);
            k++;
        }
        const float a = (yp[k + 1] - yp[k]) / fmaxf(kSamplingEps * kSamplingEps, 2.0f * (tp[k + 1] - tp[k]));
        const float td = q - tp[k];
        const float value = (a * td + yp[k]) * td + integral;
        if (j > 0) wq_out[j - 1] = fmaxf(value - previous, 0.0f);
        previous = value;
    }
}

// the raw outputs (density, rgb logits) of interval i of a ray: one 8-byte load when aligned
__device__ __forceinline__ void load_raw_outputs(const uint16_t* outputs, const int64_t index, const int vectors, float& r0, float& r1, float& r2,
                                                 float& r3) {
    const uint16_t* p = outputs + kNerfOutputs * index;
    if (vectors) {
        const uint2 words = *reinterpret_cast<const uint2*>(p);
        r0 = __uint_as_float(words.x << 16);
        r1 = __uint_as_float(words.x & 0xffff0000u);
        r2 = __uint_as_float(words.y << 16);
        r3 = __uint_as_float(words.y & 0xffff0000u);
    } else {
        r0 = bf16_bits_to_f32(p[0]);
        r1 = bf16_bits_to_f32(p[1]);
        r2 = bf16_bits_to_f32(p[2]);
        r3 = bf16_bits_to_f32(p[3]);
    }
}

// densities, rgb sigmoids, optical depths and weights of the final level (sampling_api.cu:203-220); the colors
// s (1 + 2 padding) - padding are formed from the sigmoids where they are used
__device__ __forceinline__ void evaluate_final(const uint16_t* outputs, const float* t, const int n, const float direction_norm, const int64_t ray,
                                               const int vectors, float* density, float* x, float* w, float3* sigmoids) {
    for (int i = 0; i < n; i++) {
        float r0, r1, r2, r3;
        load_raw_outputs(outputs, ray * n + i, vectors, r0, r1, r2, r3);
        // a sample with non-finite outputs is empty, so that it cannot spread NaNs to the loss and all gradients
        const bool valid = isfinite(r0) && isfinite(r1) && isfinite(r2) && isfinite(r3);
        density[i] = valid ? activate_density(r0) : 0.0f;
        sigmoids[i] = valid ? make_float3(1.0f / (1.0f + expf(-r1)), 1.0f / (1.0f + expf(-r2)), 1.0f / (1.0f + expf(-r3))) : make_float3(0.5f, 0.5f, 0.5f);
    }
    composite_depths(density, t, n, direction_norm, w, x);
}

__device__ __forceinline__ float3 padded_color(const float3 s) {
    return make_float3(s.x * (1.0f + 2.0f * kRgbPadding) - kRgbPadding, s.y * (1.0f + 2.0f * kRgbPadding) - kRgbPadding,
                       s.z * (1.0f + 2.0f * kRgbPadding) - kRgbPadding);
}

// gradients of the weights of n intervals -> the raw densities, activation exp(raw - 1) (sampling_api.cu:223-229)
__device__ __forceinline__ void weights_backward_to_raw(float* grad, const float* x, const float* w, const float* density, const float* raw, const float* t,
                                                        const int n, const float direction_norm) {
    composite_backward(grad, x, w, n);
    for (int i = 0; i < n; i++) {
        const bool clipped = raw[i] - 1.0f > kMaxDensityExponent;
        grad[i] = clipped ? 0.0f : grad[i] * (t[i + 1] - t[i]) * direction_norm * density[i];
    }
}

__device__ __forceinline__ float warp_sum(float value) {
    for (int offset = 16; offset > 0; offset /= 2) value += __shfl_down_sync(0xffffffffu, value, offset);
    return value;
}

// training losses and the gradients of all levels' raw outputs (sampling_api.cu:231-376)
__global__ void __launch_bounds__(32) fz_train_final_kernel(const __grid_constant__ TrainFinalArgs a) {
    const int ray_idx = blockIdx.x * blockDim.x + threadIdx.x;
    // inactive lanes take part in the warp reductions with zero contributions
    const bool active = ray_idx < a.n_rays;
    const int n = active ? a.n : 0;
    const float inv_n_rays = 1.0f / a.n_rays;
    float loss_data = 0.0f, loss_mse = 0.0f, loss_interlevel = 0.0f, loss_distortion = 0.0f;
    const int64_t ray = ray_idx;
    const float* t = a.tdist + ray * (a.n + 1);
    const float* s = a.sdist + ray * (a.n + 1);
    const float direction_norm = active ? norm3(make_float3(a.directions[3 * ray], a.directions[3 * ray + 1], a.directions[3 * ray + 2])) : 0.0f;
    float density[kMaxSamplingIntervals], x[kMaxSamplingIntervals], w[kMaxSamplingIntervals], grad_w[kMaxSamplingIntervals];
    float3 sigmoids[kMaxSamplingIntervals];
    evaluate_final(a.nerf_outputs, t, n, direction_norm, ray, a.vectors, density, x, w, sigmoids);

    // charbonnier data loss of the composited color over the random background
    float3 rgb = make_float3(0.0f, 0.0f, 0.0f);
    float acc = 0.0f;
    for (int i = 0; i < n; i++) {
        const float3 color = padded_color(sigmoids[i]);
        rgb.x += w[i] * color.x;
        rgb.y += w[i] * color.y;
        rgb.z += w[i] * color.z;
        acc += w[i];
    }
    float3 grad_rgb = make_float3(0.0f, 0.0f, 0.0f);
    float3 bg = make_float3(0.0f, 0.0f, 0.0f);
    if (active) {
        bg = make_float3(rng_uniform(a.seed, kStreamBackground, 3 * ray), rng_uniform(a.seed, kStreamBackground, 3 * ray + 1),
                         rng_uniform(a.seed, kStreamBackground, 3 * ray + 2));
        const float background_weight = fmaxf(1.0f - acc, 0.0f);
        const float r[3] = {rgb.x + background_weight * bg.x - a.rgb_target[3 * ray], rgb.y + background_weight * bg.y - a.rgb_target[3 * ray + 1],
                            rgb.z + background_weight * bg.z - a.rgb_target[3 * ray + 2]};
        float g[3];
        for (int c = 0; c < 3; c++) {
            const float q = sqrtf(r[c] * r[c] + a.charbonnier_padding * a.charbonnier_padding);
            loss_data += q * inv_n_rays / 3.0f;
            loss_mse += r[c] * r[c] * inv_n_rays / 3.0f;
            g[c] = r[c] / q * inv_n_rays / 3.0f;
        }
        grad_rgb = make_float3(g[0], g[1], g[2]);
    }
    const float grad_background = 1.0f - acc >= 0.0f ? grad_rgb.x * bg.x + grad_rgb.y * bg.y + grad_rgb.z * bg.z : 0.0f;
    for (int i = 0; i < n; i++) {
        const float3 color = padded_color(sigmoids[i]);
        grad_w[i] = grad_rgb.x * color.x + grad_rgb.y * color.y + grad_rgb.z * color.z - grad_background;
    }

    // distortion loss on the curved metric distances
    if (n > 0) {
        float u[kMaxSamplingIntervals], ds[kMaxSamplingIntervals];
        float previous = power_ladder(t[0], a.distortion_power, a.distortion_premult);
        float w_total = 0.0f, wu_total = 0.0f;
        for (int i = 0; i < n; i++) {
            const float next = power_ladder(t[i + 1], a.distortion_power, a.distortion_premult);
            u[i] = 0.5f * (previous + next);
            ds[i] = next - previous;
            previous = next;
            w_total += w[i];
            wu_total += w[i] * u[i];
        }
        const float scale = a.distortion_weight * inv_n_rays;
        float w_before = 0.0f, wu_before = 0.0f, loss = 0.0f;
        for (int i = 0; i < n; i++) {
            const float w_after = w_total - w_before - w[i], wu_after = wu_total - wu_before - w[i] * u[i];
            const float inter = u[i] * w_before - wu_before + wu_after - u[i] * w_after;  // sum_j w_j |u_i - u_j|
            loss += w[i] * (u[i] * w_before - wu_before) * 2.0f + w[i] * w[i] * ds[i] / 3.0f;
            grad_w[i] += scale * (2.0f * inter + 2.0f / 3.0f * w[i] * ds[i]);
            w_before += w[i];
            wu_before += w[i] * u[i];
        }
        loss_distortion += scale * loss;
    }

    // gradients of the final level's raw outputs (raw density and rgb logits, zero padding), one 16-byte row each
    float raw[kMaxSamplingIntervals];
    for (int i = 0; i < n; i++) raw[i] = bf16_bits_to_f32(a.nerf_outputs[kNerfOutputs * (ray * a.n + i)]);
    weights_backward_to_raw(grad_w, x, w, density, raw, t, n, direction_norm);
    for (int i = 0; i < n; i++) {
        uint16_t* grad = a.nerf_outputs_grad + kNerfOutputs * (ray * a.n + i);
        const float3 sg = sigmoids[i];
        const float color_scale = w[i] * (1.0f + 2.0f * kRgbPadding);
        const uint16_t g0 = f32_to_bf16_bits(grad_w[i]);
        const uint16_t g1 = f32_to_bf16_bits(color_scale * grad_rgb.x * sg.x * (1.0f - sg.x));
        const uint16_t g2 = f32_to_bf16_bits(color_scale * grad_rgb.y * sg.y * (1.0f - sg.y));
        const uint16_t g3 = f32_to_bf16_bits(color_scale * grad_rgb.z * sg.z * (1.0f - sg.z));
        const uint16_t zero = f32_to_bf16_bits(0.0f);
        if (a.vectors) {
            const uint32_t pad = static_cast<uint32_t>(zero) | static_cast<uint32_t>(zero) << 16;
            *reinterpret_cast<uint4*>(grad) = make_uint4(static_cast<uint32_t>(g0) | static_cast<uint32_t>(g1) << 16,
                                                         static_cast<uint32_t>(g2) | static_cast<uint32_t>(g3) << 16, pad, pad);
        } else {
            grad[0] = g0;
            grad[1] = g1;
            grad[2] = g2;
            grad[3] = g3;
            for (int c = 4; c < kNerfOutputs; c++) grad[c] = zero;
        }
    }

    // interlevel losses of the proposal levels against the blurred final weights
    for (int level = 0; level < a.proposals.n_levels; level++) {
        const int n_p = active ? a.proposals.n_intervals[level] : 0;
        const int64_t offset = ray * a.proposals.n_intervals[level];
        const float* s_p = a.proposals.sdist[level] + offset + ray;
        const float* t_p = a.proposals.tdist[level] + offset + ray;
        const float* w_p = a.proposals.weights[level] + offset;
        float grad_p[kMaxSamplingIntervals], raw_p[kMaxSamplingIntervals], density_p[kMaxSamplingIntervals], x_p[kMaxSamplingIntervals];
        if (n_p > 0) blur_and_resample(s_p, n_p + 1, s, w, n, a.proposals.interlevel_blur[level], grad_p);
        const float scale = a.proposals.interlevel_weight[level] * inv_n_rays / max(n_p, 1);
        for (int i = 0; i < n_p; i++) {
            const float r = fmaxf(grad_p[i] - w_p[i], 0.0f);
            const float denominator = w_p[i] + kSamplingEps;
            loss_interlevel += scale * r * r / denominator;
            grad_p[i] = scale * (-2.0f * r / denominator - r * r / (denominator * denominator));
            raw_p[i] = a.proposals.raw_density[level][offset + i];
            density_p[i] = activate_density(raw_p[i]);
            x_p[i] = density_p[i] * (t_p[i + 1] - t_p[i]) * direction_norm;
        }
        weights_backward_to_raw(grad_p, x_p, w_p, density_p, raw_p, t_p, n_p, direction_norm);
        for (int i = 0; i < n_p; i++) a.proposals.raw_density_grad[level][offset + i] = grad_p[i];
    }

    loss_data = warp_sum(loss_data);
    loss_mse = warp_sum(loss_mse);
    loss_interlevel = warp_sum(loss_interlevel);
    loss_distortion = warp_sum(loss_distortion);
    if (a.loss_sums != nullptr && threadIdx.x % 32 == 0) {
        atomicAdd(a.loss_sums, loss_data);
        atomicAdd(a.loss_sums + 1, loss_mse);
        atomicAdd(a.loss_sums + 2, loss_interlevel);
        atomicAdd(a.loss_sums + 3, loss_distortion);
    }
}

// inference: color, opacity and expected or median depth of every ray, written to its pixel (sampling_api.cu:379-424)
__global__ void __launch_bounds__(32) fz_composite_final_kernel(const __grid_constant__ CompositeFinalArgs a) {
    const int ray_idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (ray_idx >= a.n_rays) return;
    const int64_t ray = ray_idx;
    const int n = a.n;
    const float* t = a.tdist + ray * (n + 1);
    float density[kMaxSamplingIntervals], x[kMaxSamplingIntervals], w[kMaxSamplingIntervals];
    float3 sigmoids[kMaxSamplingIntervals];
    evaluate_final(a.nerf_outputs, t, n, norm3(make_float3(a.directions[3 * ray], a.directions[3 * ray + 1], a.directions[3 * ray + 2])), ray,
                   a.vectors, density, x, w, sigmoids);
    float3 color = make_float3(0.0f, 0.0f, 0.0f);
    float acc = 0.0f;
    for (int i = 0; i < n; i++) {
        const float3 c = padded_color(sigmoids[i]);
        color.x += w[i] * c.x;
        color.y += w[i] * c.y;
        color.z += w[i] * c.z;
        acc += w[i];
    }
    const float background_weight = fmaxf(1.0f - acc, 0.0f);
    const int64_t pixel = a.pixel_indices[ray];
    a.rgb[3 * pixel] = color.x + background_weight * a.background[0];
    a.rgb[3 * pixel + 1] = color.y + background_weight * a.background[1];
    a.rgb[3 * pixel + 2] = color.z + background_weight * a.background[2];
    if (a.alpha != nullptr) a.alpha[pixel] = acc;
    if (a.depth != nullptr) {
        if (a.use_median_depth) {
            // start of the interval where the normalized weights reach one half
            const float target = 0.5f * acc;
            float cw = 0.0f, median = t[n];
            for (int i = 0; i < n; i++) {
                cw += w[i];
                if (w[i] > 0.0f && cw >= target) {
                    median = t[i];
                    break;
                }
            }
            a.depth[pixel] = median;
        } else {
            // expected log distance, so that small weights far out do not dominate
            float weighted_log_t = 0.0f;
            for (int i = 0; i < n; i++) weighted_log_t += w[i] * logf(0.5f * (t[i] + t[i + 1]));
            a.depth[pixel] = fminf(fmaxf(expf(weighted_log_t / fmaxf(acc, kSamplingEps)), t[0]), t[n]);
        }
    }
}

}  // namespace zf

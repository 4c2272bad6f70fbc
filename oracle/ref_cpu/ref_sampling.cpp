// ref_sampling.cpp -- the reference's per-ray sampling functions compiled for the host (TEST INFRASTRUCTURE ONLY).
//
// Built by oracle/Makefile from the sources where they lie (-I to the reference's sampling/include and common/include
// directories) into oracle/_ref/libzf_ref_sampling_cpu.so. The per-ray math is the reference's own code
// (ray_ops.cuh: s_to_t, activate_density, sample_intervals, composite, composite_backward, power_ladder,
// blur_and_resample; random.cuh; zipnerf_config.h) with IEEE host math (libm) in place of the GPU's fast-math
// intrinsics. The kernel bodies that call it sit in sampling_api.cu next to libtorch wrappers, which do not build on the
// host, so they are restated here line by line with their citations (B/ = ZipNeRFCudaBackend/ZipNeRFCudaBackend/). It
// pins the C restatement (zf_step_oracle.c) and produces the golden vectors of tests/golden/make_golden_sampling.py.
#include "shim.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>

// ray_ops.cuh calls max / min on ints unqualified (CUDA built-ins)
inline int max(const int a, const int b) { return a > b ? a : b; }
inline int min(const int a, const int b) { return a < b ? a : b; }

#include "random.cuh"
#include "ray_ops.cuh"
#include "zipnerf_config.h"

namespace {

namespace zs = zipnerf::sampling;
namespace zr = zipnerf::random;

zs::RayWarp ray_warp(const float* w) { return {w[0], w[1], w[2], w[3], w[4], w[5], w[6]}; }

// __float2bfloat16: round to nearest even (NaN keeps a quiet NaN)
uint16_t bf16_bits(const float value) {
    uint32_t bits;
    std::memcpy(&bits, &value, sizeof(bits));
    if ((bits & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((bits >> 16) | 0x40u);
    bits += 0x7fffu + ((bits >> 16) & 1u);
    return static_cast<uint16_t>(bits >> 16);
}

// initialize_ray (B/sampling/src/sampling_api.cu:41-62)
void initialize_ray(const float3 d, const float jitter, const int direction_degree, const int n_samples, const zs::RayWarp& warp,
                    uint16_t* encoded, float* sdist, float* tdist) {
    const float inv_norm = 1.0f / std::sqrt(d.x * d.x + d.y * d.y + d.z * d.z);
    const float v[3] = {d.x * inv_norm, d.y * inv_norm, d.z * inv_norm};
    for (int i = 0; i < zipnerf::config::direction_block_width(direction_degree); i++) encoded[i] = bf16_bits(0.0f);
    for (int c = 0; c < 3; c++) {
        encoded[c] = bf16_bits(v[c]);
        for (int k = 0; k < direction_degree; k++) {
            const float x = std::scalbn(v[c], k);
            encoded[3 + 3 * k + c] = bf16_bits(std::sin(x));
            encoded[3 + 3 * (direction_degree + k) + c] = bf16_bits(std::cos(x));
        }
    }
    const float t_init[2] = {0.0f, 1.0f};
    const float w_init[1] = {1.0f};
    zs::sample_intervals(t_init, w_init, 1, 1.0f, n_samples, jitter, sdist);
    for (int i = 0; i <= n_samples; i++) tdist[i] = zs::s_to_t(sdist[i], warp);
}

float3 world_direction(const float* m, const float3 l) {
    return make_float3(m[0] * l.x + m[1] * l.y + m[2] * l.z, m[4] * l.x + m[5] * l.y + m[6] * l.z, m[8] * l.x + m[9] * l.y + m[10] * l.z);
}

float3 load3(const float* data, const int64_t i) { return make_float3(data[3 * i], data[3 * i + 1], data[3 * i + 2]); }

}  // namespace

#define REF_API extern "C" __attribute__((visibility("default")))

REF_API int ref_cpu_direction_block_width(const int degree) { return static_cast<int>(zipnerf::config::direction_block_width(degree)); }

// initialize_rays_kernel (sampling_api.cu:150-166)
REF_API void ref_cpu_initialize_rays(const int64_t seed, const float* directions, const int n_rays, const int degree, const int n_samples,
                                     const float* warp, uint16_t* encoded, float* sdist, float* tdist) {
    const int width = ref_cpu_direction_block_width(degree);
    for (int ray = 0; ray < n_rays; ray++) {
        const float jitter = seed >= 0 ? zr::uniform(seed, zr::jitter, ray) : -1.0f;
        initialize_ray(load3(directions, ray), jitter, degree, n_samples, ray_warp(warp), encoded + static_cast<int64_t>(ray) * width,
                       sdist + static_cast<int64_t>(ray) * (n_samples + 1), tdist + static_cast<int64_t>(ray) * (n_samples + 1));
    }
}

// view_rays_kernel (sampling_api.cu:120-147)
REF_API void ref_cpu_view_rays(const int64_t* pixel_indices, const int n_rays, const float* local_directions, const float* c2w, const float radius,
                               const int degree, const int n_samples, const float* warp, float* origins, float* directions, float* radii,
                               uint16_t* encoded, float* sdist, float* tdist) {
    const int width = ref_cpu_direction_block_width(degree);
    for (int ray = 0; ray < n_rays; ray++) {
        const float3 d = world_direction(c2w, load3(local_directions, pixel_indices[ray]));
        origins[3 * ray] = c2w[3];
        origins[3 * ray + 1] = c2w[7];
        origins[3 * ray + 2] = c2w[11];
        directions[3 * ray] = d.x;
        directions[3 * ray + 1] = d.y;
        directions[3 * ray + 2] = d.z;
        radii[ray] = radius;
        initialize_ray(d, -1.0f, degree, n_samples, ray_warp(warp), encoded + static_cast<int64_t>(ray) * width,
                       sdist + static_cast<int64_t>(ray) * (n_samples + 1), tdist + static_cast<int64_t>(ray) * (n_samples + 1));
    }
}

// generate_rays_kernel (sampling_api.cu:72-117)
REF_API void ref_cpu_generate_rays(const int64_t seed, const int n_rays, const int64_t* view_offsets, const int n_views, const int* view_cameras,
                                   const int64_t* camera_offsets, const float* local_directions, const float* c2w, const float* camera_radii,
                                   const uint8_t* pool_rgb, const int64_t n_pixels, const int degree, const int n_samples, const float* warp,
                                   float* origins, float* directions, float* radii, float* rgb, uint16_t* encoded, float* sdist, float* tdist) {
    const int width = ref_cpu_direction_block_width(degree);
    const uint64_t s = static_cast<uint64_t>(seed);
    for (int ray = 0; ray < n_rays; ray++) {
        const int64_t pixel = static_cast<int64_t>(zr::uniform_int(s, zr::pixel, ray, n_pixels));
        int lo = 0, hi = n_views;
        while (hi - lo > 1) {
            const int mid = (lo + hi) / 2;
            if (view_offsets[mid] <= pixel) lo = mid;
            else hi = mid;
        }
        const int camera = view_cameras[lo];
        const float3 local = load3(local_directions, camera_offsets[camera] + pixel - view_offsets[lo]);
        const float* m = c2w + 12 * lo;
        const float3 d = world_direction(m, local);
        origins[3 * ray] = m[3];
        origins[3 * ray + 1] = m[7];
        origins[3 * ray + 2] = m[11];
        directions[3 * ray] = d.x;
        directions[3 * ray + 1] = d.y;
        directions[3 * ray + 2] = d.z;
        radii[ray] = camera_radii[camera];
        for (int c = 0; c < 3; c++) rgb[3 * ray + c] = pool_rgb[3 * pixel + c] / 255.0f;
        initialize_ray(d, zr::uniform(s, zr::jitter, ray), degree, n_samples, ray_warp(warp), encoded + static_cast<int64_t>(ray) * width,
                       sdist + static_cast<int64_t>(ray) * (n_samples + 1), tdist + static_cast<int64_t>(ray) * (n_samples + 1));
    }
}

// sample_uniforms_kernel (sampling_api.cu:168-172)
REF_API void ref_cpu_sample_uniforms(const int64_t seed, const int64_t stream, const int64_t n, float* values) {
    for (int64_t i = 0; i < n; i++) values[i] = zr::uniform(static_cast<uint64_t>(seed), static_cast<uint64_t>(stream), static_cast<uint64_t>(i));
}

// composite_and_resample_kernel (sampling_api.cu:174-196)
REF_API void ref_cpu_composite_and_resample(const float* raw_density, const float* sdist, const float* tdist, const float* directions, const int n_rays,
                                            const int n_intervals, const float anneal, const int n_samples, const int64_t seed, const int next_level,
                                            const float* warp, float* weights, float* sdist_next, float* tdist_next) {
    for (int ray = 0; ray < n_rays; ray++) {
        const float* t = tdist + static_cast<int64_t>(ray) * (n_intervals + 1);
        float density[zs::max_intervals];
        for (int i = 0; i < n_intervals; i++) density[i] = zs::activate_density(raw_density[static_cast<int64_t>(ray) * n_intervals + i]);
        float* w = weights + static_cast<int64_t>(ray) * n_intervals;
        const float3 d = load3(directions, ray);
        zs::composite(density, t, n_intervals, std::sqrt(d.x * d.x + d.y * d.y + d.z * d.z), w, nullptr);
        float* s_next = sdist_next + static_cast<int64_t>(ray) * (n_samples + 1);
        const float jitter = seed >= 0 ? zr::uniform(seed, zr::jitter + next_level, ray) : -1.0f;
        zs::sample_intervals(sdist + static_cast<int64_t>(ray) * (n_intervals + 1), w, n_intervals, anneal, n_samples, jitter, s_next);
        for (int i = 0; i <= n_samples; i++) tdist_next[static_cast<int64_t>(ray) * (n_samples + 1) + i] = zs::s_to_t(s_next[i], ray_warp(warp));
    }
}

// ---------------------------------------------------------------------------------------------------------------------
// the final level (sampling_api.cu:203-424): the kernel bodies restated around the reference's own compositing,
// composite backward, power ladder and blur-and-resample functions

namespace {

constexpr int n_nerf_outputs = 8;     // sampling_api.cu:15
constexpr float rgb_padding = 0.001f;  // sampling_api.cu:14

float bf16_value(const uint16_t bits) {
    const uint32_t word = static_cast<uint32_t>(bits) << 16;
    float value;
    std::memcpy(&value, &word, sizeof(value));
    return value;
}

// evaluate_final (sampling_api.cu:203-220)
void evaluate_final(const uint16_t* outputs, const float* t, const int n, const float direction_norm, float* density, float* x, float* w,
                    float3* colors, float3* sigmoids) {
    for (int i = 0; i < n; i++) {
        const uint16_t* raw = outputs + n_nerf_outputs * i;
        const float r0 = bf16_value(raw[0]), r1 = bf16_value(raw[1]), r2 = bf16_value(raw[2]), r3 = bf16_value(raw[3]);
        const bool valid = std::isfinite(r0) && std::isfinite(r1) && std::isfinite(r2) && std::isfinite(r3);
        density[i] = valid ? zs::activate_density(r0) : 0.0f;
        const float3 s = valid ? make_float3(1.0f / (1.0f + std::exp(-r1)), 1.0f / (1.0f + std::exp(-r2)), 1.0f / (1.0f + std::exp(-r3)))
                               : make_float3(0.5f, 0.5f, 0.5f);
        sigmoids[i] = s;
        colors[i] = make_float3(s.x * (1.0f + 2.0f * rgb_padding) - rgb_padding, s.y * (1.0f + 2.0f * rgb_padding) - rgb_padding,
                                s.z * (1.0f + 2.0f * rgb_padding) - rgb_padding);
    }
    zs::composite(density, t, n, direction_norm, w, x);
}

// weights_backward_to_raw (sampling_api.cu:223-229)
void weights_backward_to_raw(float* grad, const float* x, const float* w, const float* density, const float* raw, const float* t, const int n,
                             const float direction_norm) {
    zs::composite_backward(grad, x, w, n);
    for (int i = 0; i < n; i++) {
        const bool clipped = raw[i] - 1.0f > zs::max_density_exponent;
        grad[i] = clipped ? 0.0f : grad[i] * (t[i + 1] - t[i]) * direction_norm * density[i];
    }
}

}  // namespace

// train_final_kernel (sampling_api.cu:231-376), one ray after the other; loss_sums (double [4]) += the batch's sums
REF_API void ref_cpu_train_final(const uint16_t* outputs, const float* sdist, const float* tdist, const int n_rays, const int n, const int n_levels,
                                 const int* n_p, const float* const* raw_p, const float* const* sdist_p, const float* const* tdist_p,
                                 const float* const* weights_p, float* const* grad_p_out, const float* interlevel_weights, const float* interlevel_blurs,
                                 const float* directions, const uint64_t seed, const float* rgb_target, const float charbonnier_padding,
                                 const float distortion_weight, const float distortion_power, const float distortion_premult, uint16_t* outputs_grad,
                                 double* loss_sums) {
    const float inv_n_rays = 1.0f / n_rays;
    for (int ray = 0; ray < n_rays; ray++) {
        const float* t = tdist + static_cast<int64_t>(ray) * (n + 1);
        const float* s = sdist + static_cast<int64_t>(ray) * (n + 1);
        const float3 d = load3(directions, ray);
        const float direction_norm = std::sqrt(d.x * d.x + d.y * d.y + d.z * d.z);
        float density[zs::max_intervals], x[zs::max_intervals], w[zs::max_intervals], grad_w[zs::max_intervals];
        float3 colors[zs::max_intervals], sigmoids[zs::max_intervals];
        evaluate_final(outputs + static_cast<int64_t>(n_nerf_outputs) * ray * n, t, n, direction_norm, density, x, w, colors, sigmoids);
        float3 rgb = make_float3(0.0f, 0.0f, 0.0f);
        float acc = 0.0f;
        for (int i = 0; i < n; i++) {
            rgb.x += w[i] * colors[i].x;
            rgb.y += w[i] * colors[i].y;
            rgb.z += w[i] * colors[i].z;
            acc += w[i];
        }
        const float3 bg = make_float3(zr::uniform(seed, zr::background, 3 * ray), zr::uniform(seed, zr::background, 3 * ray + 1),
                                      zr::uniform(seed, zr::background, 3 * ray + 2));
        const float background_weight = std::fmax(1.0f - acc, 0.0f);
        const float3 target = load3(rgb_target, ray);
        const float r[3] = {rgb.x + background_weight * bg.x - target.x, rgb.y + background_weight * bg.y - target.y,
                            rgb.z + background_weight * bg.z - target.z};
        float g[3];
        for (int c = 0; c < 3; c++) {
            const float q = std::sqrt(r[c] * r[c] + charbonnier_padding * charbonnier_padding);
            loss_sums[0] += q * inv_n_rays / 3.0f;
            loss_sums[1] += r[c] * r[c] * inv_n_rays / 3.0f;
            g[c] = r[c] / q * inv_n_rays / 3.0f;
        }
        const float3 grad_rgb = make_float3(g[0], g[1], g[2]);
        const float grad_background = 1.0f - acc >= 0.0f ? grad_rgb.x * bg.x + grad_rgb.y * bg.y + grad_rgb.z * bg.z : 0.0f;
        for (int i = 0; i < n; i++) grad_w[i] = grad_rgb.x * colors[i].x + grad_rgb.y * colors[i].y + grad_rgb.z * colors[i].z - grad_background;
        float u[zs::max_intervals], ds[zs::max_intervals];
        float previous = zs::power_ladder(t[0], distortion_power, distortion_premult);
        float w_total = 0.0f, wu_total = 0.0f;
        for (int i = 0; i < n; i++) {
            const float next = zs::power_ladder(t[i + 1], distortion_power, distortion_premult);
            u[i] = 0.5f * (previous + next);
            ds[i] = next - previous;
            previous = next;
            w_total += w[i];
            wu_total += w[i] * u[i];
        }
        const float scale = distortion_weight * inv_n_rays;
        float w_before = 0.0f, wu_before = 0.0f, loss = 0.0f;
        for (int i = 0; i < n; i++) {
            const float w_after = w_total - w_before - w[i], wu_after = wu_total - wu_before - w[i] * u[i];
            const float inter = u[i] * w_before - wu_before + wu_after - u[i] * w_after;
            loss += w[i] * (u[i] * w_before - wu_before) * 2.0f + w[i] * w[i] * ds[i] / 3.0f;
            grad_w[i] += scale * (2.0f * inter + 2.0f / 3.0f * w[i] * ds[i]);
            w_before += w[i];
            wu_before += w[i] * u[i];
        }
        loss_sums[3] += scale * loss;
        float raw[zs::max_intervals];
        for (int i = 0; i < n; i++) raw[i] = bf16_value(outputs[n_nerf_outputs * (static_cast<int64_t>(ray) * n + i)]);
        weights_backward_to_raw(grad_w, x, w, density, raw, t, n, direction_norm);
        for (int i = 0; i < n; i++) {
            uint16_t* grad = outputs_grad + n_nerf_outputs * (static_cast<int64_t>(ray) * n + i);
            const float3 sg = sigmoids[i];
            const float color_scale = w[i] * (1.0f + 2.0f * rgb_padding);
            grad[0] = bf16_bits(grad_w[i]);
            grad[1] = bf16_bits(color_scale * grad_rgb.x * sg.x * (1.0f - sg.x));
            grad[2] = bf16_bits(color_scale * grad_rgb.y * sg.y * (1.0f - sg.y));
            grad[3] = bf16_bits(color_scale * grad_rgb.z * sg.z * (1.0f - sg.z));
            for (int c = 4; c < n_nerf_outputs; c++) grad[c] = bf16_bits(0.0f);
        }
        for (int level = 0; level < n_levels; level++) {
            const int m = n_p[level];
            const int64_t offset = static_cast<int64_t>(ray) * m;
            const float* s_p = sdist_p[level] + offset + ray;
            const float* t_p = tdist_p[level] + offset + ray;
            const float* w_p = weights_p[level] + offset;
            float grad_p[zs::max_intervals], raw_lp[zs::max_intervals], density_p[zs::max_intervals], x_p[zs::max_intervals];
            zs::blur_and_resample(s_p, m + 1, s, w, n, interlevel_blurs[level], grad_p);
            const float lscale = interlevel_weights[level] * inv_n_rays / std::max(m, 1);
            for (int i = 0; i < m; i++) {
                const float rr = std::fmax(grad_p[i] - w_p[i], 0.0f);
                const float denominator = w_p[i] + zs::eps;
                loss_sums[2] += lscale * rr * rr / denominator;
                grad_p[i] = lscale * (-2.0f * rr / denominator - rr * rr / (denominator * denominator));
                raw_lp[i] = raw_p[level][offset + i];
                density_p[i] = zs::activate_density(raw_lp[i]);
                x_p[i] = density_p[i] * (t_p[i + 1] - t_p[i]) * direction_norm;
            }
            weights_backward_to_raw(grad_p, x_p, w_p, density_p, raw_lp, t_p, m, direction_norm);
            for (int i = 0; i < m; i++) grad_p_out[level][offset + i] = grad_p[i];
        }
    }
}

// composite_final_kernel (sampling_api.cu:379-424)
REF_API void ref_cpu_composite_final(const uint16_t* outputs, const float* tdist, const float* directions, const float* background,
                                     const int64_t* pixel_indices, const int n_rays, const int n, float* rgb, float* alpha, float* depth,
                                     const int use_median_depth) {
    for (int ray = 0; ray < n_rays; ray++) {
        const float* t = tdist + static_cast<int64_t>(ray) * (n + 1);
        float density[zs::max_intervals], x[zs::max_intervals], w[zs::max_intervals];
        float3 colors[zs::max_intervals], sigmoids[zs::max_intervals];
        const float3 d = load3(directions, ray);
        evaluate_final(outputs + static_cast<int64_t>(n_nerf_outputs) * ray * n, t, n, std::sqrt(d.x * d.x + d.y * d.y + d.z * d.z), density, x, w,
                       colors, sigmoids);
        float3 color = make_float3(0.0f, 0.0f, 0.0f);
        float acc = 0.0f;
        for (int i = 0; i < n; i++) {
            color.x += w[i] * colors[i].x;
            color.y += w[i] * colors[i].y;
            color.z += w[i] * colors[i].z;
            acc += w[i];
        }
        const float background_weight = std::fmax(1.0f - acc, 0.0f);
        const int64_t pixel = pixel_indices[ray];
        rgb[3 * pixel] = color.x + background_weight * background[0];
        rgb[3 * pixel + 1] = color.y + background_weight * background[1];
        rgb[3 * pixel + 2] = color.z + background_weight * background[2];
        if (alpha != nullptr) alpha[pixel] = acc;
        if (depth == nullptr) continue;
        if (use_median_depth) {
            const float target = 0.5f * acc;
            float cw = 0.0f, median = t[n];
            for (int i = 0; i < n; i++) {
                cw += w[i];
                if (w[i] > 0.0f && cw >= target) {
                    median = t[i];
                    break;
                }
            }
            depth[pixel] = median;
        } else {
            float weighted_log_t = 0.0f;
            for (int i = 0; i < n; i++) weighted_log_t += w[i] * std::log(0.5f * (t[i] + t[i + 1]));
            depth[pixel] = std::fmin(std::fmax(std::exp(weighted_log_t / std::fmax(acc, zs::eps)), t[0]), t[n]);
        }
    }
}

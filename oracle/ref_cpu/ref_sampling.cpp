// ref_sampling.cpp -- the reference's per-ray sampling functions compiled for the host (TEST INFRASTRUCTURE ONLY).
//
// Built by oracle/Makefile from the sources where they lie (-I to the reference's sampling/include and common/include
// directories) into oracle/_ref/libzf_ref_sampling_cpu.so. The per-ray math is the reference's own code
// (ray_ops.cuh: s_to_t, activate_density, sample_intervals, composite; random.cuh; zipnerf_config.h) with IEEE host
// math (libm) in place of the GPU's fast-math intrinsics. The kernel bodies that call it sit in sampling_api.cu next to
// libtorch wrappers, which do not build on the host, so they are restated here line by line with their citations
// (B/ = ZipNeRFCudaBackend/ZipNeRFCudaBackend/). It pins the C restatement (zf_step_oracle.c) and produces the golden
// vectors of tests/golden/make_golden.py.
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

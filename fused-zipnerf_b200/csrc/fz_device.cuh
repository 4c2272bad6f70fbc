// fz_device.cuh -- device-side math of the multisampled hash-grid featurization (sm_100a).
//
// Per interval of a ray this places six hexagonal multisamples in the conical frustum, contracts them into [0,1]^3,
// derives per-level erf downweighting from the multisample radius, and visits the trilinear corners of every grid
// level, with multisamples that fall into the same cell merged into one group of eight corners. The expressions follow
// the reference's featurize_common.cuh operation for operation (same operand order, same fast-math intrinsics), so
// the cell indices, hash rows and weights are bit-identical to the reference kernels:
//   interval setup          featurize_common.cuh:56-98
//   multisample/contraction featurize_common.cuh:101-117
//   level weighting (erf)   featurize_common.cuh:45-47, 202-204
//   corner visit + merging  featurize_common.cuh:123-173
//   counter-based RNG       common/include/random.cuh:15-29
// Kernels are compiled with --use_fast_math, like the reference's runtime compilation (rtc_kernel.cu:49).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace zf {

constexpr int kMaxLevels = 16;
constexpr int kMaxFeatures = 4;
constexpr uint32_t kMultisamples = 6;
constexpr float kGridBboxSize = 4.0f;  // grids cover the contracted space [-2, 2]^3
constexpr float kMultisampleScale = 0.5f;
constexpr uint32_t kHashPrimeY = 19349663u;
constexpr uint32_t kHashPrimeZ = 83492791u;
constexpr float kTiny = 1.17549435e-38f;
constexpr float kPreconditionScaling = 10.0f;
constexpr float kFeatureScale = kPreconditionScaling / kMultisamples;
constexpr unsigned long long kPatternStreamBase = 16ull;

// Grid layout of one featurizer, passed to every kernel by value (kernel parameters live in the constant bank; the
// per-level fields are read with the loop's level as an index).
struct GridParams {
    uint32_t n_levels;
    uint32_t n_features;
    uint32_t size[kMaxLevels];
    uint32_t entries[kMaxLevels];
    uint32_t offset[kMaxLevels + 1];
    uint32_t hashed_mask;  // bit l: level l is hashed (size^3 > entries)
    uint32_t pow2_mask;    // bit l: entries of level l is a power of two (hash modulo is a mask)
    uint32_t n_fp32_levels;  // leading levels whose backward gradient is fp32
    unsigned long long pattern_stream;
};

// Per-ray inputs shared by all kernels.
struct RayInputs {
    const float* origins;     // [n_rays, 3]
    const float* directions;  // [n_rays, 3]
    const float* radii;       // [n_rays]
    const float* tdist;       // [n_rays, n_intervals + 1]
    long long pattern_seed;   // < 0: deterministic alternating patterns
    unsigned long long sample_offset;  // added to the sample index of the pattern random numbers (batch shards)
    uint32_t n_intervals;
    uint32_t n_samples;       // n_rays * n_intervals
};

// ---------------------------------------------------------------------------------------------------------------------
// small vector helpers (the same operand order as the reference's featurize_common.cuh:38-43)

__device__ __forceinline__ float3 add3(const float3& a, const float3& b) { return make_float3(a.x + b.x, a.y + b.y, a.z + b.z); }
__device__ __forceinline__ float3 mul3(const float a, const float3& b) { return make_float3(a * b.x, a * b.y, a * b.z); }
__device__ __forceinline__ float dot3(const float3& a, const float3& b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
__device__ __forceinline__ float3 cross3(const float3& a, const float3& b) {
    return make_float3(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x);
}
__device__ __forceinline__ float3 normalize3(const float3& a) { return mul3(rsqrtf(dot3(a, a)), a); }

// ---------------------------------------------------------------------------------------------------------------------
// counter-based random numbers: splitmix64 of (seed, stream, index)

__device__ __forceinline__ unsigned long long splitmix64(unsigned long long x) {
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

__device__ __forceinline__ float rng_uniform(const unsigned long long seed, const unsigned long long stream, const unsigned long long index) {
    const unsigned long long h = splitmix64(splitmix64(seed ^ (stream << 56)) ^ index);
    return static_cast<float>(h >> 40) * (1.0f / 16777216.0f);
}

// erf approximation sign(x) sqrt(1 - exp(-4 x^2 / pi))
__device__ __forceinline__ float approx_erf(const float x) {
    return copysignf(sqrtf(-expm1f(-(4.0f / 3.14159265358979f) * x * x)), x);
}

// ---------------------------------------------------------------------------------------------------------------------
// conical frustum of one interval

struct Frustum {
    float3 origin, direction, axis1, axis2;
    float radius, t0, ratio, base, root, rotation;
    bool flip;
};

__device__ __forceinline__ float3 load_float3(const float* p, const uint32_t i) {
    return make_float3(__ldg(p + 3 * i), __ldg(p + 3 * i + 1), __ldg(p + 3 * i + 2));
}

__device__ __forceinline__ Frustum setup_frustum(const RayInputs& in, const unsigned long long pattern_stream, const uint32_t sample) {
    Frustum fr;
    const uint32_t ray = sample / in.n_intervals;
    const uint32_t interval = sample - ray * in.n_intervals;
    fr.origin = load_float3(in.origins, ray);
    fr.direction = load_float3(in.directions, ray);
    fr.radius = __ldg(in.radii + ray);
    const float3 d = fr.direction;
    float3 c = cross3(d, make_float3(0.0f, 0.0f, 1.0f));
    constexpr float eps = 1.1920929e-07f;
    if (fabsf(c.x) < eps && fabsf(c.y) < eps && fabsf(c.z) < eps) c = cross3(d, make_float3(1.0f, 1.0f, 1.0f));
    fr.axis1 = normalize3(c);
    fr.axis2 = normalize3(cross3(d, c));
    const float* t = in.tdist + static_cast<size_t>(ray) * (in.n_intervals + 1) + interval;
    const float t0 = __ldg(t), t1 = __ldg(t + 1);
    const float s = 0.5f * (t0 + t1);
    const float h = 0.5f * (t1 - t0);
    const float denominator = h * h + 3.0f * s * s;
    fr.t0 = t0;
    fr.ratio = fabsf(denominator) < kTiny ? 0.0f : h / denominator;
    fr.base = t1 * t1 + 2.0f * s * s;
    const float q = h * h - s * s;
    fr.root = sqrtf(fmaxf(q * q + 4.0f * s * s * s * s, 0.0f));
    if (in.pattern_seed >= 0) {
        const unsigned long long seed = static_cast<unsigned long long>(in.pattern_seed);
        const unsigned long long index = in.sample_offset + sample;
        fr.flip = rng_uniform(seed, pattern_stream, 2ull * index) < 0.5f;
        fr.rotation = 2.0f * 3.14159265358979f * rng_uniform(seed, pattern_stream, 2ull * index + 1);
    }
    else {
        fr.flip = interval % 2 == 1;
        fr.rotation = fr.flip ? 3.14159265358979f / 6.0f : 0.0f;
    }
    return fr;
}

// contracted position of multisample j in [0,1]^3 and its radius in the same units; contracted = |p|^2 > 1
__device__ __forceinline__ void multisample(const Frustum& fr, const uint32_t j, float3& x, float& scale, bool* contracted = nullptr) {
    constexpr float pattern[kMultisamples] = {0.0f, 2.0f, 4.0f, 3.0f, 5.0f, 1.0f};
    const float theta = (3.14159265358979f / 3.0f) * pattern[fr.flip ? kMultisamples - 1 - j : j] + fr.rotation;
    const float cz = fr.t0 + fr.ratio * (fr.base + (3.0f / sqrtf(7.0f)) * (j * 0.4f - 1.0f) * fr.root);
    const float perp = sqrtf(0.5f) * fr.radius * cz;
    float sin_theta, cos_theta;
    sincosf(theta, &sin_theta, &cos_theta);
    const float3 p = add3(add3(add3(fr.origin, mul3(perp * cos_theta, fr.axis1)), mul3(perp * sin_theta, fr.axis2)), mul3(cz, fr.direction));
    const float dot_p = dot3(p, p);
    if (contracted != nullptr) *contracted = dot_p > 1.0f;
    const float norm_sq = fmaxf(dot_p, 1.0f);
    const float norm = sqrtf(norm_sq);
    const float isoscale = expf((2.0f / 3.0f) * logf(2.0f * norm - 1.0f) - logf(norm_sq));
    const float contraction = (2.0f * norm - 1.0f) / norm_sq;
    x = add3(mul3(1.0f / kGridBboxSize, mul3(contraction, p)), make_float3(0.5f, 0.5f, 0.5f));
    scale = kMultisampleScale * perp * isoscale * (1.0f / kGridBboxSize);
}

// Arguments from which approx_erf is exactly 1.0f in this build: expm1f of the argument's square term is exactly -1
// and the square root of 1 is 1. zf_check_erf_saturation verifies that claim over every float in [threshold, +inf)
// on the device (the GPU tests run it); below the threshold the erf is evaluated as the reference does.
#ifndef ZF_ERF_SATURATION
#define ZF_ERF_SATURATION 3.66f
#endif
constexpr float kErfSaturation = ZF_ERF_SATURATION;

__device__ __forceinline__ float level_weighting(const uint32_t size, const float scale) {
    const float x = 1.0f / (sqrtf(8.0f) * scale * size);
    // coarse levels of small multisamples (the common case) saturate: skip the expm1f / sqrtf of approx_erf
    if (x >= kErfSaturation) return 1.0f;
    return approx_erf(x);
}

// table rows of the 8 corners of a cell (corner bits x, y, z = 4, 2, 1; level offset included) from per-axis terms:
// hashed levels xor the coordinate terms x, y * prime_y, z * prime_z (the +1 terms by adding the prime, modulo 2^32 as
// the product); dense levels add 1, n, n^2 to the cell's index and zero the weight of corners outside the grid
// (featurize_common.cuh:154-171: the same integers as the reference's per-corner hash or index).
__device__ __forceinline__ void cell_rows(const GridParams& gp, const uint32_t level, const int cx, const int cy, const int cz, uint32_t (&rows)[8],
                                          float (&weights)[8]) {
    const uint32_t base = gp.offset[level];
    if (gp.hashed_mask & (1u << level)) {
        const uint32_t hx[2] = {static_cast<uint32_t>(cx), static_cast<uint32_t>(cx) + 1u};
        const uint32_t y0 = static_cast<uint32_t>(cy) * kHashPrimeY, z0 = static_cast<uint32_t>(cz) * kHashPrimeZ;
        const uint32_t hy[2] = {y0, y0 + kHashPrimeY}, hz[2] = {z0, z0 + kHashPrimeZ};
        const uint32_t entries = gp.entries[level];
        const bool pow2 = (gp.pow2_mask >> level) & 1u;
        #pragma unroll
        for (uint32_t corner = 0; corner < 8; corner++) {
            const uint32_t h = hx[(corner >> 2) & 1u] ^ hy[(corner >> 1) & 1u] ^ hz[corner & 1u];
            rows[corner] = base + (pow2 ? (h & (entries - 1u)) : (h % entries));
        }
    }
    else {
        const int n = static_cast<int>(gp.size[level]);
        const bool vx[2] = {cx >= 0 && cx < n, cx + 1 >= 0 && cx + 1 < n};
        const bool vy[2] = {cy >= 0 && cy < n, cy + 1 >= 0 && cy + 1 < n};
        const bool vz[2] = {cz >= 0 && cz < n, cz + 1 >= 0 && cz + 1 < n};
        const int index = cx + n * (cy + n * cz);
        #pragma unroll
        for (uint32_t corner = 0; corner < 8; corner++) {
            const int dx = static_cast<int>((corner >> 2) & 1u), dy = static_cast<int>((corner >> 1) & 1u), dz = static_cast<int>(corner & 1u);
            const bool valid = vx[dx] && vy[dy] && vz[dz];
            if (!valid) weights[corner] = 0.0f;
            rows[corner] = base + (valid ? static_cast<uint32_t>(index + dx + n * (dy + n * dz)) : 0u);
        }
    }
}

// cell and fractional position of a contracted coordinate on a level of the given size (featurize_common.cuh:127-131)
__device__ __forceinline__ void level_cell(const float x, const uint32_t size, int& cell, float& frac) {
    const float p = x * size - 0.5f;
    const float g = floorf(p);
    cell = static_cast<int>(g);
    frac = p - g;
}

template <typename Visitor>
__device__ __forceinline__ void visit_level(const GridParams& gp, const uint32_t level, const float3* x, const float* weighting, Visitor& visitor) {
    const uint32_t size = gp.size[level];
    int cx[kMultisamples], cy[kMultisamples], cz[kMultisamples];
    float fx[kMultisamples], fy[kMultisamples], fz[kMultisamples];
    #pragma unroll
    for (uint32_t j = 0; j < kMultisamples; j++) {
        level_cell(x[j].x, size, cx[j], fx[j]);
        level_cell(x[j].y, size, cy[j], fy[j]);
        level_cell(x[j].z, size, cz[j], fz[j]);
    }
    uint32_t remaining = (1u << kMultisamples) - 1u;
    while (remaining != 0u) {
        // the group of the lowest unvisited multisample (its leader): the leader's values by selection
        const uint32_t leader = __ffs(remaining) - 1u;
        int lx = cx[0], ly = cy[0], lz = cz[0];
        float lfx = fx[0], lfy = fy[0], lfz = fz[0], lw = weighting[0];
        #pragma unroll
        for (uint32_t j = 1; j < kMultisamples; j++) {
            if (leader == j) {
                lx = cx[j];
                ly = cy[j];
                lz = cz[j];
                lfx = fx[j];
                lfy = fy[j];
                lfz = fz[j];
                lw = weighting[j];
            }
        }
        uint32_t members = 0u;
        #pragma unroll
        for (uint32_t k = 0; k < kMultisamples; k++) {
            if (((remaining >> k) & 1u) && cx[k] == lx && cy[k] == ly && cz[k] == lz) members |= 1u << k;
        }
        remaining &= ~members;
        // corner weights: the leader's trilinear weights, then the other members' in multisample order (most groups of
        // the fine levels are single multisamples, which skip the member loop)
        float corner_weights[8];
        #pragma unroll
        for (uint32_t corner = 0; corner < 8; corner++) {
            const float wx = corner & 4u ? lfx : 1.0f - lfx;
            const float wy = corner & 2u ? lfy : 1.0f - lfy;
            const float wz = corner & 1u ? lfz : 1.0f - lfz;
            corner_weights[corner] = __fmaf_rn(lw, __fmul_rn(__fmul_rn(wx, wy), wz), 0.0f);
        }
        const uint32_t others = members & ~(1u << leader);
        if (others != 0u) {
            #pragma unroll
            for (uint32_t k = 1; k < kMultisamples; k++) {
                if (!((others >> k) & 1u)) continue;
                #pragma unroll
                for (uint32_t corner = 0; corner < 8; corner++) {
                    const float wx = corner & 4u ? fx[k] : 1.0f - fx[k];
                    const float wy = corner & 2u ? fy[k] : 1.0f - fy[k];
                    const float wz = corner & 1u ? fz[k] : 1.0f - fz[k];
                    corner_weights[corner] = __fmaf_rn(weighting[k], __fmul_rn(__fmul_rn(wx, wy), wz), corner_weights[corner]);
                }
            }
        }
        uint32_t rows[8];
        cell_rows(gp, level, lx, ly, lz, rows, corner_weights);
        #pragma unroll
        for (uint32_t corner = 0; corner < 8; corner++) visitor(rows[corner], corner_weights[corner]);
    }
}

// ---------------------------------------------------------------------------------------------------------------------
// numeric conversions (round to nearest even, as the reference's cvt.rn)

__device__ __forceinline__ uint16_t f32_to_bf16_bits(const float v) {
    uint16_t r;
    asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(v));
    return r;
}

__device__ __forceinline__ float bf16_bits_to_f32(const uint16_t v) { return __uint_as_float(static_cast<uint32_t>(v) << 16); }

// packs (lo, hi) into one f16x2 word, lo at the lower address
__device__ __forceinline__ uint32_t pack_half2(const float lo, const float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ uint16_t f32_to_half_bits(const float v) {
    uint16_t r;
    asm("cvt.rn.f16.f32 %0, %1;" : "=h"(r) : "f"(v));
    return r;
}

}  // namespace zf

/*
 * zf_oracle.c -- CPU restatement of the Fused Zip-NeRF featurization (TEST INFRASTRUCTURE ONLY; see zf_oracle.h).
 *
 * Every expression keeps the operand order of the reference so that, compiled without floating-point contraction
 * (-ffp-contract=off), it reproduces the reference's featurize_common.cuh compiled for the host bit for bit. The
 * product CUDA kernels differ from it only by the GPU's fast-math intrinsics and fused multiply-adds, which the
 * parity tests bound by tolerances.
 */
#define _GNU_SOURCE
#include "zf_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* constants of featurize_common.cuh:13-21 and zipnerf_config.h:8-15 */
#define N_MULTISAMPLES 6
static const float grid_bbox_size = 4.0f;
static const float multisample_scale = 0.5f;
static const uint32_t hash_prime_y = 19349663u;
static const uint32_t hash_prime_z = 83492791u;
static const float tiny = 1.17549435e-38f;
static const float precondition_scaling = 10.0f;
static const int64_t min_half_grad_entries = (int64_t)1 << 20;
static const uint64_t pattern_stream_base = 16;

typedef struct { float x, y, z; } vec3;

static inline vec3 v3(float x, float y, float z) { vec3 r = {x, y, z}; return r; }
static inline vec3 v3_add(vec3 a, vec3 b) { return v3(a.x + b.x, a.y + b.y, a.z + b.z); }
static inline vec3 v3_scale(float a, vec3 b) { return v3(a * b.x, a * b.y, a * b.z); }
static inline float v3_dot(vec3 a, vec3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
static inline vec3 v3_cross(vec3 a, vec3 b) { return v3(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x); }
/* rsqrtf(x) * a of featurize_common.cuh:43, with the reciprocal square root as 1 / sqrtf */
static inline vec3 v3_normalize(vec3 a) { return v3_scale(1.0f / sqrtf(v3_dot(a, a)), a); }

/* random.cuh:15-29 */
static inline uint64_t splitmix64(uint64_t x) {
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}
static inline uint64_t rng_hash(uint64_t seed, uint64_t stream, uint64_t index) { return splitmix64(splitmix64(seed ^ (stream << 56)) ^ index); }
static inline float rng_uniform(uint64_t seed, uint64_t stream, uint64_t index) { return (float)(rng_hash(seed, stream, index) >> 40) * (1.0f / 16777216.0f); }

/* featurize_common.cuh:45-47 */
static inline float approx_erf(float x) { return copysignf(sqrtf(-expm1f(-(4.0f / 3.14159265358979f) * x * x)), x); }

uint16_t zfo_float_to_bf16(float value) {
    uint32_t bits;
    memcpy(&bits, &value, 4);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x40u);  /* quiet NaN */
    bits += 0x7fffu + ((bits >> 16) & 1u);
    return (uint16_t)(bits >> 16);
}

uint16_t zfo_float_to_half(float value) {
    uint32_t bits;
    memcpy(&bits, &value, 4);
    const uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    const uint32_t magnitude = bits & 0x7fffffffu;
    if (magnitude > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
    if (magnitude >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  /* rounds to >= 65520: infinity */
    if (magnitude < 0x38800000u) {
        /* half subnormal (or zero): value = m * 2^-24 with m rounded to nearest even */
        float scaled;
        memcpy(&scaled, &magnitude, 4);
        scaled *= 16777216.0f;  /* exact: times 2^24 */
        const float floor_m = floorf(scaled);
        float m = floor_m;
        const float remainder = scaled - floor_m;
        if (remainder > 0.5f || (remainder == 0.5f && fmodf(floor_m, 2.0f) == 1.0f)) m += 1.0f;
        return (uint16_t)(sign | (uint16_t)m);
    }
    uint32_t exponent = (magnitude >> 23) - 127 + 15;
    uint32_t mantissa = magnitude & 0x7fffffu;
    uint32_t half = (exponent << 10) | (mantissa >> 13);
    const uint32_t rest = mantissa & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (half & 1u))) half += 1u;
    return (uint16_t)(sign | half);
}

float zfo_half_to_float(uint16_t value) {
    const uint32_t sign = (uint32_t)(value & 0x8000u) << 16;
    const uint32_t exponent = (value >> 10) & 0x1fu;
    const uint32_t mantissa = value & 0x3ffu;
    uint32_t bits;
    if (exponent == 0) {
        float f = (float)mantissa * (1.0f / 16777216.0f);
        memcpy(&bits, &f, 4);
        bits |= sign;
    }
    else if (exponent == 31) bits = sign | 0x7f800000u | (mantissa << 13);
    else bits = sign | ((exponent - 15 + 127) << 23) | (mantissa << 13);
    float result;
    memcpy(&result, &bits, 4);
    return result;
}

static inline float bf16_to_float(uint16_t value) {
    const uint32_t bits = (uint32_t)value << 16;
    float result;
    memcpy(&result, &bits, 4);
    return result;
}

int zfo_grid_init(zfo_grid* grid, int level, const int64_t* sizes, const int64_t* entries, int n_levels, int n_features, int mlp_width) {
    if (n_levels < 1 || n_levels > ZFO_MAX_LEVELS || n_features < 1) return -1;
    memset(grid, 0, sizeof(*grid));
    grid->level = level;
    grid->n_levels = n_levels;
    grid->n_features = n_features;
    grid->mlp_width = mlp_width;
    grid->offsets[0] = 0;
    for (int l = 0; l < n_levels; l++) {
        grid->sizes[l] = sizes[l];
        grid->entries[l] = entries[l];
        grid->offsets[l + 1] = grid->offsets[l] + entries[l];
        grid->hashed[l] = sizes[l] * sizes[l] * sizes[l] > entries[l];
    }
    while (grid->n_fp32_grad_levels < n_levels && entries[grid->n_fp32_grad_levels] < min_half_grad_entries) grid->n_fp32_grad_levels++;
    return 0;
}

int zfo_n_output_features(const zfo_grid* grid) { return grid->n_levels * (grid->n_features + 1); }

/* featurize_common.cuh:50-98 */
typedef struct {
    vec3 origin, direction, perp_axis1, perp_axis2;
    float radius, t0, ratio, base, root, rotation;
    int flip;
} interval_t;

static interval_t setup_interval(const zfo_grid* grid, const float* origins, const float* directions, const float* radii,
                                 const float* tdist, int64_t pattern_seed, uint32_t sample_idx, uint32_t n_intervals) {
    interval_t iv;
    const uint32_t ray_idx = sample_idx / n_intervals;
    iv.origin = v3(origins[3 * (size_t)ray_idx], origins[3 * (size_t)ray_idx + 1], origins[3 * (size_t)ray_idx + 2]);
    iv.direction = v3(directions[3 * (size_t)ray_idx], directions[3 * (size_t)ray_idx + 1], directions[3 * (size_t)ray_idx + 2]);
    iv.radius = radii[ray_idx];
    const vec3 d = iv.direction;
    vec3 cross1 = v3_cross(d, v3(0.0f, 0.0f, 1.0f));
    const float eps = 1.1920929e-07f;
    if (fabsf(cross1.x) < eps && fabsf(cross1.y) < eps && fabsf(cross1.z) < eps) cross1 = v3_cross(d, v3(1.0f, 1.0f, 1.0f));
    iv.perp_axis1 = v3_normalize(cross1);
    iv.perp_axis2 = v3_normalize(v3_cross(d, cross1));
    const float* t = tdist + (size_t)ray_idx * (n_intervals + 1) + sample_idx % n_intervals;
    const float t0 = t[0], t1 = t[1];
    const float s = 0.5f * (t0 + t1);
    const float h = 0.5f * (t1 - t0);
    const float denominator = h * h + 3.0f * s * s;
    iv.t0 = t0;
    iv.ratio = fabsf(denominator) < tiny ? 0.0f : h / denominator;
    iv.base = t1 * t1 + 2.0f * s * s;
    const float q = h * h - s * s;
    iv.root = sqrtf(fmaxf(q * q + 4.0f * s * s * s * s, 0.0f));
    const uint64_t stream = pattern_stream_base + (uint64_t)grid->level;
    if (pattern_seed >= 0) {
        iv.flip = rng_uniform((uint64_t)pattern_seed, stream, 2ull * sample_idx) < 0.5f;
        iv.rotation = 2.0f * 3.14159265358979f * rng_uniform((uint64_t)pattern_seed, stream, 2ull * sample_idx + 1);
    }
    else {
        iv.flip = (sample_idx % n_intervals) % 2 == 1;
        iv.rotation = iv.flip ? 3.14159265358979f / 6.0f : 0.0f;
    }
    return iv;
}

/* featurize_common.cuh:101-117 */
static void multisample(const interval_t* iv, uint32_t j, vec3* x, float* scale, int* contracted) {
    static const float pattern[N_MULTISAMPLES] = {0.0f, 2.0f, 4.0f, 3.0f, 5.0f, 1.0f};
    const float theta = (3.14159265358979f / 3.0f) * pattern[iv->flip ? N_MULTISAMPLES - 1 - j : j] + iv->rotation;
    const float cz = iv->t0 + iv->ratio * (iv->base + (3.0f / sqrtf(7.0f)) * ((float)j * 0.4f - 1.0f) * iv->root);
    const float perp_mag = sqrtf(0.5f) * iv->radius * cz;
    float sin_theta, cos_theta;
    sincosf(theta, &sin_theta, &cos_theta);
    const vec3 p = v3_add(v3_add(v3_add(iv->origin, v3_scale(perp_mag * cos_theta, iv->perp_axis1)), v3_scale(perp_mag * sin_theta, iv->perp_axis2)),
                          v3_scale(cz, iv->direction));
    const float dot_p = v3_dot(p, p);
    if (contracted) *contracted = dot_p > 1.0f;
    const float norm_sq = fmaxf(dot_p, 1.0f);
    const float norm = sqrtf(norm_sq);
    const float isoscale = expf((2.0f / 3.0f) * logf(2.0f * norm - 1.0f) - logf(norm_sq));
    const float contraction = (2.0f * norm - 1.0f) / norm_sq;
    *x = v3_add(v3_scale(1.0f / grid_bbox_size, v3_scale(contraction, p)), v3(0.5f, 0.5f, 0.5f));
    *scale = multisample_scale * perp_mag * isoscale * (1.0f / grid_bbox_size);
}

/* featurize_common.cuh:202-204 */
static inline float level_weighting(const zfo_grid* grid, int level, float scale) {
    return approx_erf(1.0f / (sqrtf(8.0f) * scale * (float)(uint32_t)grid->sizes[level]));
}

/* the corners of one level, merged per cell (featurize_common.cuh:123-173) */
typedef struct {
    int n_groups;
    int cell[N_MULTISAMPLES][3];
    uint32_t rows[N_MULTISAMPLES][8];
    float weights[N_MULTISAMPLES][8];
} level_corners_t;

static void level_corners(const zfo_grid* grid, int level, const vec3* x, const float* weighting, level_corners_t* out) {
    const uint32_t size = (uint32_t)grid->sizes[level];
    int cells[N_MULTISAMPLES][3];
    float fractions[N_MULTISAMPLES][3];
    for (uint32_t j = 0; j < N_MULTISAMPLES; j++) {
        const float p[3] = {x[j].x * (float)size - 0.5f, x[j].y * (float)size - 0.5f, x[j].z * (float)size - 0.5f};
        for (uint32_t d = 0; d < 3; d++) {
            const float floored = floorf(p[d]);
            cells[j][d] = (int)floored;
            fractions[j][d] = p[d] - floored;
        }
    }
    uint32_t merged = 0;
    out->n_groups = 0;
    for (uint32_t j = 0; j < N_MULTISAMPLES; j++) {
        if (merged & (1u << j)) continue;
        float corner_weights[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        for (uint32_t k = j; k < N_MULTISAMPLES; k++) {
            if (cells[k][0] != cells[j][0] || cells[k][1] != cells[j][1] || cells[k][2] != cells[j][2]) continue;
            merged |= 1u << k;
            for (uint32_t corner = 0; corner < 8; corner++) {
                const float wx = corner & 4u ? fractions[k][0] : 1.0f - fractions[k][0];
                const float wy = corner & 2u ? fractions[k][1] : 1.0f - fractions[k][1];
                const float wz = corner & 1u ? fractions[k][2] : 1.0f - fractions[k][2];
                corner_weights[corner] += weighting[k] * (wx * wy * wz);
            }
        }
        const int g = out->n_groups++;
        out->cell[g][0] = cells[j][0];
        out->cell[g][1] = cells[j][1];
        out->cell[g][2] = cells[j][2];
        for (uint32_t corner = 0; corner < 8; corner++) {
            const int ix = cells[j][0] + (int)((corner >> 2) & 1u);
            const int iy = cells[j][1] + (int)((corner >> 1) & 1u);
            const int iz = cells[j][2] + (int)(corner & 1u);
            uint32_t index;
            float weight = corner_weights[corner];
            if (grid->hashed[level]) {
                index = ((uint32_t)ix ^ ((uint32_t)iy * hash_prime_y) ^ ((uint32_t)iz * hash_prime_z)) % (uint32_t)grid->entries[level];
            }
            else {
                const int n = (int)size;
                const int valid = ix >= 0 && ix < n && iy >= 0 && iy < n && iz >= 0 && iz < n;
                if (!valid) weight = 0.0f;
                index = valid ? (uint32_t)(ix + n * (iy + n * iz)) : 0u;
            }
            out->rows[g][corner] = (uint32_t)grid->offsets[level] + index;
            out->weights[g][corner] = weight;
        }
    }
}

static void multisamples(const interval_t* iv, vec3* x, float* scale, int* contracted) {
    for (uint32_t j = 0; j < N_MULTISAMPLES; j++) multisample(iv, j, &x[j], &scale[j], contracted ? &contracted[j] : NULL);
}

/* featurize_common.cuh:207-227 (GatherFeatures :175-199) */
static void featurize(const zfo_grid* grid, const interval_t* iv, const float* table, const float* scale_magnitudes, float* features) {
    const int F = grid->n_features;
    const float feature_scale = precondition_scaling / (float)N_MULTISAMPLES;
    vec3 x[N_MULTISAMPLES];
    float scale[N_MULTISAMPLES];
    multisamples(iv, x, scale, NULL);
    for (int level = 0; level < grid->n_levels; level++) {
        float weighting[N_MULTISAMPLES];
        float scale_feature = 0.0f;
        for (uint32_t j = 0; j < N_MULTISAMPLES; j++) {
            weighting[j] = level_weighting(grid, level, scale[j]);
            scale_feature += 2.0f * weighting[j] - 1.0f;
        }
        float values[16] = {0.0f};
        level_corners_t corners;
        level_corners(grid, level, x, weighting, &corners);
        for (int g = 0; g < corners.n_groups; g++) {
            for (int corner = 0; corner < 8; corner++) {
                const float weight = corners.weights[g][corner];
                if (weight == 0.0f) continue;
                const float* row = table + (size_t)corners.rows[g][corner] * F;
                for (int f = 0; f < F; f++) values[f] += weight * row[f];
            }
        }
        for (int f = 0; f < F; f++) features[level * (F + 1) + f] = feature_scale * values[f];
        features[level * (F + 1) + F] = feature_scale * scale_feature * scale_magnitudes[level];
    }
}

void zfo_forward(const zfo_grid* grid, int64_t n_rays, int64_t n_intervals,
                 const float* origins, const float* directions, const float* radii, const float* tdist, int64_t pattern_seed,
                 const float* table, const float* scale_magnitudes,
                 const float* w0, const float* b0, const float* w1, const float* b1,
                 float* raw_density, float* features_float,
                 uint16_t* features_bf16, int64_t features_bf16_width,
                 const uint16_t* encoded_directions, int64_t encoded_width,
                 uint16_t* nerf_inputs, int64_t nerf_inputs_width,
                 int n_threads) {
    const int n_out = zfo_n_output_features(grid);
    const int64_t n_samples = n_rays * n_intervals;
    (void)n_threads;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
    #pragma omp parallel for schedule(dynamic, 256) if (n_threads != 1)
#endif
    for (int64_t sample = 0; sample < n_samples; sample++) {
        const interval_t iv = setup_interval(grid, origins, directions, radii, tdist, pattern_seed, (uint32_t)sample, (uint32_t)n_intervals);
        float features[ZFO_MAX_LEVELS * 17];
        featurize(grid, &iv, table, scale_magnitudes, features);
        if (raw_density) {
            /* featurize_forward.cu:65-74 */
            float raw = b1[0];
            for (int j = 0; j < grid->mlp_width; j++) {
                float pre = b0[j];
                for (int i = 0; i < n_out; i++) pre += w0[j * n_out + i] * features[i];
                raw += w1[j] * fmaxf(pre, 0.0f);
            }
            raw_density[sample] = raw;
        }
        if (features_float) {
            for (int i = 0; i < n_out; i++) features_float[sample * n_out + i] = features[i];
        }
        if (features_bf16) {
            uint16_t* out = features_bf16 + sample * features_bf16_width;
            for (int i = 0; i < n_out; i++) out[i] = zfo_float_to_bf16(features[i]);
            for (int64_t i = n_out; i < features_bf16_width; i++) out[i] = 0;
        }
        if (nerf_inputs) {
            /* featurize_forward.cu:86-92: the encoded direction without its last column, then the bias lane 1.0 */
            const uint16_t* encoded = encoded_directions + (sample / n_intervals) * encoded_width;
            uint16_t* out = nerf_inputs + (sample + 1) * nerf_inputs_width - encoded_width;
            for (int64_t i = 0; i < encoded_width - 1; i++) out[i] = encoded[i];
            out[encoded_width - 1] = 0x3f80;
        }
    }
}

/* featurize_common.cuh:273-291 with the fp32 (:230-242) and fp16 (:246-268) row gradients; adds are sequential */
static void scatter_feature_gradients(const zfo_grid* grid, const interval_t* iv, const float* g_all, int n_fp32_levels,
                                      float* grad_table, uint16_t* grad_table_half) {
    const int F = grid->n_features;
    vec3 x[N_MULTISAMPLES];
    float scale[N_MULTISAMPLES];
    multisamples(iv, x, scale, NULL);
    for (int level = 0; level < grid->n_levels; level++) {
        float weighting[N_MULTISAMPLES];
        for (uint32_t j = 0; j < N_MULTISAMPLES; j++) weighting[j] = level_weighting(grid, level, scale[j]);
        const float* g = g_all + level * (F + 1);
        level_corners_t corners;
        level_corners(grid, level, x, weighting, &corners);
        for (int grp = 0; grp < corners.n_groups; grp++) {
            for (int corner = 0; corner < 8; corner++) {
                const float weight = corners.weights[grp][corner];
                if (weight == 0.0f) continue;
                const uint32_t row = corners.rows[grp][corner];
                if (level < n_fp32_levels) {
                    float* grad_row = grad_table + (size_t)row * F;
                    for (int f = 0; f < F; f++) grad_row[f] += weight * g[f];
                }
                else {
                    uint16_t* grad_row = grad_table_half + (size_t)(row - (uint32_t)grid->offsets[n_fp32_levels]) * F;
                    for (int f = 0; f < F; f++) {
                        /* odd F skips zero gradients (featurize_common.cuh:265); adding a rounded zero is a no-op otherwise */
                        if (F % 2 == 1 && g[f] == 0.0f) continue;
                        const float contribution = zfo_half_to_float(zfo_float_to_half(weight * g[f]));
                        grad_row[f] = zfo_float_to_half(zfo_half_to_float(grad_row[f]) + contribution);
                    }
                }
            }
        }
    }
}

void zfo_backward(const zfo_grid* grid, int64_t n_rays, int64_t n_intervals,
                  const float* origins, const float* directions, const float* radii, const float* tdist, int64_t pattern_seed,
                  const uint16_t* grad_features, int64_t grad_stride, float grad_scale,
                  float* grad_table, uint16_t* grad_table_half) {
    const int n_out = zfo_n_output_features(grid);
    const int64_t n_samples = n_rays * n_intervals;
    const float feature_scale = precondition_scaling / (float)N_MULTISAMPLES;
    for (int64_t sample = 0; sample < n_samples; sample++) {
        float grad[ZFO_MAX_LEVELS * 17];
        const uint16_t* row = grad_features + sample * grad_stride;
        for (int i = 0; i < n_out; i++) grad[i] = feature_scale * grad_scale * bf16_to_float(row[i]);
        const interval_t iv = setup_interval(grid, origins, directions, radii, tdist, pattern_seed, (uint32_t)sample, (uint32_t)n_intervals);
        scatter_feature_gradients(grid, &iv, grad, grid->n_fp32_grad_levels, grad_table, grad_table_half);
    }
}

void zfo_backward_mlp(const zfo_grid* grid, int64_t n_rays, int64_t n_intervals,
                      const float* origins, const float* directions, const float* radii, const float* tdist, int64_t pattern_seed,
                      const float* features, const float* grad_raw_density,
                      const float* w0, const float* b0, const float* w1,
                      float* grad_table, float* grad_w0, float* grad_b0, float* grad_w1, float* grad_b1) {
    const int n_out = zfo_n_output_features(grid);
    const int W = grid->mlp_width;
    const int64_t n_samples = n_rays * n_intervals;
    const float feature_scale = precondition_scaling / (float)N_MULTISAMPLES;
    /* parameter gradient sums before the late multiplication by w1 (featurize_backward_mlp.cu:139-147) */
    float* sum_w0 = (float*)calloc((size_t)W * n_out, sizeof(float));
    float* sum_b0 = (float*)calloc((size_t)W, sizeof(float));
    float* sum_w1 = (float*)calloc((size_t)W, sizeof(float));
    float sum_b1 = 0.0f;
    float* pre = (float*)malloc((size_t)W * sizeof(float));
    for (int64_t sample = 0; sample < n_samples; sample++) {
        const float* f = features + sample * n_out;
        const float g = grad_raw_density[sample];
        float grad_f[ZFO_MAX_LEVELS * 17];
        for (int i = 0; i < n_out; i++) grad_f[i] = 0.0f;
        for (int j = 0; j < W; j++) {
            float p = b0[j];
            for (int i = 0; i < n_out; i++) p += w0[j * n_out + i] * f[i];
            pre[j] = p;
            if (p > 0.0f) {
                const float grad_pre = g * w1[j];
                for (int i = 0; i < n_out; i++) grad_f[i] += grad_pre * w0[j * n_out + i];
            }
        }
        if (g != 0.0f) {
            for (int i = 0; i < n_out; i++) grad_f[i] *= feature_scale;
            const interval_t iv = setup_interval(grid, origins, directions, radii, tdist, pattern_seed, (uint32_t)sample, (uint32_t)n_intervals);
            scatter_feature_gradients(grid, &iv, grad_f, grid->n_levels, grad_table, NULL);
        }
        for (int j = 0; j < W; j++) {
            if (pre[j] > 0.0f) {
                for (int i = 0; i < n_out; i++) sum_w0[j * n_out + i] += g * f[i];
                sum_b0[j] += g;
            }
            sum_w1[j] += g * fmaxf(pre[j], 0.0f);
        }
        sum_b1 += g;
    }
    for (int j = 0; j < W; j++) {
        for (int i = 0; i < n_out; i++) grad_w0[j * n_out + i] += w1[j] * sum_w0[j * n_out + i];
        grad_b0[j] += w1[j] * sum_b0[j];
        grad_w1[j] += sum_w1[j];
    }
    grad_b1[0] += sum_b1;
    free(sum_w0);
    free(sum_b0);
    free(sum_w1);
    free(pre);
}

void zfo_debug_interval(const zfo_grid* grid, int64_t n_intervals,
                        const float* origins, const float* directions, const float* radii, const float* tdist, int64_t pattern_seed,
                        int64_t sample_idx,
                        float* x, float* scale, int32_t* contracted,
                        int32_t* n_groups, int32_t* group_cell, uint32_t* rows, float* weights) {
    const interval_t iv = setup_interval(grid, origins, directions, radii, tdist, pattern_seed, (uint32_t)sample_idx, (uint32_t)n_intervals);
    vec3 xs[N_MULTISAMPLES];
    float scales[N_MULTISAMPLES];
    int flags[N_MULTISAMPLES];
    multisamples(&iv, xs, scales, flags);
    for (int j = 0; j < N_MULTISAMPLES; j++) {
        x[3 * j] = xs[j].x;
        x[3 * j + 1] = xs[j].y;
        x[3 * j + 2] = xs[j].z;
        scale[j] = scales[j];
        contracted[j] = flags[j];
    }
    for (int level = 0; level < grid->n_levels; level++) {
        float weighting[N_MULTISAMPLES];
        for (uint32_t j = 0; j < N_MULTISAMPLES; j++) weighting[j] = level_weighting(grid, level, scales[j]);
        level_corners_t corners;
        level_corners(grid, level, xs, weighting, &corners);
        n_groups[level] = corners.n_groups;
        for (int g = 0; g < N_MULTISAMPLES; g++) {
            for (int d = 0; d < 3; d++) group_cell[(level * N_MULTISAMPLES + g) * 3 + d] = g < corners.n_groups ? corners.cell[g][d] : 0;
            for (int c = 0; c < 8; c++) {
                rows[(level * N_MULTISAMPLES + g) * 8 + c] = g < corners.n_groups ? corners.rows[g][c] : 0u;
                weights[(level * N_MULTISAMPLES + g) * 8 + c] = g < corners.n_groups ? corners.weights[g][c] : 0.0f;
            }
        }
    }
}

// ref_cpu.cpp -- the reference's featurization header compiled for the host (TEST INFRASTRUCTURE ONLY).
//
// Built by oracle/Makefile from the sources where they lie (-I to the reference's featurization/rtc and
// common/include directories) into oracle/_ref/libzf_ref_cpu.so. It pins the C oracle (zf_oracle.c) and produces the
// golden vectors under tests/golden/; it is also the reference arm of bench.py's CPU baseline. It runs the
// reference's own interval setup, multisampling, contraction, weighting, corner merging, hashing and gather code with
// IEEE host math (libm) in place of the GPU's fast-math intrinsics.
#include "shim.h"

#include <cstdint>
#include <cstring>
#include <vector>

#include "random.cuh"

unsigned long long zf_ref_pattern_stream = 16;

namespace {

constexpr int max_levels = 16;

struct Layout {
    uint32_t sizes[max_levels];
    uint32_t entries[max_levels];
    uint32_t offsets[max_levels + 1];
    int hashed[max_levels];
};

Layout zf_ref_layout;

uint16_t ref_float_to_bf16(const float value) {
    uint32_t bits;
    std::memcpy(&bits, &value, 4);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((bits >> 16) | 0x40u);
    bits += 0x7fffu + ((bits >> 16) & 1u);
    return static_cast<uint16_t>(bits >> 16);
}

float ref_bf16_to_float(const uint16_t value) { return __uint_as_float(static_cast<uint32_t>(value) << 16); }

uint16_t ref_float_to_half(const float value) { return static_cast<uint16_t>(__builtin_bit_cast(uint16_t, static_cast<_Float16>(value))); }

float ref_half_to_float(const uint16_t value) { return static_cast<float>(__builtin_bit_cast(_Float16, value)); }

void ref_add_float(float* target, const float value, const bool atomic) {
    if (!atomic) {
        *target += value;
        return;
    }
    uint32_t* bits = reinterpret_cast<uint32_t*>(target);
    uint32_t expected = __atomic_load_n(bits, __ATOMIC_RELAXED);
    for (;;) {
        const float sum = __uint_as_float(expected) + value;
        uint32_t desired;
        std::memcpy(&desired, &sum, 4);
        if (__atomic_compare_exchange_n(bits, &expected, desired, true, __ATOMIC_RELAXED, __ATOMIC_RELAXED)) break;
    }
}

// fp16 add of an fp16 value with round-to-nearest-even (red.global.add.noftz.f16)
void ref_add_half(uint16_t* target, const uint16_t value, const bool atomic) {
    const float addend = ref_half_to_float(value);
    if (!atomic) {
        *target = ref_float_to_half(ref_half_to_float(*target) + addend);
        return;
    }
    uint16_t expected = __atomic_load_n(target, __ATOMIC_RELAXED);
    for (;;) {
        const uint16_t desired = ref_float_to_half(ref_half_to_float(expected) + addend);
        if (__atomic_compare_exchange_n(target, &expected, desired, true, __ATOMIC_RELAXED, __ATOMIC_RELAXED)) break;
    }
}

struct ForwardArgs {
    int64_t n_rays, n_intervals;
    const float *origins, *directions, *radii, *tdist;
    int64_t pattern_seed;
    const float *table, *scale_magnitudes, *w0, *b0, *w1, *b1;
    int mlp_width;
    float *raw_density, *features_float;
    uint16_t* features_bf16;
    int64_t features_bf16_width;
    const uint16_t* encoded_directions;
    int64_t encoded_width;
    uint16_t* nerf_inputs;
    int64_t nerf_inputs_width;
    int n_threads;
};

struct BackwardArgs {
    int64_t n_rays, n_intervals;
    const float *origins, *directions, *radii, *tdist;
    int64_t pattern_seed;
    const uint16_t* grad_features;
    int64_t grad_stride;
    float grad_scale;
    int n_fp32_levels;
    float* grad_table;
    uint16_t* grad_table_half;
    int n_threads;
};

struct BackwardMlpArgs {
    int64_t n_rays, n_intervals;
    const float *origins, *directions, *radii, *tdist;
    int64_t pattern_seed;
    const float *features, *grad_raw_density, *w0, *b0, *w1;
    int mlp_width;
    float *grad_table, *grad_w0, *grad_b0, *grad_w1, *grad_b1;
    int n_threads;
};

struct DebugArgs {
    int64_t n_intervals;
    const float *origins, *directions, *radii, *tdist;
    int64_t pattern_seed;
    int64_t sample_idx;
    float *x, *scale;
    int32_t* n_groups;
    uint32_t* rows;
    float* weights;
};

}  // namespace

#define ZF_REF_CAT2(a, b, c, d) a##b##c##d
#define ZF_REF_CAT(a, b, c, d) ZF_REF_CAT2(a, b, c, d)

#define ZF_REF_VARIANTS_F(F) \
    X(1, F) X(2, F) X(3, F) X(4, F) X(5, F) X(6, F) X(7, F) X(8, F) \
    X(9, F) X(10, F) X(11, F) X(12, F) X(13, F) X(14, F) X(15, F) X(16, F)

// one namespace per (levels, features): ref_L<levels>_F<features>
#define ZF_REF_F 1
#include "variants_f.inc"
#undef ZF_REF_F
#define ZF_REF_F 2
#include "variants_f.inc"
#undef ZF_REF_F
#define ZF_REF_F 3
#include "variants_f.inc"
#undef ZF_REF_F
#define ZF_REF_F 4
#include "variants_f.inc"
#undef ZF_REF_F

namespace {

struct Variant {
    void (*forward)(const ForwardArgs&);
    void (*backward)(const BackwardArgs&);
    void (*backward_mlp)(const BackwardMlpArgs&);
    void (*debug_interval)(const DebugArgs&);
};

#define X(L, F) {ref_L##L##_F##F::forward, ref_L##L##_F##F::backward, ref_L##L##_F##F::backward_mlp, ref_L##L##_F##F::debug_interval},
const Variant variants[4][16] = {
    {ZF_REF_VARIANTS_F(1)},
    {ZF_REF_VARIANTS_F(2)},
    {ZF_REF_VARIANTS_F(3)},
    {ZF_REF_VARIANTS_F(4)},
};
#undef X

// layout of featurizer.cu:145-155 and the stream of featurizer.cu:167; returns the variant, or null if unsupported
const Variant* select(const int level, const int64_t* sizes, const int64_t* entries, const int n_levels, const int n_features, int* n_fp32_levels) {
    if (n_levels < 1 || n_levels > max_levels || n_features < 1 || n_features > 4) return nullptr;
    zf_ref_layout.offsets[0] = 0;
    for (int l = 0; l < n_levels; l++) {
        zf_ref_layout.sizes[l] = static_cast<uint32_t>(sizes[l]);
        zf_ref_layout.entries[l] = static_cast<uint32_t>(entries[l]);
        zf_ref_layout.offsets[l + 1] = zf_ref_layout.offsets[l] + static_cast<uint32_t>(entries[l]);
        zf_ref_layout.hashed[l] = sizes[l] * sizes[l] * sizes[l] > entries[l];
    }
    int n = 0;
    while (n < n_levels && entries[n] < (int64_t(1) << 20)) n++;
    if (n_fp32_levels != nullptr) *n_fp32_levels = n;
    zf_ref_pattern_stream = 16ull + static_cast<unsigned long long>(level);
    return &variants[n_features - 1][n_levels - 1];
}

}  // namespace

extern "C" {

int zfr_forward(int level, const int64_t* sizes, const int64_t* entries, int n_levels, int n_features, int mlp_width,
                int64_t n_rays, int64_t n_intervals,
                const float* origins, const float* directions, const float* radii, const float* tdist, int64_t pattern_seed,
                const float* table, const float* scale_magnitudes, const float* w0, const float* b0, const float* w1, const float* b1,
                float* raw_density, float* features_float, uint16_t* features_bf16, int64_t features_bf16_width,
                const uint16_t* encoded_directions, int64_t encoded_width, uint16_t* nerf_inputs, int64_t nerf_inputs_width,
                int n_threads) {
    const Variant* v = select(level, sizes, entries, n_levels, n_features, nullptr);
    if (v == nullptr) return -1;
    ForwardArgs a{n_rays, n_intervals, origins, directions, radii, tdist, pattern_seed, table, scale_magnitudes, w0, b0, w1, b1,
                  mlp_width, raw_density, features_float, features_bf16, features_bf16_width, encoded_directions, encoded_width,
                  nerf_inputs, nerf_inputs_width, n_threads < 1 ? 1 : n_threads};
    v->forward(a);
    return 0;
}

int zfr_backward(int level, const int64_t* sizes, const int64_t* entries, int n_levels, int n_features,
                 int64_t n_rays, int64_t n_intervals,
                 const float* origins, const float* directions, const float* radii, const float* tdist, int64_t pattern_seed,
                 const uint16_t* grad_features, int64_t grad_stride, float grad_scale,
                 float* grad_table, uint16_t* grad_table_half, int n_threads) {
    int n_fp32_levels = 0;
    const Variant* v = select(level, sizes, entries, n_levels, n_features, &n_fp32_levels);
    if (v == nullptr) return -1;
    BackwardArgs a{n_rays, n_intervals, origins, directions, radii, tdist, pattern_seed, grad_features, grad_stride, grad_scale,
                   n_fp32_levels, grad_table, grad_table_half, n_threads < 1 ? 1 : n_threads};
    v->backward(a);
    return 0;
}

int zfr_backward_mlp(int level, const int64_t* sizes, const int64_t* entries, int n_levels, int n_features, int mlp_width,
                     int64_t n_rays, int64_t n_intervals,
                     const float* origins, const float* directions, const float* radii, const float* tdist, int64_t pattern_seed,
                     const float* features, const float* grad_raw_density, const float* w0, const float* b0, const float* w1,
                     float* grad_table, float* grad_w0, float* grad_b0, float* grad_w1, float* grad_b1, int n_threads) {
    const Variant* v = select(level, sizes, entries, n_levels, n_features, nullptr);
    if (v == nullptr) return -1;
    BackwardMlpArgs a{n_rays, n_intervals, origins, directions, radii, tdist, pattern_seed, features, grad_raw_density, w0, b0, w1,
                      mlp_width, grad_table, grad_w0, grad_b0, grad_w1, grad_b1, n_threads < 1 ? 1 : n_threads};
    v->backward_mlp(a);
    return 0;
}

int zfr_debug_interval(int level, const int64_t* sizes, const int64_t* entries, int n_levels, int n_features,
                       int64_t n_intervals, const float* origins, const float* directions, const float* radii, const float* tdist,
                       int64_t pattern_seed, int64_t sample_idx, float* x, float* scale, int32_t* n_groups, uint32_t* rows, float* weights) {
    const Variant* v = select(level, sizes, entries, n_levels, n_features, nullptr);
    if (v == nullptr) return -1;
    DebugArgs a{n_intervals, origins, directions, radii, tdist, pattern_seed, sample_idx, x, scale, n_groups, rows, weights};
    v->debug_interval(a);
    return 0;
}

}  // extern "C"

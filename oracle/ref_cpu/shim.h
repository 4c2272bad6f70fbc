// shim.h -- host definitions that let the reference's runtime-compiled featurization header
// (ZipNeRFCudaBackend/ZipNeRFCudaBackend/featurization/rtc/featurize_common.cuh, with common/include/random.cuh)
// compile as plain C++ for the CPU. TEST INFRASTRUCTURE ONLY: the resulting library (oracle/_ref/) pins the C oracle
// and is the reference arm of the CPU baseline; the product never loads it.
//
// The reference header expects NVRTC built-ins (float3, rsqrtf, __uint_as_float, __umul64hi, atomicAdd) and a
// generated preamble (integer typedefs, JIT_* constants, and the per-level layout functions of
// featurizer.cu:157-184). The layout functions are supplied per variant by ref_cpu.cpp; the rest is here.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>

#define __device__
#define __forceinline__ inline
#define __restrict__ __restrict

struct float2 { float x, y; };
struct float3 { float x, y, z; };
struct float4 { float x, y, z, w; };

inline float3 make_float3(const float x, const float y, const float z) { return float3{x, y, z}; }

// the GPU's reciprocal square root, as the IEEE quotient on the host
inline float rsqrtf(const float x) { return 1.0f / sqrtf(x); }

inline float __uint_as_float(const uint32_t bits) {
    float value;
    std::memcpy(&value, &bits, sizeof(value));
    return value;
}

inline unsigned long long __umul64hi(const unsigned long long a, const unsigned long long b) {
    return static_cast<unsigned long long>((static_cast<unsigned __int128>(a) * b) >> 64);
}

// referenced by the reference's fp32 row gradient (featurize_common.cuh:239); the host driver scatters with its own
// visitor, so this is never called
inline float atomicAdd(float* address, const float value) {
    const float old = *address;
    *address = old + value;
    return old;
}

// random stream of the multisampling patterns (JIT_PATTERN_STREAM of the preamble): set per call by the driver
extern unsigned long long zf_ref_pattern_stream;
#define JIT_PATTERN_STREAM zf_ref_pattern_stream
#define JIT_PRECONDITION_SCALING 10.0f
#define JIT_MLP_WIDTH 0u
#define JIT_N_FP32_GRAD_LEVELS 0u

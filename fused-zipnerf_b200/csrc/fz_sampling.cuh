// fz_sampling.cuh -- sm_100a kernels of the per-ray sampling steps around the featurization: the first level's interval
// endpoints and view-direction encoding of new rays (training batches of random pixels, inference views, given rays),
// the counter-based uniforms, and the compositing of a proposal level's densities with the resampling of the next
// level's intervals.
//
// Per ray the arithmetic is the reference's, operation for operation (B/sampling/include/ray_ops.cuh:20-88 and
// B/sampling/src/sampling_api.cu:41-196, B/ = ZipNeRFCudaBackend/ZipNeRFCudaBackend/): sequential sums in interval
// order, the same fast-math intrinsics (the library is compiled with --use_fast_math like the reference,
// setup.py:28-34), so the outputs equal the reference kernels' bit for bit. The layout is this build's: one warp per
// block and one ray per lane; a ray's rows (densities, interval endpoints, its working arrays) live in shared memory
// rows of odd stride (conflict-free column walks), and rows move between HBM and shared memory as warp-wide coalesced
// row copies, instead of per-thread local-memory arrays and per-thread strided row accesses.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "fz_device.cuh"

namespace zf {

// ray distance warp: the mapping between normalized distances s in [0, 1] and metric distances t (the constants of
// utils.ray_warp, utils.py:19-27; the field order of RayWarp, ray_ops.cuh:16-18)
struct RayWarp {
    float near, far, fn_near, fn_far, power, premult, y_max;
};

constexpr int kMaxSamplingIntervals = 64;        // intervals per ray and level (ray_ops.cuh:10)
constexpr float kSamplingTiny = 1.17549435e-38f;  // FLT_MIN (ray_ops.cuh:12)
constexpr float kSamplingEps = 1.1920929e-07f;    // FLT_EPSILON (ray_ops.cuh:13)
constexpr float kMaxDensityExponent = 88.72283f;  // exp stays finite (ray_ops.cuh:14)
constexpr int kSamplingRays = 32;                 // rays per block: one warp, one ray per lane

// streams of the counter-based random numbers (random.cuh:8-12)
constexpr unsigned long long kStreamPixel = 0, kStreamBackground = 1, kStreamJitter = 2;

// uniform integer in [0, n): the high word of hash * n (random.cuh:32-34)
__device__ __forceinline__ unsigned long long rng_uniform_int(const unsigned long long seed, const unsigned long long stream,
                                                              const unsigned long long index, const unsigned long long n) {
    return __umul64hi(splitmix64(splitmix64(seed ^ (stream << 56)) ^ index), n);
}

// normalized distance -> metric distance through the inverse power ladder (ray_ops.cuh:26-33)
__device__ __forceinline__ float s_to_t(const float s, const RayWarp& warp) {
    const float y = s * warp.fn_far + (1.0f - s) * warp.fn_near;
    const float yp = warp.power < 0.0f ? fminf(fabsf(y), warp.y_max) : fabsf(y);
    const float p = warp.power;
    const float x = copysignf(fabsf(p - 1.0f) * (powf(p / fabsf(p - 1.0f) * yp + 1.0f, 1.0f / p) - 1.0f), y) / warp.premult;
    return fminf(fmaxf(x, warp.near), warp.far);
}

// density activation exp(raw - 1), clipped to finite values (ray_ops.cuh:35-37)
__device__ __forceinline__ float activate_density(const float raw) { return expf(fminf(raw - 1.0f, kMaxDensityExponent)); }

// smem row stride of a block's per-ray rows: odd (a warp's column walk hits 32 distinct banks), >= cols
__host__ __device__ constexpr int sampling_stride(const int cols) { return cols | 1; }

// |v| (sampling_api.cu:37)
__device__ __forceinline__ float norm3(const float3 v) { return sqrtf(v.x * v.x + v.y * v.y + v.z * v.z); }

// rows [ray0, ray0 + n_rows) of a row-major [*, cols] float matrix -> shared rows of `stride` floats, as asynchronous
// 4-byte copies (cp.async): the warp walks the block's contiguous chunk element by element (coalesced), every copy is
// in flight at once, and the caller waits for all of them (wait_async_rows) before the rows are read. A block's chunk
// is a few KB, so that many copies in flight per warp is what keeps the HBM busy at this kernel's low occupancy.
__device__ __forceinline__ void load_rows_async(const float* __restrict__ src, const int64_t ray0, const int n_rows, const int cols, float* dst,
                                                const int stride) {
    const int lane = threadIdx.x & 31;
    const float* base = src + ray0 * cols;
    const int total = n_rows * cols;
    const uint32_t dst_base = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    int row = 0, col = lane;
    while (col >= cols) {
        col -= cols;
        row++;
    }
    for (int e = lane; e < total; e += 32) {
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst_base + 4u * static_cast<uint32_t>(row * stride + col)), "l"(base + e) : "memory");
        col += 32;
        while (col >= cols) {
            col -= cols;
            row++;
        }
    }
}

__device__ __forceinline__ void wait_async_rows() {
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncwarp();
}

__device__ __forceinline__ void store_rows(const float* src, const int stride, const int n_rows, const int cols, float* __restrict__ dst, const int64_t ray0) {
    const int lane = threadIdx.x & 31;
    float* base = dst + ray0 * cols;
#pragma unroll 4
    for (int r = 0; r < n_rows; r++) {
        for (int c = lane; c < cols; c += 32) base[static_cast<int64_t>(r) * cols + c] = src[r * stride + c];
    }
}

// Resampling of one ray (ray_ops.cuh:41-88): n_out intervals from the step function (t, softmax(anneal log w)) of n
// bins. t: the n + 1 bin edges; w: the n bin weights; work: n + 1 floats of scratch (logits, then the cdf); s_out: the
// n_out + 1 new edges (may alias w: w is read only before s_out is written). jitter < 0 selects the centered pattern.
__device__ __forceinline__ void resample_ray(const float* t, const float* w, const int n, const float anneal, const int n_out, const float jitter,
                                             float* work, float* s_out) {
    // logits of the annealed weights; empty bins get -inf
    float max_logit = -INFINITY;
    for (int i = 0; i < n; i++) {
        const float logit = t[i + 1] > t[i] ? anneal * logf(fmaxf(w[i], kSamplingTiny)) : -INFINITY;
        work[i] = logit;
        max_logit = fmaxf(max_logit, logit);
    }
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        const float p = work[i] == -INFINITY ? 0.0f : expf(work[i] - max_logit);
        work[i] = p;
        sum += p;
    }
    // cdf with explicit 0 and 1 endpoints, in place over the probabilities (each entry is read before it is replaced)
    float acc = 0.0f;
    float previous = work[0];
    work[0] = 0.0f;
    for (int i = 1; i < n; i++) {
        acc += previous / sum;
        previous = work[i];
        work[i] = fminf(acc, 1.0f);
    }
    work[n] = 1.0f;
    // stratified (one jitter per ray) or centered positions in the cdf
    float u_start, u_step;
    if (jitter >= 0.0f) {
        const float u_max = kSamplingEps + (1.0f - kSamplingEps) / n_out;
        u_start = jitter * ((1.0f - u_max) / (n_out - 1) - kSamplingEps);
        u_step = (1.0f - u_max) / (n_out - 1);
    } else {
        const float pad = 1.0f / (2 * n_out);
        u_start = pad;
        u_step = (1.0f - 2.0f * pad - kSamplingEps) / (n_out - 1);
    }
    // inverse cdf at the sorted positions (a merge: idx only grows); the new edges are the midpoints of consecutive
    // sample centers, the outer two extrapolated, all clamped to [0, 1]
    int idx = 0;
    float first = 0.0f, second = 0.0f, before_last = 0.0f, last = 0.0f;
    for (int j = 0; j < n_out; j++) {
        const float u = u_start + j * u_step;
        while (idx <= n && work[idx] <= u) idx++;
        const int i0 = max(idx - 1, 0), i1 = min(idx, n);
        const float offset = fminf(fmaxf((u - work[i0]) / fmaxf(kSamplingEps * kSamplingEps, work[i1] - work[i0]), 0.0f), 1.0f);
        const float center = t[i0] + offset * (t[i1] - t[i0]);
        if (j == 0) first = center;
        if (j == 1) second = center;
        if (j > 0) s_out[j] = fminf(fmaxf(0.5f * (last + center), 0.0f), 1.0f);
        before_last = last;
        last = center;
    }
    s_out[0] = fminf(fmaxf(2.0f * first - 0.5f * (first + second), 0.0f), 1.0f);
    s_out[n_out] = fminf(fmaxf(2.0f * last - 0.5f * (before_last + last), 0.0f), 1.0f);
}

// ---------------------------------------------------------------------------------------------------------------------
// composite_and_resample (sampling_api.cu:174-196): per ray, the proposal level's alpha-compositing weights from its raw
// densities, then the next level's intervals resampled from them

struct ResampleArgs {
    const float* raw_density;  // [n_rays, n]
    const float* sdist;        // [n_rays, n + 1]
    const float* tdist;        // [n_rays, n + 1]
    const float* directions;   // [n_rays, 3]
    float* weights;            // [n_rays, n] or null
    float* sdist_next;         // [n_rays, n_out + 1]
    float* tdist_next;         // [n_rays, n_out + 1]
    int64_t n_rays;
    int n, n_out;
    float anneal;
    long long seed;
    int next_level;
    RayWarp warp;
};

__host__ __device__ constexpr int resample_smem_floats(const int n, const int n_out) {
    return 3 * kSamplingRays * sampling_stride((n > n_out ? n : n_out) + 1);
}

__global__ void __launch_bounds__(kSamplingRays) fz_composite_and_resample_kernel(const __grid_constant__ ResampleArgs a) {
    extern __shared__ float smem[];
    const int stride = sampling_stride((a.n > a.n_out ? a.n : a.n_out) + 1);
    float* rows_a = smem;                               // raw densities -> weights -> new edges s -> new edges t
    float* rows_s = rows_a + kSamplingRays * stride;    // the level's edges s
    float* rows_t = rows_s + kSamplingRays * stride;    // the level's edges t -> logits -> cdf
    const int lane = threadIdx.x;
    const int64_t ray0 = static_cast<int64_t>(blockIdx.x) * kSamplingRays;
    const int n_rows = static_cast<int>(min(static_cast<int64_t>(kSamplingRays), a.n_rays - ray0));
    const int n = a.n, n_out = a.n_out;
    load_rows_async(a.raw_density, ray0, n_rows, n, rows_a, stride);
    load_rows_async(a.sdist, ray0, n_rows, n + 1, rows_s, stride);
    load_rows_async(a.tdist, ray0, n_rows, n + 1, rows_t, stride);
    const bool active = lane < n_rows;
    const int64_t ray = ray0 + lane;
    float direction_norm = 0.0f;
    if (active) direction_norm = norm3(make_float3(a.directions[3 * ray], a.directions[3 * ray + 1], a.directions[3 * ray + 2]));
    wait_async_rows();
    float* row_a = rows_a + lane * stride;
    float* row_t = rows_t + lane * stride;
    if (active) {
        // alpha compositing (ray_ops.cuh:91-99): w_i = (1 - exp(-x_i)) exp(-sum_{j<i} x_j), x_i = sigma_i dt_i |d|
        float optical_depth = 0.0f;
#pragma unroll 4
        for (int i = 0; i < n; i++) {
            const float x = activate_density(row_a[i]) * (row_t[i + 1] - row_t[i]) * direction_norm;
            row_a[i] = -expm1f(-x) * expf(-optical_depth);
            optical_depth += x;
        }
    }
    __syncwarp();
    if (a.weights != nullptr) store_rows(rows_a, stride, n_rows, n, a.weights, ray0);
    __syncwarp();
    if (active) {
        const float jitter = a.seed >= 0 ? rng_uniform(static_cast<unsigned long long>(a.seed), kStreamJitter + a.next_level, ray) : -1.0f;
        resample_ray(rows_s + lane * stride, row_a, n, a.anneal, n_out, jitter, row_t, row_a);
    }
    __syncwarp();
    store_rows(rows_a, stride, n_rows, n_out + 1, a.sdist_next, ray0);
    __syncwarp();
    if (active) {
        for (int i = 0; i <= n_out; i++) row_a[i] = s_to_t(row_a[i], a.warp);
    }
    __syncwarp();
    store_rows(rows_a, stride, n_rows, n_out + 1, a.tdist_next, ray0);
}

// ---------------------------------------------------------------------------------------------------------------------
// new rays: the view-direction encoding and the first level's intervals (sampling_api.cu:41-62), for given rays
// (initialize_rays), the pixels of one view (view_rays) or random pixels of all training views (generate_rays)

// encoded width: identity, sines and cosines of 3 axes and `degree` octaves, a bias lane, padded to a multiple of 8
// (zipnerf_config.h:18)
__host__ __device__ constexpr int direction_block_width(const int degree) { return (3 + 6 * degree + 1 + 7) / 8 * 8; }

enum class RaySource : int { Given = 0, View = 1, Pool = 2 };

struct NewRaysArgs {
    RaySource source;
    long long seed;                     // Given: >= 0 jitter, < 0 centered; Pool: the batch seed (always jittered)
    int64_t n_rays;
    // Given
    const float* directions_in;         // [n_rays, 3]
    // View
    const int64_t* pixel_indices;       // [n_rays]
    float view_radius;
    // View and Pool
    const float* local_directions;      // [*, 3] per camera pixel
    const float* c2w;                   // [n_views, 3, 4] (View: one view)
    // Pool
    const int64_t* view_offsets;        // [n_views + 1] first pixel of each view in the pool
    int n_views;
    const int32_t* view_cameras;        // [n_views]
    const int64_t* camera_offsets;      // [n_cameras + 1] first local direction of each camera
    const float* camera_radii;          // [n_cameras]
    const uint8_t* pool_rgb;            // [n_pixels, 3]
    int64_t n_pixels;
    // outputs (View and Pool: rays; Pool: colors; all: encoding and intervals)
    float* origins;                     // [n_rays, 3]
    float* directions;                  // [n_rays, 3]
    float* radii;                       // [n_rays]
    float* rgb;                         // [n_rays, 3]
    uint16_t* encoded_directions;       // bf16 [n_rays, direction_block_width(degree)]
    int encoded_vectors;                // nonzero: encoded_directions is 16-byte aligned (16-byte row stores)
    float* sdist;                       // [n_rays, n_samples + 1]
    float* tdist;                       // [n_rays, n_samples + 1]
    int degree, n_samples;
    RayWarp warp;
};

// shared memory of a block: the rays' new edges (floats), then their encodings (bf16 rows of 16-byte multiples)
__host__ __device__ constexpr int encoded_stride(const int width) { return width + 8; }
__host__ __device__ constexpr int new_rays_smem_bytes(const int n_samples, const int width) {
    return 4 * kSamplingRays * sampling_stride(n_samples + 1) + 2 * kSamplingRays * encoded_stride(width);
}

// world-space direction of a camera-space direction (c2w row-major 3 x 4, sampling_api.cu:65-67)
__device__ __forceinline__ float3 world_direction(const float* m, const float3 local) {
    return make_float3(m[0] * local.x + m[1] * local.y + m[2] * local.z, m[4] * local.x + m[5] * local.y + m[6] * local.z,
                       m[8] * local.x + m[9] * local.y + m[10] * local.z);
}

// the view-direction encoding of one ray into a shared row (sampling_api.cu:44-56): the unit direction v, then
// sin(2^k v) at 3 + 3 k + c and cos(2^k v) at 3 + 3 (degree + k) + c for octaves k and axes c, zeros elsewhere
__device__ __forceinline__ void encode_direction(const float3 d, const int degree, const int width, uint16_t* encoded) {
    // 1 / |d| with the roundings of the reference build (its 1.0f / norm3(d) under fast math): a reciprocal square root
    // of (x x + y y) + z z fused as written here. The compiler contracts the plain expression differently from one
    // kernel to another (1 ulp on ~1 ray in 2000, visible in the bf16 sines); this form matched the reference kernels
    // on every one of 170,000 directions in a black-box comparison on the B200.
    const float inv_norm = rsqrtf(__fmaf_rn(d.z, d.z, __fmaf_rn(d.x, d.x, __fmul_rn(d.y, d.y))));
    const float v[3] = {d.x * inv_norm, d.y * inv_norm, d.z * inv_norm};
    for (int i = 0; i < width; i++) encoded[i] = f32_to_bf16_bits(0.0f);
    for (int c = 0; c < 3; c++) {
        encoded[c] = f32_to_bf16_bits(v[c]);
        for (int k = 0; k < degree; k++) {
            float sin_value, cos_value;
            sincosf(scalbnf(v[c], k), &sin_value, &cos_value);
            encoded[3 + 3 * k + c] = f32_to_bf16_bits(sin_value);
            encoded[3 + 3 * (degree + k) + c] = f32_to_bf16_bits(cos_value);
        }
    }
}

__global__ void __launch_bounds__(kSamplingRays) fz_new_rays_kernel(const __grid_constant__ NewRaysArgs a) {
    extern __shared__ __align__(16) float smem[];
    const int stride = sampling_stride(a.n_samples + 1);
    const int width = direction_block_width(a.degree);
    const int enc_stride = encoded_stride(width);
    uint16_t* enc_rows = reinterpret_cast<uint16_t*>(smem + kSamplingRays * stride);
    const int lane = threadIdx.x;
    const int64_t ray0 = static_cast<int64_t>(blockIdx.x) * kSamplingRays;
    const int n_rows = static_cast<int>(min(static_cast<int64_t>(kSamplingRays), a.n_rays - ray0));
    const int64_t ray = ray0 + lane;
    float* row = smem + lane * stride;
    uint16_t* enc = enc_rows + lane * enc_stride;
    if (lane < n_rows) {
        float3 d;
        float jitter = -1.0f;
        if (a.source == RaySource::Given) {
            d = make_float3(a.directions_in[3 * ray], a.directions_in[3 * ray + 1], a.directions_in[3 * ray + 2]);
            if (a.seed >= 0) jitter = rng_uniform(static_cast<unsigned long long>(a.seed), kStreamJitter, ray);
        } else {
            const float* m;
            const float* local;
            float radius;
            if (a.source == RaySource::View) {
                m = a.c2w;
                local = a.local_directions + 3 * a.pixel_indices[ray];
                radius = a.view_radius;
            } else {
                // a random pixel of the pool; its view is the last whose first pixel is <= it (sampling_api.cu:95-103)
                const unsigned long long seed = static_cast<unsigned long long>(a.seed);
                const int64_t pixel = static_cast<int64_t>(rng_uniform_int(seed, kStreamPixel, ray, static_cast<unsigned long long>(a.n_pixels)));
                int lo = 0, hi = a.n_views;
                while (hi - lo > 1) {
                    const int mid = (lo + hi) / 2;
                    if (a.view_offsets[mid] <= pixel) lo = mid;
                    else hi = mid;
                }
                const int camera = a.view_cameras[lo];
                local = a.local_directions + 3 * (a.camera_offsets[camera] + pixel - a.view_offsets[lo]);
                m = a.c2w + 12 * lo;
                radius = a.camera_radii[camera];
                for (int c = 0; c < 3; c++) a.rgb[3 * ray + c] = a.pool_rgb[3 * pixel + c] / 255.0f;
                jitter = rng_uniform(seed, kStreamJitter, ray);
            }
            d = world_direction(m, make_float3(local[0], local[1], local[2]));
            a.origins[3 * ray] = m[3];
            a.origins[3 * ray + 1] = m[7];
            a.origins[3 * ray + 2] = m[11];
            a.directions[3 * ray] = d.x;
            a.directions[3 * ray + 1] = d.y;
            a.directions[3 * ray + 2] = d.z;
            a.radii[ray] = radius;
        }
        encode_direction(d, a.degree, width, enc);
        // the first level samples the single unit bin [0, 1] (sampling_api.cu:57-61)
        float unit_edges[2] = {0.0f, 1.0f}, unit_weight[1] = {1.0f}, work[2];
        resample_ray(unit_edges, unit_weight, 1, 1.0f, a.n_samples, jitter, work, row);
        // the encoding row leaves as 16-byte chunks (widths are multiples of 8 values)
        uint16_t* out = a.encoded_directions + ray * width;
        for (int e0 = 0; e0 < width; e0 += 8) {
            const uint4 chunk = *reinterpret_cast<const uint4*>(enc + e0);
            if (a.encoded_vectors) {
                *reinterpret_cast<uint4*>(out + e0) = chunk;
            } else {
                for (int q = 0; q < 8; q++) out[e0 + q] = enc[e0 + q];
            }
        }
    }
    __syncwarp();
    store_rows(smem, stride, n_rows, a.n_samples + 1, a.sdist, ray0);
    __syncwarp();
    if (lane < n_rows) {
        for (int i = 0; i <= a.n_samples; i++) row[i] = s_to_t(row[i], a.warp);
    }
    __syncwarp();
    store_rows(smem, stride, n_rows, a.n_samples + 1, a.tdist, ray0);
}

// the uniforms of one counter-based stream (sampling_api.cu:168-172), grid-stride
__global__ void __launch_bounds__(256) fz_sample_uniforms_kernel(const unsigned long long seed, const unsigned long long stream, const int64_t n,
                                                                 float* __restrict__ values) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        values[i] = rng_uniform(seed, stream, static_cast<unsigned long long>(i));
    }
}

}  // namespace zf

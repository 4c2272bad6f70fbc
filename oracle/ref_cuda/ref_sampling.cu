// ref_sampling.cu -- host launchers around the reference's own sampling and optimizer kernels (TEST INFRASTRUCTURE ONLY).
//
// The reference's sampling kernels (B/sampling/src/sampling_api.cu) and its Adam kernel (B/optimizer/src/
// optimizer_api.cu) sit in files whose host wrappers take torch::Tensor arguments. This file includes both sources
// unmodified, from where they lie, against the placeholder torch headers of oracle/ref_cuda/torch_stub (the wrappers
// compile but are never called), and launches the reference kernels directly with the reference's launch shapes and
// compile options (-O3 -use_fast_math, setup.py:28-34). oracle/ref_cuda/build.py compiles it for sm_100a into
// oracle/_ref/cuda/libzfref_sampling.so. The GPU parity tests compare the product kernels with these, and
// tests/bench_vs_reference_cuda.py times both. B/ abbreviates ZipNeRFCudaBackend/ZipNeRFCudaBackend/.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>

#include "sampling_api.cu"
#include "optimizer_api.cu"

#define REF_API extern "C" __attribute__((visibility("default")))

namespace {

namespace zs = zipnerf::sampling;
namespace zo = zipnerf::optimizer;

// one thread per ray in blocks of 128 (sampling_api.cu:13,443)
unsigned n_blocks(const int64_t n) { return static_cast<unsigned>((n + zs::block_size - 1) / zs::block_size); }

zs::RayWarp ray_warp(const float* w) { return {w[0], w[1], w[2], w[3], w[4], w[5], w[6]}; }

int status() { return static_cast<int>(cudaGetLastError()); }

}  // namespace

// generate_rays_wrapper (sampling_api.cu:447-485)
REF_API int ref_generate_rays(int64_t seed, int n_rays, const int64_t* view_offsets, int n_views, const int* view_cameras, const int64_t* camera_offsets,
                              const float* local_directions, const float* c2w, const float* camera_radii, const uint8_t* pool_rgb, int64_t n_pixels,
                              int direction_degree, int n_samples, const float* warp, float* origins, float* directions, float* radii, float* rgb,
                              uint16_t* encoded_directions, float* sdist, float* tdist, cudaStream_t stream) {
    if (n_rays == 0) return 0;
    zs::generate_rays_kernel<<<n_blocks(n_rays), zs::block_size, 0, stream>>>(
        static_cast<uint64_t>(seed), n_pixels, view_offsets, n_views, view_cameras, camera_offsets, local_directions, c2w, camera_radii, pool_rgb,
        origins, directions, radii, rgb, reinterpret_cast<__nv_bfloat16*>(encoded_directions), sdist, tdist, direction_degree, n_samples, ray_warp(warp), n_rays);
    return status();
}

// view_rays_wrapper (sampling_api.cu:487-518)
REF_API int ref_view_rays(const int64_t* pixel_indices, int n_rays, const float* local_directions, const float* c2w, float radius, int direction_degree,
                          int n_samples, const float* warp, float* origins, float* directions, float* radii, uint16_t* encoded_directions, float* sdist,
                          float* tdist, cudaStream_t stream) {
    if (n_rays == 0) return 0;
    zs::view_rays_kernel<<<n_blocks(n_rays), zs::block_size, 0, stream>>>(
        pixel_indices, local_directions, c2w, radius, origins, directions, radii, reinterpret_cast<__nv_bfloat16*>(encoded_directions), sdist, tdist,
        direction_degree, n_samples, ray_warp(warp), n_rays);
    return status();
}

// initialize_rays_wrapper (sampling_api.cu:520-539)
REF_API int ref_initialize_rays(int64_t seed, const float* directions, int n_rays, int direction_degree, int n_samples, const float* warp,
                                uint16_t* encoded_directions, float* sdist, float* tdist, cudaStream_t stream) {
    if (n_rays == 0) return 0;
    zs::initialize_rays_kernel<<<n_blocks(n_rays), zs::block_size, 0, stream>>>(
        seed, directions, reinterpret_cast<__nv_bfloat16*>(encoded_directions), sdist, tdist, direction_degree, n_samples, ray_warp(warp), n_rays);
    return status();
}

// sample_uniforms_wrapper (sampling_api.cu:541-548)
REF_API int ref_sample_uniforms(int64_t seed, int64_t stream_index, int64_t n, float* values, cudaStream_t stream) {
    if (n == 0) return 0;
    zs::sample_uniforms_kernel<<<n_blocks(n), zs::block_size, 0, stream>>>(static_cast<uint64_t>(seed), values, static_cast<uint64_t>(stream_index), n);
    return status();
}

// composite_and_resample_wrapper (sampling_api.cu:550-578)
REF_API int ref_composite_and_resample(const float* raw_density, const float* sdist, const float* tdist, const float* directions, int n_rays,
                                       int n_intervals, float anneal, int n_samples, int64_t seed, int next_level, const float* warp, float* weights,
                                       float* sdist_next, float* tdist_next, cudaStream_t stream) {
    if (n_rays == 0) return 0;
    zs::composite_and_resample_kernel<<<n_blocks(n_rays), zs::block_size, 0, stream>>>(
        raw_density, sdist, tdist, directions, weights, sdist_next, tdist_next, n_intervals, anneal, n_samples, seed, next_level, ray_warp(warp), n_rays);
    return status();
}

// train_final_wrapper (sampling_api.cu:580-645): the proposal levels' arrays hold n_levels entries each
REF_API int ref_train_final(const uint16_t* nerf_outputs, const float* sdist, const float* tdist, int n_rays, int n_intervals, int n_levels,
                            const int* proposal_n_intervals, const float* const* proposal_raw_density, const float* const* proposal_sdist,
                            const float* const* proposal_tdist, const float* const* proposal_weights, float* const* proposal_raw_density_grad,
                            const float* interlevel_weights, const float* interlevel_blurs, const float* directions, int64_t seed, const float* rgb_target,
                            float charbonnier_padding, float distortion_weight, float distortion_power, float distortion_premult,
                            uint16_t* nerf_outputs_grad, float* loss_sums, cudaStream_t stream) {
    if (n_levels > zs::max_proposal_levels) return static_cast<int>(cudaErrorInvalidValue);
    zs::ProposalLevels proposals{};
    proposals.n_levels = n_levels;
    for (int level = 0; level < n_levels; level++) {
        proposals.n_intervals[level] = proposal_n_intervals[level];
        proposals.raw_density[level] = proposal_raw_density[level];
        proposals.sdist[level] = proposal_sdist[level];
        proposals.tdist[level] = proposal_tdist[level];
        proposals.weights[level] = proposal_weights[level];
        proposals.raw_density_grad[level] = proposal_raw_density_grad[level];
        proposals.interlevel_weight[level] = interlevel_weights[level];
        proposals.interlevel_blur[level] = interlevel_blurs[level];
    }
    if (n_rays == 0) return 0;
    zs::train_final_kernel<<<n_blocks(n_rays), zs::block_size, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(nerf_outputs), sdist, tdist, proposals, directions, static_cast<uint64_t>(seed), rgb_target,
        reinterpret_cast<__nv_bfloat16*>(nerf_outputs_grad), loss_sums, n_intervals, charbonnier_padding, distortion_weight, distortion_power,
        distortion_premult, n_rays);
    return status();
}

// composite_final_wrapper (sampling_api.cu:647-678); null alpha / depth are skipped
REF_API int ref_composite_final(const uint16_t* nerf_outputs, const float* tdist, const float* directions, const float* background,
                                const int64_t* pixel_indices, int n_rays, int n_intervals, float* rgb, float* alpha, float* depth, int use_median_depth,
                                cudaStream_t stream) {
    if (n_rays == 0) return 0;
    zs::composite_final_kernel<<<n_blocks(n_rays), zs::block_size, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(nerf_outputs), tdist, directions, background, pixel_indices, rgb, alpha, depth, n_intervals, n_rays,
        use_median_depth != 0);
    return status();
}

// Adam::step (optimizer_api.cu:160-220) for the buffers of an Adam object: grads[b] is fp16 when grad_half[b] is
// nonzero; level_offsets holds n_offsets[b] entries per buffer (0: no levels); step counts from 1. The caller keeps
// the object's state (exp_avgs, exp_avg_sqs, zero-initialized; level_sums and counter, zeroed once and left zeroed by
// every step) as the reference's Adam does (optimizer_api.cu:140-158).
REF_API int ref_adam_step(int n_buffers, float* const* params, void* const* grads, const int* grad_half, float* const* exp_avgs, float* const* exp_avg_sqs,
                          const int64_t* numels, const double* grad_scales, const int64_t* level_offsets, const int* n_offsets, double reg_weight,
                          double max_value, double beta1, double beta2, double eps, int64_t step, double lr, float* magnitudes, float* regularization,
                          double* level_sums, unsigned* counter, cudaStream_t stream) {
    if (n_buffers <= 0 || n_buffers > zo::max_buffers) return static_cast<int>(cudaErrorInvalidValue);
    zo::StepParams p{};
    int64_t n_groups = 0;
    int level = 0;
    const int64_t* offsets = level_offsets;
    for (int b = 0; b < n_buffers; b++) {
        p.buffers[b] = {reinterpret_cast<float4*>(params[b]), grad_half[b] ? nullptr : reinterpret_cast<float4*>(grads[b]),
                        grad_half[b] ? reinterpret_cast<uint2*>(grads[b]) : nullptr, reinterpret_cast<float4*>(exp_avgs[b]),
                        reinterpret_cast<float4*>(exp_avg_sqs[b]), n_groups, static_cast<float>(1.0 / grad_scales[b])};
        if (n_offsets[b] == 0) p.ranges[p.n_ranges++] = {n_groups + numels[b] / 4, b, -1};
        for (int i = 0; i + 1 < n_offsets[b]; i++, level++) {
            if (level >= zo::max_levels) return static_cast<int>(cudaErrorInvalidValue);
            const int64_t size = offsets[i + 1] - offsets[i];
            p.level_reg_weights[level] = static_cast<float>(reg_weight / static_cast<double>(size));
            p.level_inv_sizes[level] = 1.0 / static_cast<double>(size);
            p.ranges[p.n_ranges++] = {n_groups + offsets[i + 1] / 4, b, level};
        }
        offsets += n_offsets[b];
        n_groups += numels[b] / 4;
    }
    const float beta1_f = static_cast<float>(beta1), beta2_f = static_cast<float>(beta2);
    p.n_levels = level;
    p.n_groups = n_groups;
    p.lr = static_cast<float>(lr);
    p.beta1 = beta1_f;
    p.beta2 = beta2_f;
    p.eps = static_cast<float>(eps);
    p.bias_correction1 = static_cast<float>(1.0 - std::pow(static_cast<double>(beta1_f), static_cast<double>(step)));
    p.bias_correction2 = static_cast<float>(1.0 - std::pow(static_cast<double>(beta2_f), static_cast<double>(step)));
    p.max_value_sq = max_value * max_value;
    int device = 0, n_sms = 0;
    cudaGetDevice(&device);
    cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, device);
    const int64_t blocks = std::min<int64_t>((n_groups + zo::block_size - 1) / zo::block_size, static_cast<int64_t>(n_sms) * zo::blocks_per_sm);
    if (blocks == 0) return 0;
    zo::adam_step_kernel<<<static_cast<unsigned>(blocks), zo::block_size, 0, stream>>>(p, level_sums, counter, magnitudes, regularization);
    return status();
}

// fz_sampling.cu -- the C ABI of include/zf_sampling.h: argument validation (the checks of the reference's
// sampling_api.cu:426-678 that do not concern torch dtypes or contiguity) and launches of the fz_sampling.cuh and
// fz_final.cuh kernels.
#include "zf_sampling.h"
#include "fz_final.cuh"
#include "fz_sampling.cuh"
#include "fz_status.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <string>

namespace {

constexpr int kMinIntervals = 2;  // check_n_intervals (sampling_api.cu:443-445)
constexpr int kMaxDirectionDegree = 16;

int check_n_intervals(const int64_t n) {
    if (n < kMinIntervals || n > zf::kMaxSamplingIntervals) return zf::set_error(ZF_ERROR_UNSUPPORTED, "unsupported number of samples per level");
    return ZF_OK;
}

int check_rays(const int64_t n_rays) {
    if (n_rays < 0 || n_rays > INT_MAX) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "invalid number of rays");
    return ZF_OK;
}

int check_degree(const int degree) {
    if (degree < 0 || degree > kMaxDirectionDegree) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "invalid direction encoding degree");
    return ZF_OK;
}

zf::RayWarp ray_warp(const zf_ray_warp& w) { return {w.near, w.far, w.fn_near, w.fn_far, w.power, w.premult, w.y_max}; }

unsigned ray_blocks(const int64_t n_rays) { return static_cast<unsigned>((n_rays + zf::kSamplingRays - 1) / zf::kSamplingRays); }

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

template <typename Args>
int launch(void (*kernel)(Args), const unsigned grid, const unsigned block, const size_t smem, cudaStream_t stream, const Args& args) {
    void* params[] = {const_cast<Args*>(&args)};
    const cudaError_t error = cudaLaunchKernel(reinterpret_cast<const void*>(kernel), dim3(grid), dim3(block), params, smem, stream);
    return error == cudaSuccess ? ZF_OK : zf::set_cuda_error(error, "kernel launch");
}

int launch_new_rays(const zf::NewRaysArgs& a, cudaStream_t stream) {
    if (a.n_rays == 0) return ZF_OK;
    return launch(zf::fz_new_rays_kernel, ray_blocks(a.n_rays), zf::kSamplingRays, zf::new_rays_smem_bytes(a.n_samples, zf::direction_block_width(a.degree)),
                  stream, a);
}

}  // namespace

int64_t zf_direction_block_width(const int direction_degree) { return zf::direction_block_width(direction_degree); }

int zf_initialize_rays(const zf_initialize_rays_args* args, cudaStream_t stream) {
    if (args == nullptr) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "null arguments");
    int status = check_n_intervals(args->n_samples);
    if (status == ZF_OK) status = check_rays(args->n_rays);
    if (status == ZF_OK) status = check_degree(args->direction_degree);
    if (status != ZF_OK) return status;
    if (args->n_rays > 0 && (!args->directions || !args->encoded_directions || !args->sdist || !args->tdist)) {
        return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "initialize_rays: null tensor");
    }
    zf::NewRaysArgs a{};
    a.source = zf::RaySource::Given;
    a.seed = args->seed;
    a.n_rays = args->n_rays;
    a.directions_in = args->directions;
    a.encoded_directions = args->encoded_directions;
    a.encoded_vectors = aligned16(args->encoded_directions);
    a.sdist = args->sdist;
    a.tdist = args->tdist;
    a.degree = args->direction_degree;
    a.n_samples = args->n_samples;
    a.warp = ray_warp(args->warp);
    return launch_new_rays(a, stream);
}

int zf_view_rays(const zf_view_rays_args* args, cudaStream_t stream) {
    if (args == nullptr) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "null arguments");
    int status = check_n_intervals(args->n_samples);
    if (status == ZF_OK) status = check_rays(args->n_rays);
    if (status == ZF_OK) status = check_degree(args->direction_degree);
    if (status != ZF_OK) return status;
    if (args->n_rays > 0 && (!args->pixel_indices || !args->local_directions || !args->c2w || !args->origins || !args->directions || !args->radii
                             || !args->encoded_directions || !args->sdist || !args->tdist)) {
        return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "view_rays: null tensor");
    }
    zf::NewRaysArgs a{};
    a.source = zf::RaySource::View;
    a.seed = -1;
    a.n_rays = args->n_rays;
    a.pixel_indices = args->pixel_indices;
    a.view_radius = args->radius;
    a.local_directions = args->local_directions;
    a.c2w = args->c2w;
    a.origins = args->origins;
    a.directions = args->directions;
    a.radii = args->radii;
    a.encoded_directions = args->encoded_directions;
    a.encoded_vectors = aligned16(args->encoded_directions);
    a.sdist = args->sdist;
    a.tdist = args->tdist;
    a.degree = args->direction_degree;
    a.n_samples = args->n_samples;
    a.warp = ray_warp(args->warp);
    return launch_new_rays(a, stream);
}

int zf_generate_rays(const zf_generate_rays_args* args, cudaStream_t stream) {
    if (args == nullptr) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "null arguments");
    int status = check_n_intervals(args->n_samples);
    if (status == ZF_OK) status = check_rays(args->n_rays);
    if (status == ZF_OK) status = check_degree(args->direction_degree);
    if (status != ZF_OK) return status;
    if (args->n_rays > 0) {
        if (args->n_views < 1 || args->n_pixels < 1) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "generate_rays: empty ray pool");
        if (!args->view_offsets || !args->view_cameras || !args->camera_offsets || !args->local_directions || !args->c2w || !args->camera_radii
            || !args->pool_rgb || !args->origins || !args->directions || !args->radii || !args->rgb || !args->encoded_directions || !args->sdist
            || !args->tdist) {
            return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "generate_rays: null tensor");
        }
    }
    zf::NewRaysArgs a{};
    a.source = zf::RaySource::Pool;
    a.seed = args->seed;
    a.n_rays = args->n_rays;
    a.local_directions = args->local_directions;
    a.c2w = args->c2w;
    a.view_offsets = args->view_offsets;
    a.n_views = args->n_views;
    a.view_cameras = args->view_cameras;
    a.camera_offsets = args->camera_offsets;
    a.camera_radii = args->camera_radii;
    a.pool_rgb = args->pool_rgb;
    a.n_pixels = args->n_pixels;
    a.origins = args->origins;
    a.directions = args->directions;
    a.radii = args->radii;
    a.rgb = args->rgb;
    a.encoded_directions = args->encoded_directions;
    a.encoded_vectors = aligned16(args->encoded_directions);
    a.sdist = args->sdist;
    a.tdist = args->tdist;
    a.degree = args->direction_degree;
    a.n_samples = args->n_samples;
    a.warp = ray_warp(args->warp);
    return launch_new_rays(a, stream);
}

int zf_sample_uniforms(const int64_t seed, const int64_t stream_index, const int64_t n, float* values, cudaStream_t stream) {
    if (n < 0 || (n > 0 && values == nullptr)) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "sample_uniforms: invalid output");
    if (n == 0) return ZF_OK;
    int device = 0, n_sms = 0;
    cudaError_t error = cudaGetDevice(&device);
    if (error == cudaSuccess) error = cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, device);
    if (error != cudaSuccess) return zf::set_cuda_error(error, "device query");
    // grid-stride over at most 8 resident blocks of 256 threads per SM
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, static_cast<int64_t>(n_sms) * 8);
    zf::fz_sample_uniforms_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(static_cast<unsigned long long>(seed),
                                                                                      static_cast<unsigned long long>(stream_index), n, values);
    error = cudaGetLastError();
    return error == cudaSuccess ? ZF_OK : zf::set_cuda_error(error, "kernel launch");
}

int zf_composite_and_resample(const zf_resample_args* args, cudaStream_t stream) {
    if (args == nullptr) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "null arguments");
    int status = check_n_intervals(args->n_samples);
    if (status == ZF_OK) status = check_n_intervals(args->n_intervals);
    if (status == ZF_OK) status = check_rays(args->n_rays);
    if (status != ZF_OK) return status;
    if (args->n_rays == 0) return ZF_OK;
    if (!args->raw_density || !args->sdist || !args->tdist || !args->directions || !args->sdist_next || !args->tdist_next) {
        return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "composite_and_resample: null tensor");
    }
    zf::ResampleArgs a{};
    a.raw_density = args->raw_density;
    a.sdist = args->sdist;
    a.tdist = args->tdist;
    a.directions = args->directions;
    a.weights = args->weights;
    a.sdist_next = args->sdist_next;
    a.tdist_next = args->tdist_next;
    a.n_rays = args->n_rays;
    a.n = args->n_intervals;
    a.n_out = args->n_samples;
    a.anneal = args->anneal;
    a.seed = args->seed;
    a.next_level = args->next_level;
    a.warp = ray_warp(args->warp);
    return launch(zf::fz_composite_and_resample_kernel, ray_blocks(a.n_rays), zf::kSamplingRays,
                  sizeof(float) * zf::resample_smem_floats(a.n, a.n_out), stream, a);
}

int zf_train_final(const zf_train_final_args* args, cudaStream_t stream) {
    if (args == nullptr) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "null arguments");
    int status = check_n_intervals(args->n_intervals);
    if (status == ZF_OK) status = check_rays(args->n_rays);
    if (status != ZF_OK) return status;
    if (args->n_proposal_levels < 0 || args->n_proposal_levels > zf::kMaxProposalLevels || (args->n_proposal_levels > 0 && args->proposals == nullptr)) {
        return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "inconsistent proposal levels");
    }
    zf::TrainFinalArgs a{};
    for (int level = 0; level < args->n_proposal_levels; level++) {
        const zf_proposal_level& p = args->proposals[level];
        status = check_n_intervals(p.n_intervals);
        if (status != ZF_OK) return status;
        if (args->n_rays > 0 && (!p.raw_density || !p.sdist || !p.tdist || !p.weights || !p.raw_density_grad)) {
            return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "train_final: null proposal tensor");
        }
        a.proposals.n_intervals[level] = p.n_intervals;
        a.proposals.raw_density[level] = p.raw_density;
        a.proposals.sdist[level] = p.sdist;
        a.proposals.tdist[level] = p.tdist;
        a.proposals.weights[level] = p.weights;
        a.proposals.raw_density_grad[level] = p.raw_density_grad;
        a.proposals.interlevel_weight[level] = p.interlevel_weight;
        a.proposals.interlevel_blur[level] = p.interlevel_blur;
    }
    a.proposals.n_levels = args->n_proposal_levels;
    if (args->n_rays == 0) return ZF_OK;
    if (!args->nerf_outputs || !args->sdist || !args->tdist || !args->directions || !args->rgb_target || !args->nerf_outputs_grad) {
        return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "train_final: null tensor");
    }
    a.nerf_outputs = args->nerf_outputs;
    a.sdist = args->sdist;
    a.tdist = args->tdist;
    a.directions = args->directions;
    a.seed = static_cast<unsigned long long>(args->seed);
    a.rgb_target = args->rgb_target;
    a.nerf_outputs_grad = args->nerf_outputs_grad;
    a.loss_sums = args->loss_sums;
    a.n = args->n_intervals;
    a.charbonnier_padding = args->charbonnier_padding;
    a.distortion_weight = args->distortion_weight;
    a.distortion_power = args->distortion_power;
    a.distortion_premult = args->distortion_premult;
    a.n_rays = static_cast<int>(args->n_rays);
    a.vectors = reinterpret_cast<uintptr_t>(args->nerf_outputs) % 8 == 0 && aligned16(args->nerf_outputs_grad);
    return launch(zf::fz_train_final_kernel, ray_blocks(args->n_rays), 32, 0, stream, a);
}

int zf_composite_final(const zf_composite_final_args* args, cudaStream_t stream) {
    if (args == nullptr) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "null arguments");
    int status = check_n_intervals(args->n_intervals);
    if (status == ZF_OK) status = check_rays(args->n_rays);
    if (status != ZF_OK) return status;
    if (args->n_rays == 0) return ZF_OK;
    if (!args->nerf_outputs || !args->tdist || !args->directions || !args->background || !args->pixel_indices || !args->rgb) {
        return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "composite_final: null tensor");
    }
    zf::CompositeFinalArgs a{};
    a.nerf_outputs = args->nerf_outputs;
    a.tdist = args->tdist;
    a.directions = args->directions;
    a.background = args->background;
    a.pixel_indices = args->pixel_indices;
    a.rgb = args->rgb;
    a.alpha = args->alpha;
    a.depth = args->depth;
    a.n = args->n_intervals;
    a.n_rays = static_cast<int>(args->n_rays);
    a.use_median_depth = args->use_median_depth;
    a.vectors = reinterpret_cast<uintptr_t>(args->nerf_outputs) % 8 == 0;
    return launch(zf::fz_composite_final_kernel, ray_blocks(args->n_rays), 32, 0, stream, a);
}

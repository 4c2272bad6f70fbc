// torch_ext.cpp -- the PyTorch binding ZipNeRFCudaBackend._C over the C ABI (include/zf_featurize.h, zf_sampling.h,
// zf_optim.h).
//
// Mirrors the reference module (torch_bindings/bindings.cu:14-43) except its NeRF MLP: the attributes grid_max_value
// and nerf_grid_grad_scale, set_rtc_dirs, the class Featurizer with its constructor, n_fp32_grad_rows, forward,
// backward and backward_mlp (featurizer.h:25-82), the sampling functions generate_rays, view_rays, initialize_rays,
// sample_uniforms, composite_and_resample, train_final and composite_final (sampling_api.h:10-90), and the class Adam
// with step and regularization (optimizer_api.h:14-40), with the reference's argument order and meaning, its tensor
// checks (featurizer.cu:127-138, 207-233, 276-283, 318-331; sampling_api.cu:426-678; optimizer_api.cu:123-158) and its
// error text (RuntimeError "ZipNeRF: ..."). Launches go to the current CUDA stream. An empty tensor skips a featurizer
// output, as in the reference. All computation happens in libzf_featurize.so; this file only converts tensors to
// pointers and allocates the outputs the reference's wrappers return.
#include "zf_featurize.h"
#include "zf_mlp.h"
#include "zf_optim.h"
#include "zf_sampling.h"

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/csrc/utils/pybind.h>

#include <pybind11/stl.h>

#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

namespace {

void check_status(const int status) {
    if (status != ZF_OK) throw std::runtime_error(zf_last_error());
}

void check_input(const at::Tensor& tensor, const char* name, const at::ScalarType dtype) {
    if (!tensor.is_cuda() || !tensor.is_contiguous() || tensor.scalar_type() != dtype) {
        throw std::runtime_error(std::string("ZipNeRF: ") + name + " must be a contiguous cuda tensor of the expected type");
    }
}

// row-strided 2D tensors (e.g., column slices of a larger buffer)
void check_rows(const at::Tensor& tensor, const char* name, const at::ScalarType dtype, const int64_t n_rows, const int64_t n_columns) {
    if (!tensor.is_cuda() || tensor.scalar_type() != dtype || tensor.dim() != 2 || tensor.size(0) != n_rows || tensor.size(1) < n_columns || tensor.stride(1) != 1) {
        throw std::runtime_error(std::string("ZipNeRF: ") + name + " has an invalid layout");
    }
}

template <typename T>
T* optional_ptr(const at::Tensor& tensor) {
    return tensor.numel() > 0 ? reinterpret_cast<T*>(tensor.data_ptr()) : nullptr;
}

cudaStream_t current_stream() { return c10::cuda::getCurrentCUDAStream().stream(); }

class Featurizer {
public:
    Featurizer(const int level, const std::vector<int64_t>& level_sizes, const std::vector<int64_t>& level_entries, const int n_features, const int mlp_width) {
        if (level_sizes.size() != level_entries.size()) throw std::runtime_error("ZipNeRF: level_sizes and level_entries differ in length");
        check_status(zf_featurizer_create(level, level_sizes.data(), level_entries.data(), static_cast<int>(level_sizes.size()), n_features, mlp_width, &m_featurizer));
        m_n_features = n_features;
        m_mlp_width = mlp_width;
    }

    ~Featurizer() { zf_featurizer_destroy(m_featurizer); }

    Featurizer(const Featurizer&) = delete;
    Featurizer& operator=(const Featurizer&) = delete;

    int n_output_features() const { return zf_featurizer_n_output_features(m_featurizer); }
    int64_t n_fp32_grad_rows() const { return zf_featurizer_n_fp32_grad_rows(m_featurizer); }

    void forward(const at::Tensor& origins, const at::Tensor& directions, const at::Tensor& radii, const at::Tensor& tdist,
                 const int64_t pattern_seed, const bool interleave, const at::Tensor& table, const at::Tensor& scale_magnitudes,
                 const at::Tensor& w0, const at::Tensor& b0, const at::Tensor& w1, const at::Tensor& b1, at::Tensor& raw_density,
                 at::Tensor& features_float, at::Tensor& features_bf16, const at::Tensor& encoded_directions, at::Tensor& nerf_inputs) {
        zf_forward_args a{};
        fill_rays(origins, directions, radii, tdist, pattern_seed, a.rays);
        const int64_t n_samples = a.rays.n_rays * a.rays.n_intervals;
        check_input(table, "table", at::kFloat);
        check_input(scale_magnitudes, "scale_magnitudes", at::kFloat);
        if (scale_magnitudes.numel() < static_cast<int64_t>(zf_featurizer_n_output_features(m_featurizer) / (m_n_features + 1))) {
            throw std::runtime_error("ZipNeRF: invalid scale_magnitudes");
        }
        a.interleave = interleave ? 1 : 0;
        a.table = table.data_ptr<float>();
        a.table_rows = table.numel() / m_n_features;
        if (table.numel() != zf_featurizer_n_rows(m_featurizer) * m_n_features) throw std::runtime_error("ZipNeRF: invalid table");
        a.scale_magnitudes = scale_magnitudes.data_ptr<float>();
        if (raw_density.numel() > 0) {
            check_input(raw_density, "raw_density", at::kFloat);
            if (raw_density.numel() != n_samples) throw std::runtime_error("ZipNeRF: invalid raw_density");
            check_input(w0, "w0", at::kFloat);
            if (m_mlp_width == 0 || w0.numel() != static_cast<int64_t>(m_mlp_width) * n_output_features()) throw std::runtime_error("ZipNeRF: invalid proposal mlp weights");
            check_input(b0, "b0", at::kFloat);
            check_input(w1, "w1", at::kFloat);
            check_input(b1, "b1", at::kFloat);
            if (b0.numel() != m_mlp_width || w1.numel() != m_mlp_width || b1.numel() < 1) throw std::runtime_error("ZipNeRF: invalid proposal mlp weights");
            a.w0 = w0.data_ptr<float>();
            a.b0 = b0.data_ptr<float>();
            a.w1 = w1.data_ptr<float>();
            a.b1 = b1.data_ptr<float>();
            a.w0_numel = w0.numel();
            a.raw_density = raw_density.data_ptr<float>();
        }
        if (features_float.numel() > 0) {
            check_input(features_float, "features_float", at::kFloat);
            if (features_float.numel() != n_samples * n_output_features()) throw std::runtime_error("ZipNeRF: invalid features_float");
            a.features_float = features_float.data_ptr<float>();
        }
        if (features_bf16.numel() > 0) {
            check_input(features_bf16, "features_bf16", at::kBFloat16);
            if (features_bf16.dim() != 2 || features_bf16.size(0) != n_samples || features_bf16.size(1) < n_output_features()) {
                throw std::runtime_error("ZipNeRF: invalid features_bf16");
            }
            a.features_bf16 = reinterpret_cast<uint16_t*>(features_bf16.data_ptr());
            a.features_bf16_width = features_bf16.size(1);
        }
        if (nerf_inputs.numel() > 0) {
            check_input(nerf_inputs, "nerf_inputs", at::kBFloat16);
            check_input(encoded_directions, "encoded_directions", at::kBFloat16);
            if (nerf_inputs.dim() != 2 || encoded_directions.dim() != 2 || nerf_inputs.size(0) != n_samples || nerf_inputs.size(1) < encoded_directions.size(1) ||
                encoded_directions.size(0) != a.rays.n_rays) {
                throw std::runtime_error("ZipNeRF: invalid nerf_inputs");
            }
            a.nerf_inputs = reinterpret_cast<uint16_t*>(nerf_inputs.data_ptr());
            a.nerf_inputs_width = nerf_inputs.size(1);
            a.encoded_directions = reinterpret_cast<const uint16_t*>(encoded_directions.data_ptr());
            a.encoded_width = encoded_directions.size(1);
        }
        if (n_samples == 0) return;
        const c10::cuda::CUDAGuard guard(origins.device());
        check_status(zf_featurize_forward(m_featurizer, &a, current_stream()));
    }

    void backward(const at::Tensor& origins, const at::Tensor& directions, const at::Tensor& radii, const at::Tensor& tdist, const int64_t pattern_seed,
                  const at::Tensor& grad_features, at::Tensor& grad_table, at::Tensor& grad_table_half) {
        check_input(grad_table, "grad_table", at::kFloat);
        check_input(grad_table_half, "grad_table_half", at::kHalf);
        const int64_t split = n_fp32_grad_rows();
        const int64_t rows = zf_featurizer_n_rows(m_featurizer);
        if (grad_table.numel() != split * m_n_features || grad_table_half.numel() != (rows - split) * m_n_features) {
            throw std::runtime_error("ZipNeRF: invalid grid gradient split");
        }
        zf_backward_args a{};
        fill_rays(origins, directions, radii, tdist, pattern_seed, a.rays);
        const int64_t n_samples = a.rays.n_rays * a.rays.n_intervals;
        check_rows(grad_features, "grad_features", at::kBFloat16, n_samples, n_output_features());
        if (n_samples == 0) return;
        a.grad_features = reinterpret_cast<const uint16_t*>(grad_features.data_ptr());
        a.grad_features_cols = grad_features.size(1);
        a.grad_features_stride = grad_features.stride(0);
        a.grad_table = optional_ptr<float>(grad_table);
        a.grad_table_numel = grad_table.numel();
        a.grad_table_half = optional_ptr<uint16_t>(grad_table_half);
        a.grad_table_half_numel = grad_table_half.numel();
        const c10::cuda::CUDAGuard guard(origins.device());
        check_status(zf_featurize_backward(m_featurizer, &a, current_stream()));
    }

    void backward_mlp(const at::Tensor& origins, const at::Tensor& directions, const at::Tensor& radii, const at::Tensor& tdist, const int64_t pattern_seed,
                      const at::Tensor& features, const at::Tensor& grad_raw_density, const at::Tensor& w0, const at::Tensor& b0, const at::Tensor& w1,
                      at::Tensor& grad_table, at::Tensor& grad_w0, at::Tensor& grad_b0, at::Tensor& grad_w1, at::Tensor& grad_b1) {
        zf_backward_mlp_args a{};
        fill_rays(origins, directions, radii, tdist, pattern_seed, a.rays);
        const int64_t n_samples = a.rays.n_rays * a.rays.n_intervals;
        check_input(features, "features", at::kFloat);
        check_input(grad_raw_density, "grad_raw_density", at::kFloat);
        if (features.numel() != n_samples * n_output_features() || grad_raw_density.numel() != n_samples) throw std::runtime_error("ZipNeRF: invalid backward_mlp inputs");
        check_input(w0, "w0", at::kFloat);
        check_input(b0, "b0", at::kFloat);
        check_input(w1, "w1", at::kFloat);
        check_input(grad_table, "grad_table", at::kFloat);
        check_input(grad_w0, "grad_w0", at::kFloat);
        check_input(grad_b0, "grad_b0", at::kFloat);
        check_input(grad_w1, "grad_w1", at::kFloat);
        check_input(grad_b1, "grad_b1", at::kFloat);
        if (m_mlp_width == 0 || w0.numel() != static_cast<int64_t>(m_mlp_width) * n_output_features() || grad_w0.numel() != w0.numel()) {
            throw std::runtime_error("ZipNeRF: invalid proposal mlp weights");
        }
        if (b0.numel() != m_mlp_width || w1.numel() != m_mlp_width || grad_b0.numel() != m_mlp_width || grad_w1.numel() != m_mlp_width || grad_b1.numel() < 1) {
            throw std::runtime_error("ZipNeRF: invalid proposal mlp weights");
        }
        if (n_samples == 0) return;
        a.features = features.data_ptr<float>();
        a.features_numel = features.numel();
        a.grad_raw_density = grad_raw_density.data_ptr<float>();
        a.grad_raw_density_numel = grad_raw_density.numel();
        a.w0 = w0.data_ptr<float>();
        a.b0 = b0.data_ptr<float>();
        a.w1 = w1.data_ptr<float>();
        a.w0_numel = w0.numel();
        a.grad_table = grad_table.data_ptr<float>();
        a.grad_table_numel = grad_table.numel();
        a.grad_w0 = grad_w0.data_ptr<float>();
        a.grad_w0_numel = grad_w0.numel();
        a.grad_b0 = grad_b0.data_ptr<float>();
        a.grad_w1 = grad_w1.data_ptr<float>();
        a.grad_b1 = grad_b1.data_ptr<float>();
        const c10::cuda::CUDAGuard guard(origins.device());
        // the workspace between the MLP and the scatter kernels comes from PyTorch's caching allocator (stream-ordered on
        // the current stream, returned to the cache when this call's tensor goes out of scope)
        const int64_t workspace_bytes = zf_featurize_backward_mlp_workspace_size(m_featurizer, n_samples);
        at::Tensor workspace = at::empty({workspace_bytes}, origins.options().dtype(at::kByte));
        a.workspace = workspace.data_ptr();
        a.workspace_bytes = workspace_bytes;
        check_status(zf_featurize_backward_mlp(m_featurizer, &a, current_stream()));
    }

    // intermediate values of the given samples (no counterpart in the reference): a dict of x [n, 6, 3],
    // scale [n, 6], contracted [n, 6], n_groups [n, L], rows [n, L, 6, 8] (int64), weights [n, L, 6, 8]
    pybind11::dict debug(const at::Tensor& origins, const at::Tensor& directions, const at::Tensor& radii, const at::Tensor& tdist,
                         const int64_t pattern_seed, const at::Tensor& samples) {
        zf_rays rays{};
        fill_rays(origins, directions, radii, tdist, pattern_seed, rays);
        check_input(samples, "samples", at::kInt);
        const int64_t n = samples.numel();
        const int L = n_output_features() / (m_n_features + 1);
        const auto opts = origins.options();
        at::Tensor x = at::zeros({n, 6, 3}, opts), scale = at::zeros({n, 6}, opts), weights = at::zeros({n, L, 6, 8}, opts);
        at::Tensor contracted = at::zeros({n, 6}, opts.dtype(at::kInt)), n_groups = at::zeros({n, L}, opts.dtype(at::kInt)), rows = at::zeros({n, L, 6, 8}, opts.dtype(at::kInt));
        const c10::cuda::CUDAGuard guard(origins.device());
        check_status(zf_featurize_debug(m_featurizer, &rays, reinterpret_cast<const uint32_t*>(samples.data_ptr()), n, x.data_ptr<float>(), scale.data_ptr<float>(),
                                        contracted.data_ptr<int32_t>(), n_groups.data_ptr<int32_t>(), reinterpret_cast<uint32_t*>(rows.data_ptr()),
                                        weights.data_ptr<float>(), current_stream()));
        pybind11::dict out;
        out["x"] = x;
        out["scale"] = scale;
        out["contracted"] = contracted;
        out["n_groups"] = n_groups;
        out["rows"] = rows.to(at::kLong).bitwise_and(0xFFFFFFFFLL);
        out["weights"] = weights;
        return out;
    }

private:
    void fill_rays(const at::Tensor& origins, const at::Tensor& directions, const at::Tensor& radii, const at::Tensor& tdist, const int64_t pattern_seed, zf_rays& rays) const {
        check_input(origins, "origins", at::kFloat);
        check_input(directions, "directions", at::kFloat);
        check_input(radii, "radii", at::kFloat);
        check_input(tdist, "tdist", at::kFloat);
        if (tdist.dim() != 2 || tdist.size(1) < 2) throw std::runtime_error("ZipNeRF: invalid tdist");
        const int64_t n_rays = tdist.size(0);
        if (origins.numel() != 3 * n_rays || directions.numel() != 3 * n_rays || radii.numel() != n_rays) throw std::runtime_error("ZipNeRF: invalid rays");
        rays.origins = origins.data_ptr<float>();
        rays.directions = directions.data_ptr<float>();
        rays.radii = radii.data_ptr<float>();
        rays.tdist = tdist.data_ptr<float>();
        rays.n_rays = n_rays;
        rays.n_intervals = tdist.size(1) - 1;
        rays.pattern_seed = pattern_seed;
        rays.sample_offset = m_sample_offset;
    }

public:
    // batch index of the first sample of this featurizer's calls, for the pattern random numbers (0: the reference's
    // behaviour; a data-parallel shard sets the index of its first sample in the global batch)
    int64_t sample_offset() const { return m_sample_offset; }
    void set_sample_offset(const int64_t offset) {
        if (offset < 0) throw std::runtime_error("ZipNeRF: sample_offset must not be negative");
        m_sample_offset = offset;
    }

private:

    zf_featurizer* m_featurizer = nullptr;
    int64_t m_sample_offset = 0;
    int m_n_features = 0;
    int m_mlp_width = 0;
};

// the reference compiles its featurization kernels at runtime from a source directory into a cache directory
// (featurizer.cu:112-117); these kernels are compiled ahead of time, so the directories are accepted and unused
void set_rtc_dirs(const std::string&, const std::string&) {}

// ---------------------------------------------------------------------------------------------------------------------
// sampling (sampling_api.h:10-58, sampling_api.cu:426-578): the reference's wrappers allocate and return the outputs

zf_ray_warp make_ray_warp(const std::vector<double>& values) {
    if (values.size() != 7) throw std::runtime_error("ZipNeRF: invalid ray warp");
    return {static_cast<float>(values[0]), static_cast<float>(values[1]), static_cast<float>(values[2]), static_cast<float>(values[3]),
            static_cast<float>(values[4]), static_cast<float>(values[5]), static_cast<float>(values[6])};
}

void check_n_intervals(const int64_t n) {
    if (n < 2 || n > 64) throw std::runtime_error("ZipNeRF: unsupported number of samples per level");
}

uint16_t* bf16_ptr(const at::Tensor& tensor) { return reinterpret_cast<uint16_t*>(tensor.data_ptr()); }

std::vector<at::Tensor> generate_rays(const int64_t seed, const int n_rays, const at::Tensor& view_offsets, const at::Tensor& view_cameras,
                                      const at::Tensor& camera_offsets, const at::Tensor& local_directions, const at::Tensor& c2w,
                                      const at::Tensor& camera_radii, const at::Tensor& pool_rgb, const int direction_degree, const int n_samples,
                                      const std::vector<double>& ray_warp) {
    check_input(view_offsets, "view_offsets", at::kLong);
    check_input(view_cameras, "view_cameras", at::kInt);
    check_input(camera_offsets, "camera_offsets", at::kLong);
    check_input(local_directions, "local_directions", at::kFloat);
    check_input(c2w, "c2w", at::kFloat);
    check_input(camera_radii, "camera_radii", at::kFloat);
    check_input(pool_rgb, "pool_rgb", at::kByte);
    check_n_intervals(n_samples);
    const zf_ray_warp warp = make_ray_warp(ray_warp);
    const int64_t n_views = view_cameras.size(0);
    if (n_rays < 0 || view_offsets.numel() != n_views + 1 || c2w.numel() != 12 * n_views) throw std::runtime_error("ZipNeRF: invalid ray pool");
    const auto options = local_directions.options();
    at::Tensor origins = at::empty({n_rays, 3}, options), directions = at::empty({n_rays, 3}, options), radii = at::empty({n_rays}, options);
    at::Tensor rgb = at::empty({n_rays, 3}, options);
    at::Tensor encoded = at::empty({n_rays, zf_direction_block_width(direction_degree)}, options.dtype(at::kBFloat16));
    at::Tensor sdist = at::empty({n_rays, n_samples + 1}, options), tdist = at::empty({n_rays, n_samples + 1}, options);
    zf_generate_rays_args a{};
    a.seed = seed;
    a.n_rays = n_rays;
    a.view_offsets = view_offsets.data_ptr<int64_t>();
    a.n_views = static_cast<int>(n_views);
    a.view_cameras = view_cameras.data_ptr<int32_t>();
    a.camera_offsets = camera_offsets.data_ptr<int64_t>();
    a.local_directions = local_directions.data_ptr<float>();
    a.c2w = c2w.data_ptr<float>();
    a.camera_radii = camera_radii.data_ptr<float>();
    a.pool_rgb = pool_rgb.data_ptr<uint8_t>();
    a.n_pixels = pool_rgb.size(0);
    a.direction_degree = direction_degree;
    a.n_samples = n_samples;
    a.warp = warp;
    a.origins = origins.data_ptr<float>();
    a.directions = directions.data_ptr<float>();
    a.radii = radii.data_ptr<float>();
    a.rgb = rgb.data_ptr<float>();
    a.encoded_directions = bf16_ptr(encoded);
    a.sdist = sdist.data_ptr<float>();
    a.tdist = tdist.data_ptr<float>();
    const c10::cuda::CUDAGuard guard(local_directions.device());
    check_status(zf_generate_rays(&a, current_stream()));
    return {origins, directions, radii, rgb, encoded, sdist, tdist};
}

std::vector<at::Tensor> view_rays(const at::Tensor& pixel_indices, const at::Tensor& local_directions, const at::Tensor& c2w, const double radius,
                                  const int direction_degree, const int n_samples, const std::vector<double>& ray_warp) {
    check_input(pixel_indices, "pixel_indices", at::kLong);
    check_input(local_directions, "local_directions", at::kFloat);
    check_input(c2w, "c2w", at::kFloat);
    if (c2w.numel() != 12) throw std::runtime_error("ZipNeRF: c2w must be a 3x4 matrix");
    check_n_intervals(n_samples);
    const zf_ray_warp warp = make_ray_warp(ray_warp);
    const int64_t n_rays = pixel_indices.numel();
    const auto options = local_directions.options();
    at::Tensor origins = at::empty({n_rays, 3}, options), directions = at::empty({n_rays, 3}, options), radii = at::empty({n_rays}, options);
    at::Tensor encoded = at::empty({n_rays, zf_direction_block_width(direction_degree)}, options.dtype(at::kBFloat16));
    at::Tensor sdist = at::empty({n_rays, n_samples + 1}, options), tdist = at::empty({n_rays, n_samples + 1}, options);
    zf_view_rays_args a{};
    a.pixel_indices = pixel_indices.data_ptr<int64_t>();
    a.n_rays = n_rays;
    a.local_directions = local_directions.data_ptr<float>();
    a.c2w = c2w.data_ptr<float>();
    a.radius = static_cast<float>(radius);
    a.direction_degree = direction_degree;
    a.n_samples = n_samples;
    a.warp = warp;
    a.origins = origins.data_ptr<float>();
    a.directions = directions.data_ptr<float>();
    a.radii = radii.data_ptr<float>();
    a.encoded_directions = bf16_ptr(encoded);
    a.sdist = sdist.data_ptr<float>();
    a.tdist = tdist.data_ptr<float>();
    const c10::cuda::CUDAGuard guard(local_directions.device());
    check_status(zf_view_rays(&a, current_stream()));
    return {origins, directions, radii, encoded, sdist, tdist};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> initialize_rays(const int64_t seed, const at::Tensor& directions, const int direction_degree,
                                                               const int n_samples, const std::vector<double>& ray_warp) {
    check_input(directions, "directions", at::kFloat);
    check_n_intervals(n_samples);
    const zf_ray_warp warp = make_ray_warp(ray_warp);
    const int64_t n_rays = directions.size(0);
    if (directions.numel() != 3 * n_rays) throw std::runtime_error("ZipNeRF: invalid rays");
    const auto options = directions.options();
    at::Tensor encoded = at::empty({n_rays, zf_direction_block_width(direction_degree)}, options.dtype(at::kBFloat16));
    at::Tensor sdist = at::empty({n_rays, n_samples + 1}, options), tdist = at::empty({n_rays, n_samples + 1}, options);
    zf_initialize_rays_args a{};
    a.seed = seed;
    a.directions = directions.data_ptr<float>();
    a.n_rays = n_rays;
    a.direction_degree = direction_degree;
    a.n_samples = n_samples;
    a.warp = warp;
    a.encoded_directions = bf16_ptr(encoded);
    a.sdist = sdist.data_ptr<float>();
    a.tdist = tdist.data_ptr<float>();
    const c10::cuda::CUDAGuard guard(directions.device());
    check_status(zf_initialize_rays(&a, current_stream()));
    return {encoded, sdist, tdist};
}

at::Tensor sample_uniforms(const int64_t seed, const int64_t stream, const int64_t n) {
    if (n < 0) throw std::runtime_error("ZipNeRF: invalid number of uniforms");
    at::Tensor values = at::empty({n}, at::TensorOptions().dtype(at::kFloat).device(at::kCUDA));
    const c10::cuda::CUDAGuard guard(values.device());
    check_status(zf_sample_uniforms(seed, stream, n, values.data_ptr<float>(), current_stream()));
    return values;
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> composite_and_resample(const at::Tensor& raw_density, const at::Tensor& sdist, const at::Tensor& tdist,
                                                                      const at::Tensor& directions, const double anneal, const int n_samples,
                                                                      const int64_t seed, const int next_level, const std::vector<double>& ray_warp) {
    check_input(raw_density, "raw_density", at::kFloat);
    check_input(sdist, "sdist", at::kFloat);
    check_input(tdist, "tdist", at::kFloat);
    check_input(directions, "directions", at::kFloat);
    check_n_intervals(n_samples);
    if (raw_density.dim() != 2) throw std::runtime_error("ZipNeRF: invalid raw_density");
    const int64_t n_rays = raw_density.size(0), n_intervals = raw_density.size(1);
    check_n_intervals(n_intervals);
    if (sdist.numel() != n_rays * (n_intervals + 1) || tdist.numel() != n_rays * (n_intervals + 1) || directions.numel() != 3 * n_rays) {
        throw std::runtime_error("ZipNeRF: invalid composite_and_resample inputs");
    }
    const zf_ray_warp warp = make_ray_warp(ray_warp);
    at::Tensor weights = at::empty_like(raw_density);
    at::Tensor sdist_next = at::empty({n_rays, n_samples + 1}, raw_density.options()), tdist_next = at::empty({n_rays, n_samples + 1}, raw_density.options());
    zf_resample_args a{};
    a.raw_density = raw_density.data_ptr<float>();
    a.sdist = sdist.data_ptr<float>();
    a.tdist = tdist.data_ptr<float>();
    a.directions = directions.data_ptr<float>();
    a.n_rays = n_rays;
    a.n_intervals = static_cast<int>(n_intervals);
    a.anneal = static_cast<float>(anneal);
    a.n_samples = n_samples;
    a.seed = seed;
    a.next_level = next_level;
    a.warp = warp;
    a.weights = weights.data_ptr<float>();
    a.sdist_next = sdist_next.data_ptr<float>();
    a.tdist_next = tdist_next.data_ptr<float>();
    const c10::cuda::CUDAGuard guard(raw_density.device());
    check_status(zf_composite_and_resample(&a, current_stream()));
    return {weights, sdist_next, tdist_next};
}

std::tuple<at::Tensor, std::vector<at::Tensor>, at::Tensor> train_final(
    const at::Tensor& nerf_outputs, const at::Tensor& sdist, const at::Tensor& tdist, const std::vector<at::Tensor>& proposal_raw_densities,
    const std::vector<at::Tensor>& proposal_sdists, const std::vector<at::Tensor>& proposal_tdists, const std::vector<at::Tensor>& proposal_weights,
    const at::Tensor& directions, const int64_t seed, const at::Tensor& rgb_target, const double charbonnier_padding,
    const std::vector<double>& interlevel_weights, const std::vector<double>& interlevel_blurs, const double distortion_weight,
    const double distortion_power, const double distortion_premult, const bool compute_loss_sums) {
    check_input(nerf_outputs, "nerf_outputs", at::kBFloat16);
    check_input(sdist, "sdist", at::kFloat);
    check_input(tdist, "tdist", at::kFloat);
    check_input(directions, "directions", at::kFloat);
    check_input(rgb_target, "rgb_target", at::kFloat);
    if (tdist.dim() != 2) throw std::runtime_error("ZipNeRF: invalid tdist");
    const int64_t n_rays = tdist.size(0), n_intervals = tdist.size(1) - 1;
    check_n_intervals(n_intervals);
    if (nerf_outputs.numel() != n_rays * n_intervals * 8) throw std::runtime_error("ZipNeRF: invalid nerf_outputs");
    if (sdist.numel() != tdist.numel() || directions.numel() != 3 * n_rays || rgb_target.numel() != 3 * n_rays) {
        throw std::runtime_error("ZipNeRF: invalid train_final inputs");
    }
    const size_t n_levels = proposal_raw_densities.size();
    if (n_levels > 4 || proposal_sdists.size() != n_levels || proposal_tdists.size() != n_levels || proposal_weights.size() != n_levels
        || interlevel_weights.size() != n_levels || interlevel_blurs.size() != n_levels) {
        throw std::runtime_error("ZipNeRF: inconsistent proposal levels");
    }
    std::vector<at::Tensor> grads;
    std::vector<zf_proposal_level> levels(n_levels);
    for (size_t level = 0; level < n_levels; level++) {
        check_input(proposal_raw_densities[level], "proposal_raw_density", at::kFloat);
        check_input(proposal_sdists[level], "proposal_sdist", at::kFloat);
        check_input(proposal_tdists[level], "proposal_tdist", at::kFloat);
        check_input(proposal_weights[level], "proposal_weights", at::kFloat);
        const at::Tensor& raw = proposal_raw_densities[level];
        if (raw.dim() != 2 || raw.size(0) != n_rays) throw std::runtime_error("ZipNeRF: inconsistent proposal levels");
        const int64_t n_p = raw.size(1);
        check_n_intervals(n_p);
        if (proposal_sdists[level].numel() != n_rays * (n_p + 1) || proposal_tdists[level].numel() != n_rays * (n_p + 1)
            || proposal_weights[level].numel() != n_rays * n_p) {
            throw std::runtime_error("ZipNeRF: inconsistent proposal levels");
        }
        grads.push_back(at::empty_like(raw));
        levels[level] = {static_cast<int>(n_p), raw.data_ptr<float>(), proposal_sdists[level].data_ptr<float>(), proposal_tdists[level].data_ptr<float>(),
                         proposal_weights[level].data_ptr<float>(), grads.back().data_ptr<float>(), static_cast<float>(interlevel_weights[level]),
                         static_cast<float>(interlevel_blurs[level])};
    }
    at::Tensor nerf_outputs_grad = at::empty_like(nerf_outputs);
    at::Tensor loss_sums = compute_loss_sums ? at::zeros({4}, tdist.options()) : at::Tensor();
    zf_train_final_args a{};
    a.nerf_outputs = bf16_ptr(nerf_outputs);
    a.sdist = sdist.data_ptr<float>();
    a.tdist = tdist.data_ptr<float>();
    a.n_rays = n_rays;
    a.n_intervals = static_cast<int>(n_intervals);
    a.proposals = levels.data();
    a.n_proposal_levels = static_cast<int>(n_levels);
    a.directions = directions.data_ptr<float>();
    a.seed = seed;
    a.rgb_target = rgb_target.data_ptr<float>();
    a.charbonnier_padding = static_cast<float>(charbonnier_padding);
    a.distortion_weight = static_cast<float>(distortion_weight);
    a.distortion_power = static_cast<float>(distortion_power);
    a.distortion_premult = static_cast<float>(distortion_premult);
    a.nerf_outputs_grad = bf16_ptr(nerf_outputs_grad);
    a.loss_sums = compute_loss_sums ? loss_sums.data_ptr<float>() : nullptr;
    const c10::cuda::CUDAGuard guard(tdist.device());
    check_status(zf_train_final(&a, current_stream()));
    return {nerf_outputs_grad, grads, loss_sums};
}

void composite_final(const at::Tensor& nerf_outputs, const at::Tensor& tdist, const at::Tensor& directions, const at::Tensor& background,
                     const at::Tensor& pixel_indices, at::Tensor& rgb, at::Tensor& alpha, at::Tensor& depth, const bool use_median_depth) {
    check_input(nerf_outputs, "nerf_outputs", at::kBFloat16);
    check_input(tdist, "tdist", at::kFloat);
    check_input(directions, "directions", at::kFloat);
    check_input(background, "background", at::kFloat);
    check_input(pixel_indices, "pixel_indices", at::kLong);
    check_input(rgb, "rgb", at::kFloat);
    if (alpha.numel() > 0) check_input(alpha, "alpha", at::kFloat);
    if (depth.numel() > 0) check_input(depth, "depth", at::kFloat);
    if (tdist.dim() != 2) throw std::runtime_error("ZipNeRF: invalid tdist");
    const int64_t n_rays = tdist.size(0), n_intervals = tdist.size(1) - 1;
    check_n_intervals(n_intervals);
    if (nerf_outputs.numel() != n_rays * n_intervals * 8 || pixel_indices.numel() != n_rays) throw std::runtime_error("ZipNeRF: invalid composite_final inputs");
    if (directions.numel() != 3 * n_rays || background.numel() < 3) throw std::runtime_error("ZipNeRF: invalid composite_final inputs");
    zf_composite_final_args a{};
    a.nerf_outputs = bf16_ptr(nerf_outputs);
    a.tdist = tdist.data_ptr<float>();
    a.n_rays = n_rays;
    a.n_intervals = static_cast<int>(n_intervals);
    a.directions = directions.data_ptr<float>();
    a.background = background.data_ptr<float>();
    a.pixel_indices = pixel_indices.data_ptr<int64_t>();
    a.rgb = rgb.data_ptr<float>();
    a.alpha = optional_ptr<float>(alpha);
    a.depth = optional_ptr<float>(depth);
    a.use_median_depth = use_median_depth ? 1 : 0;
    const c10::cuda::CUDAGuard guard(tdist.device());
    check_status(zf_composite_final(&a, current_stream()));
}

// the ReLU backward of a bf16 layer with its bias gradient (no counterpart in the reference module: its NeRF MLP does
// this in cuBLASLt epilogues); grad [n, c] masked in place by activation [n, c] (row-strided), bias_grad += column sums
void relu_backward_(at::Tensor& grad, const at::Tensor& activation, const at::Tensor& bias_grad) {
    if (!grad.is_cuda() || grad.scalar_type() != at::kBFloat16 || grad.dim() != 2 || grad.stride(1) != 1 || !activation.is_cuda()
        || activation.scalar_type() != at::kBFloat16 || activation.dim() != 2 || activation.stride(1) != 1 || activation.size(0) != grad.size(0)
        || activation.size(1) != grad.size(1)) {
        throw std::runtime_error("ZipNeRF: relu_backward_ needs matching 2D bf16 cuda tensors with unit column stride");
    }
    float* bias = nullptr;
    if (bias_grad.numel() > 0) {
        check_input(bias_grad, "bias_grad", at::kFloat);
        if (bias_grad.numel() != grad.size(1)) throw std::runtime_error("ZipNeRF: relu_backward_ bias_grad has the wrong size");
        bias = bias_grad.data_ptr<float>();
    }
    const c10::cuda::CUDAGuard guard(grad.device());
    check_status(zf_relu_backward_bf16(bf16_ptr(grad), grad.stride(0), reinterpret_cast<const uint16_t*>(activation.data_ptr()), activation.stride(0),
                                       grad.size(0), static_cast<int>(grad.size(1)), bias, current_stream()));
}

// ---------------------------------------------------------------------------------------------------------------------
// Adam (optimizer_api.h:14-40, optimizer_api.cu:123-221): the tensor checks and messages of the reference; the object
// keeps the tensors it updates alive

void check_adam_buffer(const at::Tensor& tensor, const char* name, const bool allow_half) {
    const bool valid_type = tensor.scalar_type() == at::kFloat || (allow_half && tensor.scalar_type() == at::kHalf);
    if (!tensor.is_cuda() || !tensor.is_contiguous() || !valid_type || tensor.numel() % 4 != 0) {
        throw std::runtime_error(std::string("ZipNeRF: ") + name + " must be a contiguous float (or half) cuda tensor with a multiple of four elements");
    }
}

class Adam {
public:
    Adam(const std::vector<at::Tensor>& params, const std::vector<at::Tensor>& grads, const std::vector<double>& grad_scales,
         const std::vector<std::vector<int64_t>>& level_offsets, const double reg_weight, const double max_value, const double beta1,
         const double beta2, const double eps, const at::Tensor& magnitudes)
        : m_params(params), m_grads(grads), m_magnitudes(magnitudes) {
        const size_t n = params.size();
        if (n == 0 || n > 8 || grads.size() != n || grad_scales.size() != n || level_offsets.size() != n) {
            throw std::runtime_error("ZipNeRF: invalid optimizer buffers");
        }
        std::vector<zf_adam_buffer> buffers(n);
        for (size_t b = 0; b < n; b++) {
            check_adam_buffer(params[b], "param", false);
            check_adam_buffer(grads[b], "grad", true);
            if (grads[b].numel() != params[b].numel()) throw std::runtime_error("ZipNeRF: optimizer gradient size mismatch");
            buffers[b] = {params[b].data_ptr<float>(), grads[b].data_ptr(), grads[b].scalar_type() == at::kHalf ? 1 : 0, params[b].numel(),
                          grad_scales[b], level_offsets[b].data(), static_cast<int>(level_offsets[b].size())};
        }
        if (!magnitudes.is_cuda() || !magnitudes.is_contiguous() || magnitudes.scalar_type() != at::kFloat) {
            throw std::runtime_error("ZipNeRF: magnitudes must be a contiguous float cuda tensor with one entry per level");
        }
        m_regularization = at::zeros({}, params.front().options());
        const c10::cuda::CUDAGuard guard(params.front().device());
        check_status(zf_adam_create(buffers.data(), static_cast<int>(n), reg_weight, max_value, beta1, beta2, eps, m_magnitudes.data_ptr<float>(),
                                    m_magnitudes.numel(), m_regularization.data_ptr<float>(), &m_adam));
    }

    ~Adam() { zf_adam_destroy(m_adam); }

    Adam(const Adam&) = delete;
    Adam& operator=(const Adam&) = delete;

    void step(const double lr) {
        const c10::cuda::CUDAGuard guard(m_params.front().device());
        check_status(zf_adam_step(m_adam, lr, current_stream()));
    }

    at::Tensor regularization() const { return m_regularization; }

    // copies of one buffer's moments (no counterpart in the reference, whose moments are private)
    std::tuple<at::Tensor, at::Tensor> state(const int buffer) const {
        float* exp_avg = nullptr;
        float* exp_avg_sq = nullptr;
        int64_t steps = 0;
        check_status(zf_adam_state(m_adam, buffer, &exp_avg, &exp_avg_sq, &steps));
        const at::Tensor& param = m_params[buffer];
        return {at::from_blob(exp_avg, {param.numel()}, param.options()).clone(), at::from_blob(exp_avg_sq, {param.numel()}, param.options()).clone()};
    }

private:
    std::vector<at::Tensor> m_params, m_grads;
    at::Tensor m_magnitudes, m_regularization;
    zf_adam* m_adam = nullptr;
};

}  // namespace

PYBIND11_MODULE(_C, m) {
    m.attr("grid_max_value") = zf_grid_max_value();
    m.attr("nerf_grid_grad_scale") = zf_nerf_grid_grad_scale();
    m.def("set_rtc_dirs", &set_rtc_dirs);
    pybind11::class_<Featurizer>(m, "Featurizer")
        .def(pybind11::init<int, const std::vector<int64_t>&, const std::vector<int64_t>&, int, int>())
        .def_property_readonly("n_fp32_grad_rows", &Featurizer::n_fp32_grad_rows)
        .def_property_readonly("n_output_features", &Featurizer::n_output_features)
        .def_property("sample_offset", &Featurizer::sample_offset, &Featurizer::set_sample_offset)
        .def("forward", &Featurizer::forward)
        .def("backward", &Featurizer::backward)
        .def("backward_mlp", &Featurizer::backward_mlp)
        .def("debug", &Featurizer::debug);
    pybind11::class_<Adam>(m, "Adam")
        .def(pybind11::init<const std::vector<at::Tensor>&, const std::vector<at::Tensor>&, const std::vector<double>&,
                            const std::vector<std::vector<int64_t>>&, double, double, double, double, double, const at::Tensor&>())
        .def("step", &Adam::step)
        .def("regularization", &Adam::regularization)
        .def("state", &Adam::state);
    m.def("generate_rays", &generate_rays);
    m.def("view_rays", &view_rays);
    m.def("initialize_rays", &initialize_rays);
    m.def("sample_uniforms", &sample_uniforms);
    m.def("composite_and_resample", &composite_and_resample);
    m.def("train_final", &train_final);
    m.def("composite_final", &composite_final);
    m.def("relu_backward_", &relu_backward_);
}

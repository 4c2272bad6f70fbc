// fz_capi.cu -- the C ABI of include/zf_featurize.h: featurizer objects, argument validation (the checks of the
// reference's featurizer.cu:127-155,188-355, minus the torch dtype/contiguity checks that the torch binding makes),
// kernel selection from the ahead-of-time table, and launches on the caller's stream.
#include "zf_featurize.h"
#include "fz_kernel_set.h"
#include "fz_status.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

// the instantiation objects (fz_inst.cu); weak, so that a partial development build (build.py --subset) links and
// reports the missing instantiations as unsupported
#define ZF_DECLARE_KSET(F) extern "C" const zf::KernelSet ZF_KSET_NAME(F) __attribute__((weak));
ZF_DECLARE_KSET(1) ZF_DECLARE_KSET(2) ZF_DECLARE_KSET(3) ZF_DECLARE_KSET(4)
#undef ZF_DECLARE_KSET
#define ZF_DECLARE_MLP_KSET(F, P) extern "C" const zf::MlpKernelSet ZF_MLP_KSET_NAME(F, P) __attribute__((weak));
ZF_FOR_EACH_MLP(ZF_DECLARE_MLP_KSET)
#undef ZF_DECLARE_MLP_KSET
extern "C" void (*const zf_debug_kernel)(zf::GridParams, zf::DebugArgs) __attribute__((weak));
extern "C" void (*const zf_check_erf_kernel)(uint32_t, uint32_t, unsigned long long*, uint32_t*) __attribute__((weak));

namespace {

using zf::kMaxFeatures;
using zf::kMaxLevels;

// Level passes. A grid whose rows exceed the L2 (the NeRF grid: 240 MB of fp32 table rows) is featurized a few levels
// at a time, so that a pass's random row reads (forward) or gradient atomics (backward) hit the L2 instead of DRAM;
// each pass recomputes its intervals' multisamples. The budgets are the randomly accessed bytes of one pass, measured
// on the B200 (126 MB L2) for the NeRF grid of 10 levels, 16-8192, 2^21 rows: the forward is fastest with one 32 MB
// table per pass (7 passes; two tables per pass were 13 % slower), the backward with up to four 16 MB fp16 gradient
// slices per pass (2 passes; 32, 48 and 100 MB passes were 2-6 % slower).
#ifndef ZF_FORWARD_PASS_BYTES
#define ZF_FORWARD_PASS_BYTES (40ll << 20)
#endif
#ifndef ZF_BACKWARD_PASS_BYTES
#define ZF_BACKWARD_PASS_BYTES (64ll << 20)
#endif
constexpr int64_t kForwardPassBytes = ZF_FORWARD_PASS_BYTES;
constexpr int64_t kBackwardPassBytes = ZF_BACKWARD_PASS_BYTES;

struct LevelPasses {
    int n = 1;
    int begin[kMaxLevels + 1] = {};

    // consecutive levels whose bytes[] together fit the budget (a larger level alone)
    void split(const int64_t* bytes, const int n_levels, const int64_t budget) {
        n = 1;
        begin[0] = 0;
        int64_t sum = 0;
        for (int l = 0; l < n_levels; l++) {
            if (l > begin[n - 1] && sum + bytes[l] > budget) {
                begin[n++] = l;
                sum = 0;
            }
            sum += bytes[l];
        }
        begin[n] = n_levels;
    }
};

const zf::KernelSet* kernel_set(const int n_features) {
    static const zf::KernelSet* const table[kMaxFeatures] = {&ZF_KSET_NAME(1), &ZF_KSET_NAME(2), &ZF_KSET_NAME(3), &ZF_KSET_NAME(4)};
    return table[n_features - 1];
}

const zf::MlpKernelSet* mlp_kernel_set(const int n_features, const int pad) {
    struct Entry {
        int features, pad;
        const zf::MlpKernelSet* set;
    };
    static const Entry entries[] = {
#define ZF_MLP_ENTRY(F, P) {F, P, &ZF_MLP_KSET_NAME(F, P)},
        ZF_FOR_EACH_MLP(ZF_MLP_ENTRY)
#undef ZF_MLP_ENTRY
    };
    for (const Entry& e : entries) {
        if (e.features == n_features && e.pad == pad) return e.set;
    }
    return nullptr;
}

thread_local std::string last_error;

int fail(const int code, const std::string& message) {
    last_error = "ZipNeRF: " + message;
    return code;
}

int cuda_fail(const cudaError_t error, const char* what) {
    return fail(ZF_ERROR_CUDA, std::string(what) + ": " + cudaGetErrorString(error));
}

constexpr int64_t kMinHalfGradEntries = int64_t(1) << 20;  // zipnerf_config.h:15
constexpr double kGridMaxValue = 1e-4 / 10.0;              // hash_init_range / precondition_scaling
constexpr double kNerfGridGradScale = 1048576.0;           // zipnerf_config.h:12
constexpr int kBackwardMlpBlocksPerSm = 8;                 // featurizer.h:15

// raises the dynamic shared memory limit of a kernel once per (kernel, size) high-water mark
cudaError_t ensure_smem(const void* kernel, const size_t bytes) {
    static std::mutex mutex;
    static const void* kernels[1024];
    static size_t limits[1024];
    static int n = 0;
    if (bytes <= 48 * 1024) return cudaSuccess;
    std::lock_guard<std::mutex> lock(mutex);
    int i = 0;
    while (i < n && kernels[i] != kernel) i++;
    if (i < n && limits[i] >= bytes) return cudaSuccess;
    const cudaError_t error = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (error != cudaSuccess) return error;
    if (i == n && n < 1024) {
        kernels[n] = kernel;
        n++;
    }
    if (i < 1024) limits[i] = bytes;
    return cudaSuccess;
}

template <typename Args>
cudaError_t launch(void (*kernel)(zf::GridParams, Args), const unsigned grid, const size_t smem, cudaStream_t stream,
                   const zf::GridParams& gp, const Args& args, const int block = zf::kBlock) {
    cudaError_t error = ensure_smem(reinterpret_cast<const void*>(kernel), smem);
    if (error != cudaSuccess) return error;
    void* params[] = {const_cast<zf::GridParams*>(&gp), const_cast<Args*>(&args)};
    return cudaLaunchKernel(reinterpret_cast<const void*>(kernel), dim3(grid), dim3(block), params, smem, stream);
}

unsigned n_blocks(const int64_t n) { return static_cast<unsigned>((n + zf::kBlock - 1) / zf::kBlock); }

bool aligned(const void* p, const size_t bytes) { return reinterpret_cast<uintptr_t>(p) % bytes == 0; }

}  // namespace

namespace zf {

int set_error(const int code, const std::string& message) { return fail(code, message); }
int set_cuda_error(const cudaError_t error, const char* what) { return cuda_fail(error, what); }

}  // namespace zf

struct zf_featurizer {
    int level = 0;
    int n_levels = 0;
    int n_features = 0;
    int mlp_width = 0;
    int n_fp32_grad_levels = 0;
    int device = 0;
    int n_sms = 0;
    int64_t offsets[kMaxLevels + 1] = {};
    zf::GridParams params{};
    const zf::KernelSet* kernels = nullptr;
    const zf::MlpKernelSet* mlp_kernels = nullptr;  // null without an MLP
    // stream-ordered pool of the proposal backward's workspace when the caller passes none; it keeps its memory after
    // a call (no release threshold), so repeated calls neither map nor unmap device memory
    cudaMemPool_t workspace_pool = nullptr;
    // level passes of the forward without MLP and of the NeRF backward: pass p covers levels [begin[p], begin[p + 1])
    LevelPasses forward_passes, backward_passes;

    int n_output_features() const { return n_levels * (n_features + 1); }
    int64_t n_rows() const { return offsets[n_levels]; }
    int64_t n_fp32_grad_rows() const { return offsets[n_fp32_grad_levels]; }
};

namespace {

// shared checks of the rays (featurizer.cu:207-214); fills the kernel's RayInputs
int check_rays(const zf_rays* rays, zf::RayInputs& in) {
    if (rays == nullptr) return fail(ZF_ERROR_INVALID_ARGUMENT, "rays must not be null");
    if (rays->n_rays < 0 || rays->n_intervals < 1) return fail(ZF_ERROR_INVALID_ARGUMENT, "tdist must have at least two columns");
    // bounded before the product is formed, so that it cannot overflow
    if (rays->n_intervals > static_cast<int64_t>(UINT32_MAX) || rays->n_rays > static_cast<int64_t>(UINT32_MAX) / rays->n_intervals) {
        return fail(ZF_ERROR_INVALID_ARGUMENT, "too many samples for 32-bit indexing");
    }
    const int64_t n_samples = rays->n_rays * rays->n_intervals;
    if (n_samples > 0 && (rays->origins == nullptr || rays->directions == nullptr || rays->radii == nullptr || rays->tdist == nullptr)) {
        return fail(ZF_ERROR_INVALID_ARGUMENT, "origins, directions, radii and tdist must be given");
    }
    in.origins = rays->origins;
    in.directions = rays->directions;
    in.radii = rays->radii;
    in.tdist = rays->tdist;
    if (rays->sample_offset < 0) return fail(ZF_ERROR_INVALID_ARGUMENT, "sample_offset must not be negative");
    in.pattern_seed = rays->pattern_seed;
    in.sample_offset = static_cast<unsigned long long>(rays->sample_offset);
    in.n_intervals = static_cast<uint32_t>(rays->n_intervals);
    in.n_samples = static_cast<uint32_t>(n_samples);
    return ZF_OK;
}

}  // namespace

extern "C" {

int zf_featurizer_create(const int level, const int64_t* level_sizes, const int64_t* level_entries, const int n_levels,
                         const int n_features, const int mlp_width, zf_featurizer** out) {
    if (out == nullptr) return fail(ZF_ERROR_INVALID_ARGUMENT, "output pointer must not be null");
    *out = nullptr;
    if (n_levels < 1 || n_levels > kMaxLevels) return fail(ZF_ERROR_UNSUPPORTED, "grid levels must be in [1, 16]");
    if (n_features < 1 || n_features > kMaxFeatures) return fail(ZF_ERROR_UNSUPPORTED, "features per level must be in [1, 4]");
    if (mlp_width < 0) return fail(ZF_ERROR_INVALID_ARGUMENT, "mlp_width must not be negative");
    if (level_sizes == nullptr || level_entries == nullptr) return fail(ZF_ERROR_INVALID_ARGUMENT, "level sizes and entries must be given");
    zf_featurizer f;
    f.level = level;
    f.n_levels = n_levels;
    f.n_features = n_features;
    f.mlp_width = mlp_width;
    f.offsets[0] = 0;
    for (int l = 0; l < n_levels; l++) {
        if (level_sizes[l] < 1 || level_sizes[l] > (int64_t(1) << 20) || level_entries[l] < 1 || level_entries[l] > static_cast<int64_t>(UINT32_MAX)) {
            return fail(ZF_ERROR_INVALID_ARGUMENT, "invalid level size or entries");
        }
        const int64_t size = level_sizes[l];
        // the kernels' group records pack cell coordinates into 16 bits
        if (size > static_cast<int64_t>(zf::kMaxPackedSize)) return fail(ZF_ERROR_UNSUPPORTED, "level sizes above 65534 are not supported");
        const bool hashed = size * size * size > level_entries[l];
        if (!hashed && size * size * size > static_cast<int64_t>(INT32_MAX)) return fail(ZF_ERROR_INVALID_ARGUMENT, "dense level too large");
        f.offsets[l + 1] = f.offsets[l] + level_entries[l];
        f.params.size[l] = static_cast<uint32_t>(size);
        f.params.entries[l] = static_cast<uint32_t>(level_entries[l]);
        f.params.offset[l] = static_cast<uint32_t>(std::min<int64_t>(f.offsets[l], UINT32_MAX));
        if (hashed) f.params.hashed_mask |= 1u << l;
        if ((level_entries[l] & (level_entries[l] - 1)) == 0) f.params.pow2_mask |= 1u << l;
    }
    // featurizer.cu:154: 32-bit row indexing
    if (f.offsets[n_levels] * n_features > static_cast<int64_t>(UINT32_MAX)) return fail(ZF_ERROR_INVALID_ARGUMENT, "grid table too large for 32-bit indexing");
    f.params.offset[n_levels] = static_cast<uint32_t>(f.offsets[n_levels]);
    while (f.n_fp32_grad_levels < n_levels && level_entries[f.n_fp32_grad_levels] < kMinHalfGradEntries) f.n_fp32_grad_levels++;
    f.params.n_fp32_levels = static_cast<uint32_t>(f.n_fp32_grad_levels);
    f.params.pattern_stream = zf::kPatternStreamBase + static_cast<unsigned long long>(level);
    f.params.n_levels = static_cast<uint32_t>(n_levels);
    f.params.n_features = static_cast<uint32_t>(n_features);
    int64_t table_bytes[kMaxLevels], grad_bytes[kMaxLevels];
    for (int l = 0; l < n_levels; l++) {
        table_bytes[l] = level_entries[l] * n_features * static_cast<int64_t>(sizeof(float));
        grad_bytes[l] = level_entries[l] * n_features * (l < f.n_fp32_grad_levels ? 4 : 2);
    }
    f.forward_passes.split(table_bytes, n_levels, kForwardPassBytes);
    f.backward_passes.split(grad_bytes, n_levels, kBackwardPassBytes);
    f.kernels = kernel_set(n_features);
    if (f.kernels == nullptr) return fail(ZF_ERROR_UNSUPPORTED, "this feature count is not compiled into this build");
    if (mlp_width > 0) {
        f.mlp_kernels = mlp_kernel_set(n_features, zf::mlp_pad(f.n_output_features()));
        if (f.mlp_kernels == nullptr) return fail(ZF_ERROR_UNSUPPORTED, "this mlp input width is not compiled into this build");
        const size_t fwd = static_cast<size_t>(zf::forward_smem_floats(f.n_output_features(), f.n_features)) * sizeof(float);
        const size_t bwd = static_cast<size_t>(zf::backward_mlp_smem_floats(f.n_output_features(), zf::mlp_pad(f.n_output_features()), mlp_width)) * sizeof(float);
        if (std::max(fwd, bwd) > 227 * 1024) return fail(ZF_ERROR_UNSUPPORTED, "mlp_width too large for the kernels' shared memory");
    }
    cudaError_t error = cudaGetDevice(&f.device);
    if (error != cudaSuccess) return cuda_fail(error, "cudaGetDevice");
    error = cudaDeviceGetAttribute(&f.n_sms, cudaDevAttrMultiProcessorCount, f.device);
    if (error != cudaSuccess) return cuda_fail(error, "cudaDeviceGetAttribute");
    if (mlp_width > 0) {
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = f.device;
        error = cudaMemPoolCreate(&f.workspace_pool, &props);
        if (error != cudaSuccess) return cuda_fail(error, "workspace pool creation");
        uint64_t keep = UINT64_MAX;
        error = cudaMemPoolSetAttribute(f.workspace_pool, cudaMemPoolAttrReleaseThreshold, &keep);
        if (error != cudaSuccess) {
            cudaMemPoolDestroy(f.workspace_pool);
            return cuda_fail(error, "workspace pool release threshold");
        }
    }
    *out = new zf_featurizer(f);
    return ZF_OK;
}

void zf_featurizer_destroy(zf_featurizer* featurizer) {
    if (featurizer == nullptr) return;
    // memory still in use by queued work is released when that work completes
    if (featurizer->workspace_pool != nullptr) cudaMemPoolDestroy(featurizer->workspace_pool);
    delete featurizer;
}

int zf_featurizer_n_output_features(const zf_featurizer* featurizer) { return featurizer ? featurizer->n_output_features() : 0; }

int64_t zf_featurizer_n_fp32_grad_rows(const zf_featurizer* featurizer) { return featurizer ? featurizer->n_fp32_grad_rows() : 0; }

int64_t zf_featurizer_n_rows(const zf_featurizer* featurizer) { return featurizer ? featurizer->n_rows() : 0; }

int zf_featurizer_launches(const zf_featurizer* featurizer, const int call) {
    if (featurizer == nullptr) return 0;
    switch (call) {
        case 0: return featurizer->forward_passes.n;
        case 1: return featurizer->mlp_width > 0 ? 1 : 0;
        case 2: return featurizer->backward_passes.n;
        case 3: return featurizer->mlp_width > 0 ? 2 : 0;  // the MLP kernel and the scatter
        default: return 0;
    }
}

int zf_featurize_forward(zf_featurizer* f, const zf_forward_args* a, cudaStream_t stream) {
    if (f == nullptr || a == nullptr) return fail(ZF_ERROR_INVALID_ARGUMENT, "featurizer and arguments must not be null");
    zf::ForwardArgs k{};
    int rc = check_rays(&a->rays, k.in);
    if (rc != ZF_OK) return rc;
    const int64_t n_samples = k.in.n_samples;
    const int n_out = f->n_output_features();
    if (a->table == nullptr || a->scale_magnitudes == nullptr) return fail(ZF_ERROR_INVALID_ARGUMENT, "table and scale_magnitudes must be given");
    if (a->table_rows != f->n_rows()) return fail(ZF_ERROR_INVALID_ARGUMENT, "table rows do not match the grid layout");
    if (a->raw_density != nullptr) {
        // featurizer.cu:215-223
        if (f->mlp_width == 0 || a->w0 == nullptr || a->w0_numel != static_cast<int64_t>(f->mlp_width) * n_out || a->b0 == nullptr || a->w1 == nullptr || a->b1 == nullptr) {
            return fail(ZF_ERROR_INVALID_ARGUMENT, "invalid proposal mlp weights");
        }
    }
    if (a->features_bf16 != nullptr && a->features_bf16_width < n_out) return fail(ZF_ERROR_INVALID_ARGUMENT, "invalid features_bf16");
    if (a->nerf_inputs != nullptr && (a->encoded_directions == nullptr || a->encoded_width < 1 || a->nerf_inputs_width < a->encoded_width)) {
        return fail(ZF_ERROR_INVALID_ARGUMENT, "invalid nerf_inputs");
    }
    if (n_samples == 0) return ZF_OK;
    k.table = a->table;
    k.scale_magnitudes = a->scale_magnitudes;
    const bool mlp = a->raw_density != nullptr;
    k.w0 = mlp ? a->w0 : nullptr;
    k.b0 = mlp ? a->b0 : nullptr;
    k.w1 = mlp ? a->w1 : nullptr;
    k.b1 = mlp ? a->b1 : nullptr;
    k.mlp_width = mlp ? f->mlp_width : 0;
    k.raw_density = a->raw_density;
    k.features_float = a->features_float;
    k.features_bf16 = a->features_bf16;
    k.features_bf16_width = static_cast<int>(a->features_bf16_width);
    k.bf16_pairs = a->features_bf16 != nullptr && a->features_bf16_width % 2 == 0 && aligned(a->features_bf16, 4);
    k.encoded_directions = a->nerf_inputs != nullptr ? a->encoded_directions : nullptr;
    k.nerf_inputs = a->nerf_inputs;
    k.nerf_inputs_width = a->nerf_inputs != nullptr ? static_cast<int>(a->nerf_inputs_width) : 0;
    k.encoded_width = a->nerf_inputs != nullptr ? static_cast<int>(a->encoded_width) : 0;
    k.inputs_vectors = a->nerf_inputs != nullptr && a->nerf_inputs_width % 8 == 0 && a->encoded_width % 8 == 0 && aligned(a->nerf_inputs, 16) && aligned(a->encoded_directions, 16);
    k.w0_vectors = mlp && n_out % 4 == 0 && aligned(a->w0, 16);
    k.interleave_rays = a->interleave ? 32u : 0u;
    const size_t smem = static_cast<size_t>(zf::forward_smem_floats(n_out, f->n_features)) * sizeof(float);
    // the fused MLP needs every level of an interval in one launch; without it, one launch per level pass
    const int n_passes = mlp ? 1 : f->forward_passes.n;
    for (int p = 0; p < n_passes; p++) {
        k.level_begin = static_cast<uint32_t>(mlp ? 0 : f->forward_passes.begin[p]);
        k.level_end = static_cast<uint32_t>(mlp ? f->n_levels : f->forward_passes.begin[p + 1]);
        const cudaError_t error = launch(mlp ? f->mlp_kernels->forward : f->kernels->forward, n_blocks(n_samples), smem, stream, f->params, k);
        if (error != cudaSuccess) return cuda_fail(error, "featurize_forward launch");
    }
    return ZF_OK;
}

int zf_featurize_backward(zf_featurizer* f, const zf_backward_args* a, cudaStream_t stream) {
    if (f == nullptr || a == nullptr) return fail(ZF_ERROR_INVALID_ARGUMENT, "featurizer and arguments must not be null");
    // featurizer.cu:276-283
    const int64_t n_fp32 = f->n_fp32_grad_rows() * f->n_features;
    const int64_t n_half = (f->n_rows() - f->n_fp32_grad_rows()) * f->n_features;
    if (a->grad_table_numel != n_fp32 || a->grad_table_half_numel != n_half || (n_fp32 > 0 && a->grad_table == nullptr) || (n_half > 0 && a->grad_table_half == nullptr)) {
        return fail(ZF_ERROR_INVALID_ARGUMENT, "invalid grid gradient split");
    }
    zf::BackwardArgs k{};
    int rc = check_rays(&a->rays, k.in);
    if (rc != ZF_OK) return rc;
    if (a->grad_features_cols < f->n_output_features() || a->grad_features_stride < a->grad_features_cols || (k.in.n_samples > 0 && a->grad_features == nullptr)) {
        return fail(ZF_ERROR_INVALID_ARGUMENT, "grad_features has an invalid layout");
    }
    if (k.in.n_samples == 0) return ZF_OK;
    k.grad_features = a->grad_features;
    k.grad_stride = a->grad_features_stride;
    k.grad_scale = static_cast<float>(kNerfGridGradScale);
    k.n_fp32_levels = static_cast<uint32_t>(f->n_fp32_grad_levels);
    k.grad_table = a->grad_table;
    k.grad_table_half = a->grad_table_half;
    int max_levels = 0;
    for (int p = 0; p < f->backward_passes.n; p++) max_levels = std::max(max_levels, f->backward_passes.begin[p + 1] - f->backward_passes.begin[p]);
    const size_t smem = static_cast<size_t>(zf::backward_smem_bytes(max_levels * (f->n_features + 1), 2));
    for (int p = 0; p < f->backward_passes.n; p++) {
        k.level_begin = static_cast<uint32_t>(f->backward_passes.begin[p]);
        k.level_end = static_cast<uint32_t>(f->backward_passes.begin[p + 1]);
        const cudaError_t error = launch(f->kernels->backward, n_blocks(k.in.n_samples), smem, stream, f->params, k);
        if (error != cudaSuccess) return cuda_fail(error, "featurize_backward launch");
    }
    return ZF_OK;
}

int64_t zf_featurize_backward_mlp_workspace_size(const zf_featurizer* f, const int64_t n_samples) {
    if (f == nullptr || n_samples < 0) return 0;
    // the scaled feature gradient of every sample, between the MLP and the scatter kernels
    return n_samples * f->n_output_features() * static_cast<int64_t>(sizeof(float));
}

int zf_featurize_backward_mlp(zf_featurizer* f, const zf_backward_mlp_args* a, cudaStream_t stream) {
    if (f == nullptr || a == nullptr) return fail(ZF_ERROR_INVALID_ARGUMENT, "featurizer and arguments must not be null");
    zf::BackwardMlpArgs k{};
    int rc = check_rays(&a->rays, k.in);
    if (rc != ZF_OK) return rc;
    const int64_t n_samples = k.in.n_samples;
    const int n_out = f->n_output_features();
    // featurizer.cu:318-331
    if (a->features_numel != n_samples * n_out || a->grad_raw_density_numel != n_samples) return fail(ZF_ERROR_INVALID_ARGUMENT, "invalid backward_mlp inputs");
    if (f->mlp_width == 0 || a->w0_numel != static_cast<int64_t>(f->mlp_width) * n_out || a->grad_w0_numel != a->w0_numel) {
        return fail(ZF_ERROR_INVALID_ARGUMENT, "invalid proposal mlp weights");
    }
    if (a->grad_table_numel != f->n_rows() * f->n_features) return fail(ZF_ERROR_INVALID_ARGUMENT, "invalid grad_table");
    if (a->w0 == nullptr || a->b0 == nullptr || a->w1 == nullptr || a->grad_table == nullptr || a->grad_w0 == nullptr || a->grad_b0 == nullptr ||
        a->grad_w1 == nullptr || a->grad_b1 == nullptr || (n_samples > 0 && (a->features == nullptr || a->grad_raw_density == nullptr))) {
        return fail(ZF_ERROR_INVALID_ARGUMENT, "backward_mlp tensors must be given");
    }
    const int64_t workspace_bytes = zf_featurize_backward_mlp_workspace_size(f, n_samples);
    if (a->workspace != nullptr && (a->workspace_bytes < workspace_bytes || !aligned(a->workspace, 16))) {
        return fail(ZF_ERROR_INVALID_ARGUMENT, "workspace too small or not 16-byte aligned");
    }
    if (n_samples == 0) return ZF_OK;
    float* rows = static_cast<float*>(a->workspace);
    if (rows == nullptr) {
        const cudaError_t error = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&rows), static_cast<size_t>(workspace_bytes), f->workspace_pool, stream);
        if (error != cudaSuccess) return cuda_fail(error, "backward_mlp workspace allocation");
    }
    k.features = a->features;
    k.grad_raw_density = a->grad_raw_density;
    k.w0 = a->w0;
    k.b0 = a->b0;
    k.w1 = a->w1;
    k.mlp_width = f->mlp_width;
    k.grad_rows = rows;
    k.grad_w0 = a->grad_w0;
    k.grad_b0 = a->grad_b0;
    k.grad_w1 = a->grad_w1;
    k.grad_b1 = a->grad_b1;
    // one resident wave of the MLP kernel (its per-block parameter sums end in one atomic per parameter and block)
    const size_t smem = static_cast<size_t>(zf::backward_mlp_smem_floats(n_out, zf::mlp_pad(n_out), f->mlp_width)) * sizeof(float);
    cudaError_t error = ensure_smem(reinterpret_cast<const void*>(f->mlp_kernels->backward_mlp), smem);
    int resident = 0;
    if (error == cudaSuccess) error = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, reinterpret_cast<const void*>(f->mlp_kernels->backward_mlp), zf::kMlpBlock, smem);
    if (error == cudaSuccess) {
        const unsigned mlp_blocks = static_cast<unsigned>((n_samples + zf::kMlpBlock - 1) / zf::kMlpBlock);
        const unsigned blocks = std::min<unsigned>(mlp_blocks, static_cast<unsigned>(f->n_sms * std::max(resident, 1)));
        error = launch(f->mlp_kernels->backward_mlp, blocks, smem, stream, f->params, k, zf::kMlpBlock);
    }
    if (error == cudaSuccess) {
        // the scatter of the scaled feature gradients into the fp32 grid gradient (all levels), skipping samples with a
        // zero raw density gradient (featurize_backward_mlp.cu:103-108)
        zf::BackwardArgs s{};
        s.in = k.in;
        s.grad_rows = rows;
        s.skip_if_zero = a->grad_raw_density;
        s.n_fp32_levels = static_cast<uint32_t>(f->n_levels);
        s.grad_table = a->grad_table;
        s.level_begin = 0;
        s.level_end = static_cast<uint32_t>(f->n_levels);
        const size_t scatter_smem = static_cast<size_t>(zf::backward_smem_bytes(n_out, 4));
        error = launch(f->kernels->backward, n_blocks(n_samples), scatter_smem, stream, f->params, s);
    }
    if (a->workspace == nullptr) {
        const cudaError_t free_error = cudaFreeAsync(rows, stream);
        if (error == cudaSuccess) error = free_error;
    }
    if (error != cudaSuccess) return cuda_fail(error, "featurize_backward_mlp launch");
    return ZF_OK;
}

int zf_featurize_debug(zf_featurizer* f, const zf_rays* rays, const uint32_t* samples, const int64_t n_debug, float* x, float* scale,
                       int32_t* contracted, int32_t* n_groups, uint32_t* rows, float* weights, cudaStream_t stream) {
    if (f == nullptr) return fail(ZF_ERROR_INVALID_ARGUMENT, "featurizer must not be null");
    zf::DebugArgs k{};
    int rc = check_rays(rays, k.in);
    if (rc != ZF_OK) return rc;
    if (n_debug < 0 || n_debug > static_cast<int64_t>(UINT32_MAX)) return fail(ZF_ERROR_INVALID_ARGUMENT, "invalid debug sample count");
    if (n_debug == 0) return ZF_OK;
    if (samples == nullptr || x == nullptr || scale == nullptr || contracted == nullptr || n_groups == nullptr || rows == nullptr || weights == nullptr) {
        return fail(ZF_ERROR_INVALID_ARGUMENT, "debug outputs must be given");
    }
    k.samples = samples;
    k.n_debug = static_cast<uint32_t>(n_debug);
    k.x = x;
    k.scale = scale;
    k.contracted = contracted;
    k.n_groups = n_groups;
    k.rows = rows;
    k.weights = weights;
    if (&zf_debug_kernel == nullptr) return fail(ZF_ERROR_UNSUPPORTED, "the debug kernel is not compiled into this build");
    void (*kernel)(zf::GridParams, zf::DebugArgs) = zf_debug_kernel;
    void* params[] = {&f->params, &k};
    const cudaError_t error = cudaLaunchKernel(reinterpret_cast<const void*>(kernel), dim3(static_cast<unsigned>((n_debug + 63) / 64)), dim3(64), params, 0, stream);
    if (error != cudaSuccess) return cuda_fail(error, "featurize_debug launch");
    return ZF_OK;
}

int zf_check_erf_saturation(const uint32_t first_bits, const uint32_t last_bits, unsigned long long* n_not_one, uint32_t* max_bits, cudaStream_t stream) {
    if (&zf_check_erf_kernel == nullptr) return fail(ZF_ERROR_UNSUPPORTED, "the erf check is not compiled into this build");
    if (n_not_one == nullptr || max_bits == nullptr || last_bits < first_bits) return fail(ZF_ERROR_INVALID_ARGUMENT, "invalid erf check arguments");
    const uint32_t count = last_bits - first_bits + 1u;
    void (*kernel)(uint32_t, uint32_t, unsigned long long*, uint32_t*) = zf_check_erf_kernel;
    uint32_t first = first_bits, n = count;
    void* params[] = {&first, &n, &n_not_one, &max_bits};
    const cudaError_t error = cudaLaunchKernel(reinterpret_cast<const void*>(kernel), dim3(148 * 16), dim3(256), params, 0, stream);
    if (error != cudaSuccess) return cuda_fail(error, "erf check launch");
    return ZF_OK;
}

float zf_erf_saturation_threshold(void) { return zf::kErfSaturation; }

}  // extern "C"

// ---------------------------------------------------------------------------------------------------------------------
// Allocation-free variant of the proposal-level backward, for hosts that must not allocate device memory while they run:
// a host that plans a fixed device-memory budget up front, or a plugin inside a framework that owns every device
// allocation and does not let its plugins call cudaMalloc / cudaMallocAsync, and that cannot hand this library a
// workspace either. Its workspace is this file-scope device array instead: every GPU that loads the library holds it
// (kStaticWorkspaceBytes) until the process exits, and every call on a device shares it.

namespace {

constexpr size_t kStaticWorkspaceBytes = size_t(32) << 20;  // 32 MiB: n_samples * n_output_features * 4 bytes at most
constexpr int kMaxDevices = 64;

}  // namespace

static __device__ __align__(256) unsigned char zf_static_workspace[kStaticWorkspaceBytes];

namespace {

// device address of zf_static_workspace on the current device, looked up once per device with that device current
int static_workspace_address(void** address) {
    static std::mutex mutex;
    static void* addresses[kMaxDevices] = {};
    int device = 0;
    cudaError_t error = cudaGetDevice(&device);
    if (error != cudaSuccess) return cuda_fail(error, "cudaGetDevice");
    if (device < 0 || device >= kMaxDevices) return fail(ZF_ERROR_UNSUPPORTED, "device index beyond the static workspace table");
    std::lock_guard<std::mutex> lock(mutex);
    if (addresses[device] == nullptr) {
        void* ptr = nullptr;
        error = cudaGetSymbolAddress(&ptr, zf_static_workspace);
        if (error != cudaSuccess) return cuda_fail(error, "cudaGetSymbolAddress of the static workspace");
        addresses[device] = ptr;
    }
    *address = addresses[device];
    return ZF_OK;
}

}  // namespace

extern "C" {

int zf_featurize_backward_mlp_no_alloc(zf_featurizer* f, const zf_backward_mlp_args* a, cudaStream_t stream) {
    if (f == nullptr || a == nullptr) return fail(ZF_ERROR_INVALID_ARGUMENT, "featurizer and arguments must not be null");
    if (a->rays.n_rays < 0 || a->rays.n_intervals < 1) return fail(ZF_ERROR_INVALID_ARGUMENT, "tdist must have at least two columns");
    // the sample limit of the static workspace, checked on the ray count before any product is formed (no overflow)
    const int64_t limit = static_cast<int64_t>(kStaticWorkspaceBytes) / (f->n_output_features() * static_cast<int64_t>(sizeof(float)));
    if (a->rays.n_rays > limit / a->rays.n_intervals) {
        return fail(ZF_ERROR_INVALID_ARGUMENT, "backward_mlp without allocation supports at most " + std::to_string(limit) +
                    " samples of this featurizer (a static 32 MiB workspace); got " + std::to_string(a->rays.n_rays) + " rays x " +
                    std::to_string(a->rays.n_intervals) + " intervals");
    }
    void* workspace = nullptr;
    const int rc = static_workspace_address(&workspace);
    if (rc != ZF_OK) return rc;
    // the MLP kernel writes every workspace row before the scatter kernel reads it, so nothing needs clearing
    zf_backward_mlp_args args = *a;
    args.workspace = workspace;
    args.workspace_bytes = static_cast<int64_t>(kStaticWorkspaceBytes);
    return zf_featurize_backward_mlp(f, &args, stream);
}


const char* zf_last_error(void) { return last_error.c_str(); }

double zf_grid_max_value(void) { return kGridMaxValue; }

double zf_nerf_grid_grad_scale(void) { return kNerfGridGradScale; }

}  // extern "C"

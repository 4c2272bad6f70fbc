// fz_optim.cu -- the C ABI of include/zf_optim.h: Adam objects (moments, the block split of the buffers' level ranges)
// with the reference's argument checks and messages (optimizer_api.cu:123-158), and the step launch.
#include "zf_optim.h"
#include "fz_optim.cuh"
#include "fz_status.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <string>
#include <vector>

struct zf_adam {
    int n_buffers = 0;
    int n_levels = 0;
    int device = 0;
    int64_t step = 0;
    int64_t numels[zf::kAdamMaxBuffers] = {};
    float* exp_avgs[zf::kAdamMaxBuffers] = {};
    float* exp_avg_sqs[zf::kAdamMaxBuffers] = {};
    double* block_sums = nullptr;
    unsigned* counter = nullptr;
    float beta1 = 0.0f, beta2 = 0.0f;
    zf::AdamParams params{};  // everything but the learning rate and the bias corrections of the step

    ~zf_adam() {
        for (int b = 0; b < n_buffers; b++) {
            cudaFree(exp_avgs[b]);
            cudaFree(exp_avg_sqs[b]);
        }
        cudaFree(block_sums);
        cudaFree(counter);
    }
};

namespace {

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

int invalid(const std::string& message) { return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, message); }

int device_zeros(void** pointer, const size_t bytes) {
    cudaError_t error = cudaMalloc(pointer, std::max<size_t>(bytes, 16));
    if (error == cudaSuccess) error = cudaMemset(*pointer, 0, std::max<size_t>(bytes, 16));
    return error == cudaSuccess ? ZF_OK : zf::set_cuda_error(error, "optimizer state allocation");
}

}  // namespace

int zf_adam_create(const zf_adam_buffer* buffers, const int n_buffers, const double reg_weight, const double max_value, const double beta1,
                   const double beta2, const double eps, float* magnitudes, const int64_t n_magnitudes, float* regularization, zf_adam** out) {
    if (out == nullptr) return invalid("null output handle");
    *out = nullptr;
    if (buffers == nullptr || n_buffers <= 0 || n_buffers > zf::kAdamMaxBuffers) return invalid("invalid optimizer buffers");
    // the checks of optimizer_api.cu:123-155, in its order
    int n_levels = 0;
    for (int b = 0; b < n_buffers; b++) {
        const zf_adam_buffer& buffer = buffers[b];
        if (buffer.param == nullptr || buffer.numel % 4 != 0 || buffer.numel < 0 || !aligned16(buffer.param)) {
            return invalid("param must be a contiguous float (or half) cuda tensor with a multiple of four elements");
        }
        if (buffer.grad == nullptr || !aligned16(buffer.grad)) {
            return invalid("grad must be a contiguous float (or half) cuda tensor with a multiple of four elements");
        }
        if (!(buffer.grad_scale > 0.0) || !std::isfinite(buffer.grad_scale)) return invalid("invalid optimizer gradient scale");
        if (buffer.n_level_offsets > 0) {
            const int64_t* offsets = buffer.level_offsets;
            if (offsets == nullptr || buffer.n_level_offsets < 2 || offsets[0] != 0 || offsets[buffer.n_level_offsets - 1] != buffer.numel) {
                return invalid("level offsets must cover the buffer");
            }
            for (int i = 0; i + 1 < buffer.n_level_offsets; i++) {
                if (offsets[i] % 4 != 0 || offsets[i + 1] <= offsets[i]) return invalid("invalid level offsets");
            }
            n_levels += buffer.n_level_offsets - 1;
        }
    }
    if (n_levels > zf::kAdamMaxLevels || n_levels + n_buffers > zf::kAdamMaxRanges) return invalid("too many optimizer levels");
    if (n_magnitudes != n_levels || (n_levels > 0 && magnitudes == nullptr)) {
        return invalid("magnitudes must be a contiguous float cuda tensor with one entry per level");
    }
    if (regularization == nullptr) return invalid("null regularization output");

    zf_adam* adam = new zf_adam();
    cudaError_t error = cudaGetDevice(&adam->device);
    int n_sms = 0;
    if (error == cudaSuccess) error = cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, adam->device);
    if (error != cudaSuccess) {
        delete adam;
        return zf::set_cuda_error(error, "device query");
    }
    adam->n_levels = n_levels;
    adam->beta1 = static_cast<float>(beta1);
    adam->beta2 = static_cast<float>(beta2);
    zf::AdamParams& p = adam->params;
    // ranges in buffer order (optimizer_api.cu:166-181), as buffer-local group spans
    int64_t n_groups = 0;
    int level = 0;
    for (int b = 0; b < n_buffers; b++) {
        const zf_adam_buffer& buffer = buffers[b];
        adam->n_buffers = b + 1;
        adam->numels[b] = buffer.numel;
        int status = device_zeros(reinterpret_cast<void**>(&adam->exp_avgs[b]), sizeof(float) * buffer.numel);
        if (status == ZF_OK) status = device_zeros(reinterpret_cast<void**>(&adam->exp_avg_sqs[b]), sizeof(float) * buffer.numel);
        if (status != ZF_OK) {
            delete adam;
            return status;
        }
        p.buffers[b] = {reinterpret_cast<float4*>(buffer.param), buffer.grad_half ? nullptr : reinterpret_cast<float4*>(buffer.grad),
                        buffer.grad_half ? reinterpret_cast<uint2*>(buffer.grad) : nullptr, reinterpret_cast<float4*>(adam->exp_avgs[b]),
                        reinterpret_cast<float4*>(adam->exp_avg_sqs[b]), static_cast<float>(1.0 / buffer.grad_scale)};
        if (buffer.n_level_offsets == 0) {
            if (buffer.numel > 0) p.ranges[p.n_ranges++] = {0, buffer.numel / 4, 0, b, -1, 0};
        }
        for (int i = 0; i + 1 < buffer.n_level_offsets; i++, level++) {
            const int64_t size = buffer.level_offsets[i + 1] - buffer.level_offsets[i];
            p.level_reg_weights[level] = static_cast<float>(reg_weight / static_cast<double>(size));
            p.level_inv_sizes[level] = 1.0 / static_cast<double>(size);
            p.ranges[p.n_ranges++] = {buffer.level_offsets[i] / 4, buffer.level_offsets[i + 1] / 4, 0, b, level, 0};
        }
        n_groups += buffer.numel / 4;
    }
    // blocks: about kAdamBlocksPerSm per SM over all groups, every range at least one, chunks of whole ranges
    const int64_t target = static_cast<int64_t>(n_sms) * zf::kAdamBlocksPerSm;
    int n_blocks = 0;
    for (int r = 0; r < p.n_ranges; r++) {
        zf::AdamRange& range = p.ranges[r];
        const int64_t groups = range.end - range.begin;
        const int64_t wanted = std::max<int64_t>(1, (groups * target + n_groups - 1) / std::max<int64_t>(n_groups, 1));
        range.chunk = std::max<int64_t>(1, (groups + wanted - 1) / wanted);
        range.first_block = n_blocks;
        n_blocks += static_cast<int>((groups + range.chunk - 1) / range.chunk);
    }
    p.n_levels = n_levels;
    p.n_blocks = n_blocks;
    p.eps = static_cast<float>(eps);
    p.beta1 = adam->beta1;
    p.beta2 = adam->beta2;
    p.max_value_sq = max_value * max_value;
    p.magnitudes = magnitudes;
    p.regularization = regularization;
    int status = device_zeros(reinterpret_cast<void**>(&adam->block_sums), sizeof(double) * std::max(n_blocks, 1));
    if (status == ZF_OK) status = device_zeros(reinterpret_cast<void**>(&adam->counter), sizeof(unsigned));
    if (status != ZF_OK) {
        delete adam;
        return status;
    }
    p.block_sums = adam->block_sums;
    p.counter = adam->counter;
    *out = adam;
    return ZF_OK;
}

void zf_adam_destroy(zf_adam* adam) { delete adam; }

int zf_adam_step(zf_adam* adam, const double lr, cudaStream_t stream) {
    if (adam == nullptr) return invalid("null optimizer");
    adam->step++;
    zf::AdamParams p = adam->params;
    p.lr = static_cast<float>(lr);
    p.bias_correction1 = static_cast<float>(1.0 - std::pow(static_cast<double>(adam->beta1), static_cast<double>(adam->step)));
    p.bias_correction2 = static_cast<float>(1.0 - std::pow(static_cast<double>(adam->beta2), static_cast<double>(adam->step)));
    if (p.n_blocks == 0) return ZF_OK;
    void* args[] = {&p};
    const cudaError_t error = cudaLaunchKernel(reinterpret_cast<const void*>(zf::fz_adam_kernel), dim3(p.n_blocks), dim3(zf::kAdamBlock), args, 0, stream);
    return error == cudaSuccess ? ZF_OK : zf::set_cuda_error(error, "kernel launch");
}

int zf_adam_state(const zf_adam* adam, const int buffer, float** exp_avg, float** exp_avg_sq, int64_t* steps) {
    if (adam == nullptr || buffer < 0 || buffer >= adam->n_buffers) return invalid("invalid optimizer buffer");
    if (exp_avg != nullptr) *exp_avg = adam->exp_avgs[buffer];
    if (exp_avg_sq != nullptr) *exp_avg_sq = adam->exp_avg_sqs[buffer];
    if (steps != nullptr) *steps = adam->step;
    return ZF_OK;
}

// fz_mlp.cu -- the C ABI of include/zf_mlp.h: the ReLU backward with the bias gradient of the NeRF MLP's layers, one
// pass over the gradient (16-byte rows in and out) instead of separate mask, multiply and column-sum passes.
#include "zf_mlp.h"
#include "fz_device.cuh"
#include "fz_status.h"

#include <cuda_runtime.h>

#include <algorithm>

namespace zf {

constexpr int kReluBlock = 256;
constexpr int kReluMaxCols = 512;

// thread t of a block takes the 8 columns (t % chunks) * 8 of rows t / chunks, t / chunks + rows_per_pass, ... of its
// block's share; its column sums stay in registers until one shared-memory and one global atomic per column and block
__global__ void __launch_bounds__(kReluBlock) fz_relu_backward_kernel(uint16_t* __restrict__ grad, const int64_t grad_stride,
                                                                      const uint16_t* __restrict__ activation, const int64_t activation_stride,
                                                                      const int64_t n_rows, const int n_cols, float* __restrict__ bias_grad) {
    __shared__ float column_sums[kReluMaxCols];
    const int chunks = n_cols / 8;
    const int rows_per_pass = kReluBlock / chunks;
    const int chunk = threadIdx.x % chunks, row_in_pass = threadIdx.x / chunks;
    const bool lane_used = row_in_pass < rows_per_pass;
    for (int c = threadIdx.x; c < n_cols; c += kReluBlock) column_sums[c] = 0.0f;
    __syncthreads();
    float sums[8] = {};
    if (lane_used) {
        for (int64_t row = static_cast<int64_t>(blockIdx.x) * rows_per_pass + row_in_pass; row < n_rows; row += static_cast<int64_t>(gridDim.x) * rows_per_pass) {
            uint4* g = reinterpret_cast<uint4*>(grad + row * grad_stride + 8 * chunk);
            const uint4 a = *reinterpret_cast<const uint4*>(activation + row * activation_stride + 8 * chunk);
            uint4 v = *g;
            uint32_t* words = reinterpret_cast<uint32_t*>(&v);
            const uint32_t* acts = reinterpret_cast<const uint32_t*>(&a);
            for (int q = 0; q < 4; q++) {
                const uint16_t g_lo = static_cast<uint16_t>(words[q] & 0xffffu), g_hi = static_cast<uint16_t>(words[q] >> 16);
                const bool keep_lo = bf16_bits_to_f32(static_cast<uint16_t>(acts[q] & 0xffffu)) > 0.0f;
                const bool keep_hi = bf16_bits_to_f32(static_cast<uint16_t>(acts[q] >> 16)) > 0.0f;
                const uint16_t out_lo = keep_lo ? g_lo : 0, out_hi = keep_hi ? g_hi : 0;
                sums[2 * q] += bf16_bits_to_f32(out_lo);
                sums[2 * q + 1] += bf16_bits_to_f32(out_hi);
                words[q] = static_cast<uint32_t>(out_lo) | static_cast<uint32_t>(out_hi) << 16;
            }
            *g = v;
        }
    }
    if (bias_grad == nullptr) return;
    if (lane_used) {
        for (int k = 0; k < 8; k++) atomicAdd(&column_sums[8 * chunk + k], sums[k]);
    }
    __syncthreads();
    for (int c = threadIdx.x; c < n_cols; c += kReluBlock) atomicAdd(&bias_grad[c], column_sums[c]);
}

}  // namespace zf

int zf_relu_backward_bf16(uint16_t* grad, const int64_t grad_stride, const uint16_t* activation, const int64_t activation_stride, const int64_t n_rows,
                          const int n_cols, float* bias_grad, cudaStream_t stream) {
    if (n_rows < 0 || n_cols <= 0 || n_cols % 8 != 0 || n_cols > zf::kReluMaxCols || grad_stride < n_cols || activation_stride < n_cols
        || grad_stride % 8 != 0 || activation_stride % 8 != 0) {
        return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "relu_backward: invalid layout");
    }
    if (n_rows == 0) return ZF_OK;
    if (grad == nullptr || activation == nullptr || reinterpret_cast<uintptr_t>(grad) % 16 != 0 || reinterpret_cast<uintptr_t>(activation) % 16 != 0) {
        return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "relu_backward: tensors must be 16-byte aligned");
    }
    int device = 0, n_sms = 0;
    cudaError_t error = cudaGetDevice(&device);
    if (error == cudaSuccess) error = cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, device);
    if (error != cudaSuccess) return zf::set_cuda_error(error, "device query");
    const int rows_per_pass = zf::kReluBlock / (n_cols / 8);
    const int64_t blocks = std::min<int64_t>((n_rows + rows_per_pass - 1) / rows_per_pass, static_cast<int64_t>(n_sms) * 8);
    zf::fz_relu_backward_kernel<<<static_cast<unsigned>(blocks), zf::kReluBlock, 0, stream>>>(grad, grad_stride, activation, activation_stride, n_rows,
                                                                                             n_cols, bias_grad);
    error = cudaGetLastError();
    return error == cudaSuccess ? ZF_OK : zf::set_cuda_error(error, "kernel launch");
}

// c10/cuda/CUDAStream.h stand-in (TEST INFRASTRUCTURE ONLY; see torch/extension.h beside it): the reference's host
// wrappers launch on the current stream and check the launch; neither runs in the checker.
#pragma once

#include <cuda_runtime.h>

namespace c10::cuda {

struct CUDAStream {
    operator cudaStream_t() const { return nullptr; }
    cudaStream_t stream() const { return nullptr; }
};

inline CUDAStream getCurrentCUDAStream() { return {}; }

}  // namespace c10::cuda

#define C10_CUDA_KERNEL_LAUNCH_CHECK() \
    do {                               \
    } while (0)

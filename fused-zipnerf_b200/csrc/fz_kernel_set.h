// fz_kernel_set.h -- host-visible tables of the ahead-of-time kernel instantiations.
//
// Per features-per-level F: the forward without MLP and the NeRF-level backward. Per (F, padded MLP input width P,
// P a multiple of 4 up to 16 (F + 1)): the forward with the fused MLP and the proposal-level backward.
#pragma once

#include "fz_kernels.cuh"

namespace zf {

struct KernelSet {
    void (*forward)(GridParams, ForwardArgs);
    void (*backward)(GridParams, BackwardArgs);
};

struct MlpKernelSet {
    void (*forward)(GridParams, ForwardArgs);
    void (*backward_mlp)(GridParams, BackwardMlpArgs);
};

constexpr int kMlpPadStep = 4;

// padded MLP input width of n_out features
__host__ __device__ constexpr int mlp_pad(const int n_out) { return (n_out + kMlpPadStep - 1) / kMlpPadStep * kMlpPadStep; }

}  // namespace zf

#define ZF_KSET_NAME2(F) zf_kernel_set_F##F
#define ZF_KSET_NAME(F) ZF_KSET_NAME2(F)
#define ZF_MLP_KSET_NAME2(F, P) zf_mlp_kernel_set_F##F##_P##P
#define ZF_MLP_KSET_NAME(F, P) ZF_MLP_KSET_NAME2(F, P)

// X(F, P) over the compiled MLP instantiations
#define ZF_FOR_EACH_MLP(X) \
    X(1, 4) X(1, 8) X(1, 12) X(1, 16) X(1, 20) X(1, 24) X(1, 28) X(1, 32) \
    X(2, 4) X(2, 8) X(2, 12) X(2, 16) X(2, 20) X(2, 24) X(2, 28) X(2, 32) X(2, 36) X(2, 40) X(2, 44) X(2, 48) \
    X(3, 4) X(3, 8) X(3, 12) X(3, 16) X(3, 20) X(3, 24) X(3, 28) X(3, 32) X(3, 36) X(3, 40) X(3, 44) X(3, 48) X(3, 52) X(3, 56) \
    X(3, 60) X(3, 64) \
    X(4, 4) X(4, 8) X(4, 12) X(4, 16) X(4, 20) X(4, 24) X(4, 28) X(4, 32) X(4, 36) X(4, 40) X(4, 44) X(4, 48) X(4, 52) X(4, 56) \
    X(4, 60) X(4, 64) X(4, 68) X(4, 72) X(4, 76) X(4, 80)

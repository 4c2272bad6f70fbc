// fz_kernel_set.h -- host-visible tables of the ahead-of-time kernel instantiations.
//
// Per features-per-level F: the forward without MLP and the NeRF-level backward. Per (F, padded MLP input width P,
// P a multiple of 8 up to 16 (F + 1)): the forward with the fused MLP and the proposal-level backward.
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

constexpr int kMlpPadStep = 8;

// padded MLP input width of n_out features
__host__ __device__ constexpr int mlp_pad(const int n_out) { return (n_out + kMlpPadStep - 1) / kMlpPadStep * kMlpPadStep; }

}  // namespace zf

#define ZF_KSET_NAME2(F) zf_kernel_set_F##F
#define ZF_KSET_NAME(F) ZF_KSET_NAME2(F)
#define ZF_MLP_KSET_NAME2(F, P) zf_mlp_kernel_set_F##F##_P##P
#define ZF_MLP_KSET_NAME(F, P) ZF_MLP_KSET_NAME2(F, P)

// X(F, P) over the compiled MLP instantiations
#define ZF_FOR_EACH_MLP(X) \
    X(1, 8) X(1, 16) X(1, 24) X(1, 32) \
    X(2, 8) X(2, 16) X(2, 24) X(2, 32) X(2, 40) X(2, 48) \
    X(3, 8) X(3, 16) X(3, 24) X(3, 32) X(3, 40) X(3, 48) X(3, 56) X(3, 64) \
    X(4, 8) X(4, 16) X(4, 24) X(4, 32) X(4, 40) X(4, 48) X(4, 56) X(4, 64) X(4, 72) X(4, 80)

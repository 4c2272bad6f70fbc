/*
 * zf_mlp.h -- C ABI of the elementwise step of the NeRF MLP's backward that the reference fuses into its cuBLASLt
 * epilogues (CUBLASLT_EPILOGUE_DRELU_BGRAD, ZipNeRFCudaBackend/ZipNeRFCudaBackend/mlp/src/nerf_mlp.cu:583-591): the
 * gradient of a ReLU layer's output masked by the layer's activation, with the bias gradient (the column sums)
 * accumulated in the same pass. Used by the training-step driver's NeRF MLP (cuBLAS GEMMs). Conventions as
 * zf_featurize.h.
 */
#ifndef ZF_MLP_H
#define ZF_MLP_H

#include <stdint.h>

#include "zf_featurize.h"

#ifdef __cplusplus
extern "C" {
#endif

/* grad[r, c] = activation[r, c] > 0 ? grad[r, c] : 0 for r < n_rows, c < n_cols (bf16, in place; row strides in
 * elements, both rows 16-byte aligned, n_cols a multiple of 8 and at most 512); bias_grad (float [n_cols], or NULL)
 * += the column sums of the masked gradient, accumulated in fp32 with atomics (order not fixed). Replaces the
 * DRELU / DRELU_BGRAD cuBLASLt epilogues of NerfMlp::backward (nerf_mlp.cu:583-607). */
ZF_API int zf_relu_backward_bf16(uint16_t* grad, int64_t grad_stride, const uint16_t* activation, int64_t activation_stride, int64_t n_rows,
                                 int n_cols, float* bias_grad, struct CUstream_st* stream);

#ifdef __cplusplus
}
#endif

#endif

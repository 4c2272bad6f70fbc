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

/* Packed NeRF MLP weights of zf_nerf_mlp_forward_tc: bf16 [out x in] matrices with zero padding, each stored as
 * consecutive K-slices (all output rows, 64 input columns each; the combined layer's last slice 32; skip and rgb one
 * slice), every slice in the tensor cores' no-swizzle K-major order (8-row x 8-column core matrices of 128 bytes,
 * K-adjacent ones next, then the next 8 rows); zipnerf_b200.nerf_mlp.pack writes it. fp32 biases. The fold of the
 * reference's parameters (nerf_mlp.cu:186-234: bottleneck folded into the first view layer and the rgb skip columns,
 * biases of the layers that read the inputs in their last column). All 16-byte aligned. */
typedef struct zf_nerf_mlp_weights {
    const uint16_t* density;       /* [64, 64]: 56 feature columns, zero padding to the MMA K step */
    const float* density_bias;     /* [64] */
    const uint16_t* combined;      /* [256, 96] */
    const uint16_t* skip;          /* [16, 96]: rows 0-3 raw density and rgb skip terms, the others zero */
    const uint16_t* view_1;        /* [256, 256] */
    const float* view_1_bias;      /* [256] */
    const uint16_t* view_2;        /* [256, 256] */
    const float* view_2_bias;      /* [256] */
    const uint16_t* rgb;           /* [16, 256]: rows 1-3 the rgb weights, the others zero */
} zf_nerf_mlp_weights;

/* Bytes of the training forward's record for n samples: the hidden view-layer activations v0, v1, v2 ([3, n, 256]
 * bf16), then their ReLU masks ([3, n, 8] uint32: bit c % 32 of word c / 32 set where column c is positive), then the
 * hidden layer h's ([n, 2] uint32). No counterpart in the reference, whose training forward keeps v0-v2 in tensors it
 * allocates (nerf_mlp.cu:527-560). */
ZF_API int64_t zf_nerf_mlp_activations_size(int64_t n);

/* The forward of NerfMlp::forward (nerf_mlp.cu:503-560) for the reference model's widths, one persistent
 * tcgen05 kernel (bf16 operands in shared memory, fp32 accumulators in tensor memory, 128-sample tiles, one CTA per
 * SM; each sample's outputs depend on its own row only): features [n, 56] bf16,
 * inputs [n, 96] bf16 (the direction block in columns 64-95 is read, the hidden layer written to columns 0-63),
 * outputs [n, 8] bf16 (raw density, 3 rgb logits, 4 zeros); activations: NULL (inference), or the training record of
 * zf_nerf_mlp_activations_size(n) bytes, which receives v0, v1, v2 and the ReLU masks for the backward (the training
 * forward, as NerfMlp::forward with training = true keeps v0-v2, nerf_mlp.cu:527-560); row strides in elements,
 * multiples of 8; status: a device
 * int the kernel sets to 1 if one of its bounded waits ran out, which leaves this launch's outputs undefined (the
 * kernel still waits for its own copies and MMAs in flight and frees its tensor memory before it exits). Within bf16
 * rounding of the reference's cuBLASLt chain. */
ZF_API int zf_nerf_mlp_forward_tc(const uint16_t* features, int64_t features_stride, uint16_t* inputs, int64_t inputs_stride,
                                  const zf_nerf_mlp_weights* weights, uint16_t* outputs, uint16_t* activations, int64_t n, int* status,
                                  struct CUstream_st* stream);

/* Transposed packed NeRF MLP weights of zf_nerf_mlp_backward_tc ([inputs x outputs], the B operands of the data
 * gradients dX = dY W): bf16, stored as consecutive K-slices of the outputs (16 for rgb_t and skip_t, 64 for the others)
 * in the no-swizzle K-major order; zipnerf_b200.nerf_mlp.pack_transposed writes them. All 16-byte aligned. */
typedef struct zf_nerf_mlp_weights_t {
    const uint16_t* rgb_t;         /* [256, 16] */
    const uint16_t* view_2_t;      /* [256, 256] */
    const uint16_t* view_1_t;      /* [256, 256] */
    const uint16_t* combined_t;    /* [96, 256] */
    const uint16_t* skip_t;        /* [96, 16] */
    const uint16_t* density_t;     /* [64, 64] */
} zf_nerf_mlp_weights_t;

/* fp32 gradients of the packed weights (row-major, the shapes of zf_nerf_mlp_weights), accumulated (+=): density
 * [64, 64] (the first 56 columns), density_bias [64], combined [256, 96], skip [16, 96] (rows 0-7), view_1 and view_2
 * [256, 256], view_1_bias and view_2_bias [256], rgb [16, 256] (rows 0-7). */
typedef struct zf_nerf_mlp_grads {
    float* density;
    float* density_bias;
    float* combined;
    float* skip;
    float* view_1;
    float* view_1_bias;
    float* view_2;
    float* view_2_bias;
    float* rgb;
} zf_nerf_mlp_grads;

/* Bytes of the backward's workspace for n samples (the masked gradients g_v0, g_v1, g_v2 and g_h in bf16); no
 * counterpart in the reference, whose NerfMlp::backward allocates its intermediates itself (nerf_mlp.cu:575-582). */
ZF_API int64_t zf_nerf_mlp_backward_workspace_size(int64_t n);

/* The backward of NerfMlp::backward (nerf_mlp.cu:565-620) on the tcgen05 tensor cores, for the reference model's widths:
 * grad_outputs [n, 8] bf16 (columns 4-7 zero), features [n, 56] and inputs [n, 96] bf16 of the forward (h in columns
 * 0-63), activations the training forward's record (v0, v1, v2 and the ReLU masks), weights_t the transposed packed
 * weights; grad_features [n, 56] bf16 out; grads += the gradients of the packed weights (their unfold into the
 * reference's parameters is the caller's); workspace of zf_nerf_mlp_backward_workspace_size(n) bytes; n < 2^31 - 64.
 * Seven launches: the data-gradient chain of each 128-sample tile (masked by the record's ReLU masks), then six weight
 * gradients as split-K GEMMs over the samples (TMA tensor copies of this GPU's memory, no multicast) with fp32 atomics.
 * status: as zf_nerf_mlp_forward_tc. */
ZF_API int zf_nerf_mlp_backward_tc(const uint16_t* grad_outputs, const uint16_t* features, int64_t features_stride, const uint16_t* inputs,
                                   int64_t inputs_stride, const uint16_t* activations, const zf_nerf_mlp_weights_t* weights_t,
                                   uint16_t* grad_features, int64_t grad_features_stride, const zf_nerf_mlp_grads* grads, void* workspace,
                                   int64_t workspace_bytes, int64_t n, int* status, struct CUstream_st* stream);

/* Targets of zf_nerf_mlp_pack (any may be NULL: not written), the packed operands of NerfMlp::pack for the reference
 * model's widths (nerf_mlp.cu:493-501, pack_kernel nerf_mlp.cu:186-234):
 * - the layer chain's bf16 row-major weights: density [64, 56], density_bias [64], combined [256, 96], skip [8, 96],
 *   view_1 and view_2 [256, 256], view_1_bias and view_2_bias [256], rgb [8, 256] (the reference's packed tensors);
 * - the tensor-core forward's operands (zf_nerf_mlp_weights): bf16 weights in its K-slice order (density [64, 64],
 *   combined [256, 96], skip [16, 96], view_1 and view_2 [256, 256], rgb [16, 256]) and the bf16-rounded biases as fp32;
 * - the tensor-core backward's transposed operands (zf_nerf_mlp_weights_t). */
typedef struct zf_nerf_mlp_packed {
    uint16_t* density;
    uint16_t* density_bias;
    uint16_t* combined;
    uint16_t* skip;
    uint16_t* view_1;
    uint16_t* view_1_bias;
    uint16_t* view_2;
    uint16_t* view_2_bias;
    uint16_t* rgb;
    uint16_t* tc_density;
    float* tc_density_bias;
    uint16_t* tc_combined;
    uint16_t* tc_skip;
    uint16_t* tc_view_1;
    float* tc_view_1_bias;
    uint16_t* tc_view_2;
    float* tc_view_2_bias;
    uint16_t* tc_rgb;
    uint16_t* rgb_t;
    uint16_t* view_2_t;
    uint16_t* view_1_t;
    uint16_t* combined_t;
    uint16_t* skip_t;
    uint16_t* density_t;
} zf_nerf_mlp_packed;

/* Elements of the fp32 parameter buffer of the reference model's widths (nerf_mlp_parameters(50, 64, 256, 256, 4),
 * nerf_mlp.cu:440-455): 227,556. */
ZF_API int64_t zf_nerf_mlp_parameter_count(void);

/* NerfMlp::pack (nerf_mlp.cu:493-501) for the reference model's widths, one launch: folds the fp32 parameters (the
 * bottleneck into the first view layer and the rgb skip rows, the biases of the layers reading the inputs into the bias
 * lane) with the reference's fp32 multiply-add order and rounds to bf16, writing every given target. */
ZF_API int zf_nerf_mlp_pack(const float* params, const zf_nerf_mlp_packed* out, struct CUstream_st* stream);

/* The unfold of NerfMlp::backward (unpack_kernel, nerf_mlp.cu:236-284, 616-617) for the reference model's widths, one
 * launch: grad_params (fp32, the parameter layout) += the chain rule of the fold applied to the packed-weight
 * gradients of zf_nerf_mlp_backward_tc (fp32; the reference's bias gradients are bf16). */
ZF_API int zf_nerf_mlp_unfold_grads(const float* params, const zf_nerf_mlp_grads* grads, float* grad_params, struct CUstream_st* stream);

#ifdef __cplusplus
}
#endif

#endif

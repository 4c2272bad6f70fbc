/*
 * zf_optim.h -- C ABI of the B200 (sm_100a) fused Adam step of Fused Zip-NeRF's hash grids and MLP parameters.
 *
 * Replaces zipnerf::optimizer::Adam (ZipNeRFCudaBackend/ZipNeRFCudaBackend/optimizer/include/optimizer_api.h:10-40,
 * src/optimizer_api.cu:132-221) and its binding (torch_bindings/bindings.cu:31-35). One launch per step over all
 * buffers: gradients (fp32, or fp16 clamped to the fp16 range) are divided by their buffer's grad_scale, NaNs become
 * 0 and infinities the largest float (jnp.nan_to_num), grid levels add the gradient of the regularizer
 * 0.5 reg_weight mean(p^2), the moments and parameters take the Adam update (beta1, beta2, eps, bias corrections of
 * the step count), and every gradient is zeroed for the next accumulation. The step also writes, per grid level in
 * buffer order, magnitudes[level] = sqrt(max_value^2 + mean(p^2)) of the updated parameters and the regularizer
 * value 0.5 reg_weight sum_levels mean(p^2) (both device floats). Conventions as zf_featurize.h.
 */
#ifndef ZF_OPTIM_H
#define ZF_OPTIM_H

#include <stdint.h>

#include "zf_featurize.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct zf_adam zf_adam;

/* One optimized buffer (a contiguous device array of numel floats, numel a multiple of 4, 16-byte aligned) and its
 * gradient of the same size. level_offsets: n_level_offsets element offsets of the grid levels in the buffer, from 0
 * to numel, each a multiple of 4 and increasing (NULL / 0: the buffer has no levels and no regularizer). */
typedef struct zf_adam_buffer {
    float* param;
    void* grad;                 /* float, or fp16 bits (uint16_t) when grad_half is nonzero */
    int grad_half;
    int64_t numel;
    double grad_scale;
    const int64_t* level_offsets;
    int n_level_offsets;
} zf_adam_buffer;

/* Adam ctor (optimizer_api.cu:132-158): 1 to 8 buffers with at most 32 levels in all; the moments (zero) are device
 * arrays of the object, allocated on the current device. magnitudes: device float [n_magnitudes], n_magnitudes = the
 * number of levels; regularization: a device float. The buffers, magnitudes and regularization stay owned by the
 * caller and must outlive the object. */
ZF_API int zf_adam_create(const zf_adam_buffer* buffers, int n_buffers, double reg_weight, double max_value, double beta1, double beta2,
                          double eps, float* magnitudes, int64_t n_magnitudes, float* regularization, zf_adam** out);
/* frees the moments and scratch arrays (the end of an Adam object's lifetime) */
ZF_API void zf_adam_destroy(zf_adam* adam);

/* Adam::step (optimizer_api.cu:160-220): the next step (counting from 1) with learning rate lr, on the stream. The
 * steps of one object share its scratch arrays (per-block sums, a completion counter that the last block resets):
 * enqueue them on one stream, or order them, as the reference's single-stream use does. */
ZF_API int zf_adam_step(zf_adam* adam, double lr, struct CUstream_st* stream);

/* The moments of one buffer (device float [numel] each) and the steps taken so far; no counterpart in the reference,
 * whose moments are private. */
ZF_API int zf_adam_state(const zf_adam* adam, int buffer, float** exp_avg, float** exp_avg_sq, int64_t* steps);

#ifdef __cplusplus
}
#endif

#endif

/*
 * zf_sampling.h -- C ABI of the B200 (sm_100a) per-ray sampling steps around the featurization.
 *
 * Replaces the producers of the featurizer's interval endpoints in Fused Zip-NeRF's ZipNeRFCudaBackend
 * (ZipNeRFCudaBackend/ZipNeRFCudaBackend/sampling/include/sampling_api.h:10-58, src/sampling_api.cu:447-578):
 * generate_rays, view_rays, initialize_rays, sample_uniforms and composite_and_resample; and the final level's losses
 * and compositing around the NeRF MLP (sampling_api.h:60-90, sampling_api.cu:580-678): train_final and composite_final.
 * Conventions as zf_featurize.h: plain device pointers, an int status (ZF_OK or an error code, message in
 * zf_last_error()), no exceptions, asynchronous launches on the given stream. The caller allocates every output; the reference's wrappers
 * allocate them and return tensors, which the PyTorch binding does on top of these calls.
 *
 * Layouts (row-major; n = intervals of the level, n_samples = intervals of the produced level):
 *   origins, directions, rgb  float [n_rays, 3]          radii  float [n_rays]
 *   sdist, tdist              float [n_rays, n + 1]      encoded_directions  bf16 [n_rays, zf_direction_block_width()]
 *   raw_density, weights      float [n_rays, n]
 * Supported: 2 <= n, n_samples <= 64 (sampling_api.cu:443-445), n_rays <= 2^31 - 1.
 */
#ifndef ZF_SAMPLING_H
#define ZF_SAMPLING_H

#include <stdint.h>

#include "zf_featurize.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Mapping between normalized ray distances s in [0, 1] and metric distances t: the seven float32 constants of
 * utils.ray_warp (utils.py:19-27) in the order of the reference's RayWarp (ray_ops.cuh:16-18). */
typedef struct zf_ray_warp {
    float near, far, fn_near, fn_far, power, premult, y_max;
} zf_ray_warp;

/* initialize_rays_wrapper (sampling_api.cu:520-539): the encoded view directions and first-level intervals of given
 * rays; seed >= 0 jitters each ray's samples with the counter-based stream 2, seed < 0 centers them. */
typedef struct zf_initialize_rays_args {
    int64_t seed;
    const float* directions;
    int64_t n_rays;
    int direction_degree;
    int n_samples;
    zf_ray_warp warp;
    uint16_t* encoded_directions;
    float* sdist;
    float* tdist;
} zf_initialize_rays_args;

/* view_rays_wrapper (sampling_api.cu:487-518): inference rays of the given pixels of one view, centered samples. */
typedef struct zf_view_rays_args {
    const int64_t* pixel_indices;        /* [n_rays] indices into local_directions */
    int64_t n_rays;
    const float* local_directions;       /* [*, 3] camera-space directions of the view's camera */
    const float* c2w;                    /* [3, 4] camera-to-world */
    float radius;
    int direction_degree;
    int n_samples;
    zf_ray_warp warp;
    float* origins;
    float* directions;
    float* radii;
    uint16_t* encoded_directions;
    float* sdist;
    float* tdist;
} zf_view_rays_args;

/* generate_rays_wrapper (sampling_api.cu:447-485): rays, colors, encodings and jittered first-level intervals of
 * n_rays random pixels of all training views (pixel i of the batch: stream 0, index i; jitter: stream 2). */
typedef struct zf_generate_rays_args {
    int64_t seed;
    int64_t n_rays;
    const int64_t* view_offsets;         /* [n_views + 1] first pool pixel of each view */
    int n_views;
    const int32_t* view_cameras;         /* [n_views] camera of each view */
    const int64_t* camera_offsets;       /* [n_cameras + 1] first local direction of each camera */
    const float* local_directions;       /* [*, 3] camera-space pixel directions of all cameras */
    const float* c2w;                    /* [n_views, 3, 4] */
    const float* camera_radii;           /* [n_cameras] */
    const uint8_t* pool_rgb;             /* [n_pixels, 3] */
    int64_t n_pixels;
    int direction_degree;
    int n_samples;
    zf_ray_warp warp;
    float* origins;
    float* directions;
    float* radii;
    float* rgb;
    uint16_t* encoded_directions;
    float* sdist;
    float* tdist;
} zf_generate_rays_args;

/* composite_and_resample_wrapper (sampling_api.cu:550-578): the alpha-compositing weights of a proposal level's raw
 * densities and the next level's n_samples intervals resampled from them (softmax(anneal log w); seed >= 0 jitters
 * with stream 2 + next_level, seed < 0 centers). weights may be NULL (inference discards them). */
typedef struct zf_resample_args {
    const float* raw_density;
    const float* sdist;
    const float* tdist;
    const float* directions;
    int64_t n_rays;
    int n_intervals;
    float anneal;
    int n_samples;
    int64_t seed;
    int next_level;
    zf_ray_warp warp;
    float* weights;
    float* sdist_next;
    float* tdist_next;
} zf_resample_args;

/* One proposal level of zf_train_final (the ProposalLevels of sampling_api.cu:17-27): its raw densities, interval edges
 * and compositing weights (as composite_and_resample returned them), the gradient it receives (written, not
 * accumulated), and its interlevel loss weight and blur half width. */
typedef struct zf_proposal_level {
    int n_intervals;
    const float* raw_density;            /* [n_rays, n_intervals] */
    const float* sdist;                  /* [n_rays, n_intervals + 1] */
    const float* tdist;
    const float* weights;                /* [n_rays, n_intervals] */
    float* raw_density_grad;             /* [n_rays, n_intervals] */
    float interlevel_weight;
    float interlevel_blur;
} zf_proposal_level;

/* train_final_wrapper (sampling_api.cu:580-645): the training losses of a ray batch and the gradients of every level's
 * raw outputs. nerf_outputs: bf16 [n_rays, n_intervals, 8] (raw density, rgb logits, padding) of the final level;
 * nerf_outputs_grad: bf16 [n_rays, n_intervals, 8] (written); loss_sums: NULL or float [4] that the (data, mse,
 * interlevel, distortion) sums are added to, divided by n_rays (the reference returns them from zeros). */
typedef struct zf_train_final_args {
    const uint16_t* nerf_outputs;
    const float* sdist;
    const float* tdist;
    int64_t n_rays;
    int n_intervals;
    const zf_proposal_level* proposals;
    int n_proposal_levels;               /* <= 4 */
    const float* directions;
    int64_t seed;                        /* random backgrounds: stream 1, index 3 ray + channel */
    const float* rgb_target;             /* [n_rays, 3] */
    float charbonnier_padding;
    float distortion_weight;
    float distortion_power;
    float distortion_premult;
    uint16_t* nerf_outputs_grad;
    float* loss_sums;
} zf_train_final_args;

/* composite_final_wrapper (sampling_api.cu:647-678): color (over the given background), opacity and the expected
 * log-distance (or median) depth of every ray, written to its pixel; alpha and depth may be NULL. */
typedef struct zf_composite_final_args {
    const uint16_t* nerf_outputs;        /* bf16 [n_rays, n_intervals, 8] */
    const float* tdist;                  /* [n_rays, n_intervals + 1] */
    int64_t n_rays;
    int n_intervals;
    const float* directions;
    const float* background;             /* [3] */
    const int64_t* pixel_indices;        /* [n_rays] */
    float* rgb;                          /* [pixels, 3] */
    float* alpha;                        /* [pixels] */
    float* depth;                        /* [pixels] */
    int use_median_depth;
} zf_composite_final_args;

/* width of the encoded view direction block: (3 + 6 degree + 1) rounded up to a multiple of 8 (zipnerf_config.h:18) */
ZF_API int64_t zf_direction_block_width(int direction_degree);

/* initialize_rays_wrapper (sampling_api.cu:522-541) */
ZF_API int zf_initialize_rays(const zf_initialize_rays_args* args, struct CUstream_st* stream);
/* view_rays_wrapper (sampling_api.cu:489-520) */
ZF_API int zf_view_rays(const zf_view_rays_args* args, struct CUstream_st* stream);
/* generate_rays_wrapper (sampling_api.cu:446-487) */
ZF_API int zf_generate_rays(const zf_generate_rays_args* args, struct CUstream_st* stream);

/* sample_uniforms_wrapper (sampling_api.cu:541-548): values[i] = the uniform of (seed, stream_index, i), i < n */
ZF_API int zf_sample_uniforms(int64_t seed, int64_t stream_index, int64_t n, float* values, struct CUstream_st* stream);

/* composite_and_resample_wrapper (sampling_api.cu:552-581) */
ZF_API int zf_composite_and_resample(const zf_resample_args* args, struct CUstream_st* stream);

/* train_final_wrapper (sampling_api.cu:583-647) */
ZF_API int zf_train_final(const zf_train_final_args* args, struct CUstream_st* stream);
/* composite_final_wrapper (sampling_api.cu:649-679) */
ZF_API int zf_composite_final(const zf_composite_final_args* args, struct CUstream_st* stream);

#ifdef __cplusplus
}
#endif

#endif

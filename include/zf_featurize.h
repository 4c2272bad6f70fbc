/*
 * zf_featurize.h -- C ABI of the B200 (sm_100a) multisampled hash-grid featurization.
 *
 * Drop-in replacement for the featurization path of Fused Zip-NeRF's ZipNeRFCudaBackend: the class
 * zipnerf::featurization::Featurizer (ZipNeRFCudaBackend/ZipNeRFCudaBackend/featurization/include/featurizer.h:22-95,
 * src/featurizer.cu:145-355) and its Python binding (torch_bindings/bindings.cu:14-22). Every entry point takes plain
 * device pointers and sizes, returns an int status (ZF_OK or an error code, with a message from zf_last_error()), never
 * throws, and launches asynchronously on the given CUDA stream (NULL: the legacy default stream).
 *
 * Tensor layouts are the reference's (row-major, element counts in the comments):
 *   origins, directions  float [n_rays, 3]
 *   radii                float [n_rays]
 *   tdist                float [n_rays, n_intervals + 1]   (a sample is one interval; n_samples = n_rays * n_intervals)
 *   table                float [rows, n_features]           (rows = sum of level_entries; Model.py:24)
 *   scale_magnitudes     float [n_levels]
 *   w0 [mlp_width, n_out], b0 [mlp_width], w1 [mlp_width], b1 [1]  float, n_out = n_levels * (n_features + 1)
 * bf16 and fp16 values are passed as their 16-bit patterns (uint16_t).
 */
#ifndef ZF_FEATURIZE_H
#define ZF_FEATURIZE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct CUstream_st;  /* cudaStream_t */

#if defined(__GNUC__)
#define ZF_API __attribute__((visibility("default")))
#else
#define ZF_API
#endif

#define ZF_OK 0
#define ZF_ERROR_INVALID_ARGUMENT 1  /* a size, pointer or layout the reference rejects as well */
#define ZF_ERROR_UNSUPPORTED 2       /* a layout outside this build's compiled range (see zf_featurizer_create) */
#define ZF_ERROR_CUDA 3              /* a CUDA runtime error (launch or device query) */

typedef struct zf_featurizer zf_featurizer;

/* Rays and interval endpoints of one call (the first five tensor arguments of Featurizer::forward/backward/backward_mlp,
 * featurizer.h:36-40). pattern_seed >= 0 draws random multisample pattern flips and rotations from the counter-based
 * stream 16 + level (random.cuh:12) at index sample_offset + sample; pattern_seed < 0 alternates flips with a pi/6
 * rotation. sample_offset is 0 for the reference's behaviour; a shard of a larger batch passes the batch index of its
 * first sample, so that the shards together draw exactly the patterns of the whole batch. */
typedef struct zf_rays {
    const float* origins;
    const float* directions;
    const float* radii;
    const float* tdist;
    int64_t n_rays;
    int64_t n_intervals;
    int64_t pattern_seed;
    int64_t sample_offset;
} zf_rays;

/* Arguments of zf_featurize_forward (Featurizer::forward, featurizer.h:35-52). A NULL output is skipped, as an empty
 * tensor is in the reference. The MLP weights are read only when raw_density is given. */
typedef struct zf_forward_args {
    zf_rays rays;
    int interleave;                      /* nonzero: one interval of 32 consecutive rays per warp (coherent rays) */
    const float* table;
    int64_t table_rows;                  /* must equal the featurizer's row count */
    const float* scale_magnitudes;
    const float* w0;
    const float* b0;
    const float* w1;
    const float* b1;
    int64_t w0_numel;                    /* must equal mlp_width * n_out when raw_density is given */
    float* raw_density;                  /* [n_samples] */
    float* features_float;               /* [n_samples, n_out] */
    uint16_t* features_bf16;             /* bf16 [n_samples, features_bf16_width], width >= n_out, zero-padded */
    int64_t features_bf16_width;
    const uint16_t* encoded_directions;  /* bf16 [n_rays, encoded_width] */
    int64_t encoded_width;
    uint16_t* nerf_inputs;               /* bf16 [n_samples, nerf_inputs_width]: the last encoded_width columns are the
                                            encoded direction with its last column set to 1.0 (bias lane) */
    int64_t nerf_inputs_width;
} zf_forward_args;

/* Arguments of zf_featurize_backward (Featurizer::backward, featurizer.h:56-64): accumulates the NeRF grid gradient,
 * scaled by zf_nerf_grid_grad_scale(), into grad_table (fp32, the first zf_featurizer_n_fp32_grad_rows() rows) and
 * grad_table_half (fp16, the remaining rows). */
typedef struct zf_backward_args {
    zf_rays rays;
    const uint16_t* grad_features;       /* bf16 [n_samples, grad_features_cols], row stride grad_features_stride */
    int64_t grad_features_cols;          /* >= n_out */
    int64_t grad_features_stride;        /* elements between rows */
    float* grad_table;                   /* fp32 [n_fp32_grad_rows * n_features], accumulated into */
    int64_t grad_table_numel;
    uint16_t* grad_table_half;           /* fp16 [(rows - n_fp32_grad_rows) * n_features], accumulated into */
    int64_t grad_table_half_numel;
} zf_backward_args;

/* Arguments of zf_featurize_backward_mlp (Featurizer::backward_mlp, featurizer.h:67-82): recomputes the fused MLP
 * from the stored fp32 features and accumulates the fp32 grid gradient and the MLP parameter gradients. */
typedef struct zf_backward_mlp_args {
    zf_rays rays;
    const float* features;               /* [n_samples, n_out] as written by forward's features_float */
    int64_t features_numel;
    const float* grad_raw_density;       /* [n_samples] */
    int64_t grad_raw_density_numel;
    const float* w0;
    const float* b0;
    const float* w1;
    int64_t w0_numel;
    float* grad_table;                   /* fp32 [rows * n_features], accumulated into */
    int64_t grad_table_numel;
    float* grad_w0;                      /* [mlp_width, n_out], accumulated into */
    int64_t grad_w0_numel;
    float* grad_b0;                      /* [mlp_width] */
    float* grad_w1;                      /* [mlp_width] */
    float* grad_b1;                      /* [1] */
    void* workspace;                     /* optional device scratch (16-byte aligned) of at least
                                            zf_featurize_backward_mlp_workspace_size() bytes; NULL: the call takes it
                                            from the featurizer's own stream-ordered memory pool, which keeps the
                                            largest workspace used reserved until zf_featurizer_destroy */
    int64_t workspace_bytes;
} zf_backward_mlp_args;

/* Creates a featurizer for one sampling level (Featurizer ctor, featurizer.h:25 / featurizer.cu:145-155) on the
 * current CUDA device. level selects the pattern stream; level_sizes / level_entries give each grid level's
 * resolution and table entries (a level is hashed when size^3 > entries; its rows follow the previous levels').
 * Supported here: 1 <= n_levels <= 16, 1 <= n_features <= 4, 0 <= mlp_width (0: no fused MLP), rows * n_features
 * <= 2^32 - 1, level sizes <= 65534 (the kernels pack cell coordinates into 16 bits). */
ZF_API int zf_featurizer_create(int level, const int64_t* level_sizes, const int64_t* level_entries, int n_levels,
                         int n_features, int mlp_width, zf_featurizer** out);
/* releases the featurizer and its workspace pool (the end of a Featurizer's lifetime) */
ZF_API void zf_featurizer_destroy(zf_featurizer* featurizer);

/* n_levels * (n_features + 1) (Featurizer::n_output_features, featurizer.h:27) */
ZF_API int zf_featurizer_n_output_features(const zf_featurizer* featurizer);
/* table rows of the leading levels with fewer than 2^20 entries, whose NeRF-level gradient is fp32
 * (Featurizer::n_fp32_grad_rows, featurizer.h:30) */
ZF_API int64_t zf_featurizer_n_fp32_grad_rows(const zf_featurizer* featurizer);
/* total table rows (sum of level_entries, the grid's last offset, Model.py:22); no Featurizer counterpart */
ZF_API int64_t zf_featurizer_n_rows(const zf_featurizer* featurizer);
/* kernel launches of one call (no counterpart in the reference, which launches one kernel per call): call 0 =
 * zf_featurize_forward without the MLP, 1 = with the MLP, 2 = zf_featurize_backward, 3 = zf_featurize_backward_mlp.
 * Grids larger than the L2 run their forward and backward as level passes, one launch each; 0 for other calls. */
ZF_API int zf_featurizer_launches(const zf_featurizer* featurizer, int call);

/* Featurizer::forward (featurizer.cu:188-264) */
ZF_API int zf_featurize_forward(zf_featurizer* featurizer, const zf_forward_args* args, struct CUstream_st* stream);
/* Featurizer::backward (featurizer.cu:266-299) */
ZF_API int zf_featurize_backward(zf_featurizer* featurizer, const zf_backward_args* args, struct CUstream_st* stream);
/* Featurizer::backward_mlp (featurizer.cu:301-355). Runs as two kernels: the MLP recomputation with the parameter
 * gradient reduction, which writes each sample's feature gradient to the workspace, and the scatter of those into
 * grad_table. */
ZF_API int zf_featurize_backward_mlp(zf_featurizer* featurizer, const zf_backward_mlp_args* args, struct CUstream_st* stream);
/* workspace bytes of zf_featurize_backward_mlp for n_samples intervals (n_samples * n_output_features floats); no
 * reference counterpart (its backward_mlp is one kernel) */
ZF_API int64_t zf_featurize_backward_mlp_workspace_size(const zf_featurizer* featurizer, int64_t n_samples);
/* zf_featurize_backward_mlp without any device allocation. No counterpart in the reference. For callers that must not
 * allocate device memory while they run (a host with a fixed device-memory budget, or a plugin whose framework owns
 * every device allocation) and cannot pass a workspace: the workspace is a static 32 MiB device array of this library,
 * held by every GPU that loads it until the process exits, so a call takes at most
 * 32 MiB / (4 * n_output_features) samples (419430 at 20 output features) and larger calls fail with
 * ZF_ERROR_INVALID_ARGUMENT. args->workspace is ignored. The first call on a device looks up the array's address on that
 * device (make it before any stream capture). All calls share the array: calls whose kernels overlap on the GPU (other
 * streams, other threads) race and must be serialized by the caller. The array keeps the last call's contents; every
 * call overwrites what it reads, so nothing needs clearing. */
ZF_API int zf_featurize_backward_mlp_no_alloc(zf_featurizer* featurizer, const zf_backward_mlp_args* args, struct CUstream_st* stream);

/* Intermediate values of the listed samples, for exact checks of sample placement, contraction and hashing. No
 * counterpart in the reference (whose kernels keep these in registers). Outputs (device memory, n = n_debug):
 * x float [n, 6, 3] contracted positions in [0,1]^3; scale float [n, 6]; contracted int32 [n, 6] (|p|^2 > 1);
 * n_groups int32 [n, n_levels] merged corner groups; rows uint32 [n, n_levels, 6, 8] and weights float
 * [n, n_levels, 6, 8] (groups beyond n_groups are zero). */
ZF_API int zf_featurize_debug(zf_featurizer* featurizer, const zf_rays* rays, const uint32_t* samples, int64_t n_debug,
                       float* x, float* scale, int32_t* contracted, int32_t* n_groups, uint32_t* rows, float* weights,
                       struct CUstream_st* stream);

/* Numerics self-check of this build (no counterpart in the reference). The per-level erf downweighting
 * sign(x) sqrt(1 - exp(-4 x^2 / pi)) of featurize_common.cuh:45-47 is evaluated for every float whose bit pattern lies in
 * [first_bits, last_bits]; *n_not_one (device, zeroed by the caller) counts the arguments whose result is not exactly
 * 1.0f and *max_bits (device, zeroed by the caller) receives the largest such bit pattern. The kernels skip the erf for
 * arguments >= zf_erf_saturation_threshold(); the check over [threshold, +inf) must count 0 on every device. */
ZF_API int zf_check_erf_saturation(uint32_t first_bits, uint32_t last_bits, unsigned long long* n_not_one, uint32_t* max_bits,
                                   struct CUstream_st* stream);
/* the smallest argument of the kernels' erf early-out; no reference counterpart */
ZF_API float zf_erf_saturation_threshold(void);

/* Message of the calling thread's last failed call ("" if none): the text of the std::runtime_error the reference
 * would have thrown (featurizer.cu:127-138). */
ZF_API const char* zf_last_error(void);

/* Module constants of the reference binding (bindings.cu:14-15): the hash grid initialization range over the
 * feature preconditioning (1e-5), and the static scale of the NeRF grid gradients (2^20). */
ZF_API double zf_grid_max_value(void);
/* nerf_grid_grad_scale (bindings.cu:15) */
ZF_API double zf_nerf_grid_grad_scale(void);

#ifdef __cplusplus
}
#endif

#endif

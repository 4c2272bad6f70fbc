/*
 * zf_step_oracle.c -- CPU restatement of the reference's per-ray sampling steps and its Adam step
 * (TEST INFRASTRUCTURE ONLY: the checker of the product's sampling and optimizer kernels; the product never loads it).
 *
 * Restates, in plain C with IEEE float arithmetic (libm, no contraction: oracle/Makefile), the algorithms of
 * B/sampling/include/ray_ops.cuh:20-99 and B/sampling/src/sampling_api.cu:41-196 (B/ = ZipNeRFCudaBackend/
 * ZipNeRFCudaBackend/), the counter-based random numbers of B/common/include/random.cuh:15-34, and the Adam step of
 * B/optimizer/src/optimizer_api.cu:43-127,160-220. Pinned bit for bit to the reference's own sampling functions built
 * for the host (oracle/ref_cpu/ref_sampling.cpp, tests/test_oracle.py). The reference's Adam kernel has no host build
 * (it sits in a libtorch source): the Adam restatement is pinned against the reference kernel itself on the GPU
 * (tests/test_gpu_sampling.py).
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#define MAX_INTERVALS 64  /* ray_ops.cuh:10 */

typedef struct {
    float near, far, fn_near, fn_far, power, premult, y_max;
} warp_t;

/* splitmix64 counter hash and the uniforms drawn from it (random.cuh:15-34) */
static uint64_t splitmix64(uint64_t x) {
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

static uint64_t counter_hash(uint64_t seed, uint64_t stream, uint64_t index) { return splitmix64(splitmix64(seed ^ (stream << 56)) ^ index); }

static float uniform(uint64_t seed, uint64_t stream, uint64_t index) { return (float)(counter_hash(seed, stream, index) >> 40) * (1.0f / 16777216.0f); }

static uint64_t uniform_int(uint64_t seed, uint64_t stream, uint64_t index, uint64_t n) {
    return (uint64_t)(((unsigned __int128)counter_hash(seed, stream, index) * n) >> 64);
}

/* float -> bf16 bits, round to nearest even */
static uint16_t to_bf16(float value) {
    uint32_t bits;
    memcpy(&bits, &value, sizeof(bits));
    if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x40u);
    bits += 0x7fffu + ((bits >> 16) & 1u);
    return (uint16_t)(bits >> 16);
}

/* normalized -> metric distance, inverse power ladder (ray_ops.cuh:26-33) */
static float normalized_to_metric(float s, const warp_t* w) {
    float y = s * w->fn_far + (1.0f - s) * w->fn_near;
    float magnitude = w->power < 0.0f ? fminf(fabsf(y), w->y_max) : fabsf(y);
    float q = fabsf(w->power - 1.0f);
    float x = copysignf(q * (powf(w->power / q * magnitude + 1.0f, 1.0f / w->power) - 1.0f), y) / w->premult;
    return fminf(fmaxf(x, w->near), w->far);
}

/* n_out intervals resampled from the step function (t, softmax(anneal log w)) of n bins (ray_ops.cuh:41-88) */
static void resample(const float* t, const float* w, int n, float anneal, int n_out, float jitter, float* s_out) {
    float p[MAX_INTERVALS], cdf[MAX_INTERVALS + 1], centers[MAX_INTERVALS];
    float largest = -INFINITY;
    for (int i = 0; i < n; i++) {
        p[i] = t[i + 1] > t[i] ? anneal * logf(fmaxf(w[i], FLT_MIN)) : -INFINITY;
        largest = fmaxf(largest, p[i]);
    }
    float total = 0.0f;
    for (int i = 0; i < n; i++) {
        p[i] = p[i] == -INFINITY ? 0.0f : expf(p[i] - largest);
        total += p[i];
    }
    float running = 0.0f;
    cdf[0] = 0.0f;
    for (int i = 1; i < n; i++) {
        running += p[i - 1] / total;
        cdf[i] = fminf(running, 1.0f);
    }
    cdf[n] = 1.0f;
    float first, step;
    if (jitter >= 0.0f) {
        float u_max = FLT_EPSILON + (1.0f - FLT_EPSILON) / (float)n_out;
        step = (1.0f - u_max) / (float)(n_out - 1);
        first = jitter * (step - FLT_EPSILON);
    } else {
        float pad = 1.0f / (float)(2 * n_out);
        first = pad;
        step = (1.0f - 2.0f * pad - FLT_EPSILON) / (float)(n_out - 1);
    }
    int k = 0; /* cdf entries <= u */
    for (int j = 0; j < n_out; j++) {
        float u = first + (float)j * step;
        while (k <= n && cdf[k] <= u) k++;
        int lo = k - 1 < 0 ? 0 : k - 1, hi = k > n ? n : k;
        float frac = (u - cdf[lo]) / fmaxf(FLT_EPSILON * FLT_EPSILON, cdf[hi] - cdf[lo]);
        frac = fminf(fmaxf(frac, 0.0f), 1.0f);
        centers[j] = t[lo] + frac * (t[hi] - t[lo]);
    }
    for (int j = 1; j < n_out; j++) s_out[j] = fminf(fmaxf(0.5f * (centers[j - 1] + centers[j]), 0.0f), 1.0f);
    s_out[0] = fminf(fmaxf(2.0f * centers[0] - 0.5f * (centers[0] + centers[1]), 0.0f), 1.0f);
    s_out[n_out] = fminf(fmaxf(2.0f * centers[n_out - 1] - 0.5f * (centers[n_out - 2] + centers[n_out - 1]), 0.0f), 1.0f);
}

static float norm3(const float* v) { return sqrtf(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]); }

int oracle_direction_block_width(int degree) { return (3 + 6 * degree + 1 + 7) / 8 * 8; } /* zipnerf_config.h:18 */

/* encoding and first-level intervals of one ray (sampling_api.cu:41-62) */
static void new_ray(const float* d, float jitter, int degree, int n_samples, const warp_t* warp, uint16_t* encoded, float* sdist, float* tdist) {
    float inv = 1.0f / norm3(d);
    float v[3] = {d[0] * inv, d[1] * inv, d[2] * inv};
    int width = oracle_direction_block_width(degree);
    for (int i = 0; i < width; i++) encoded[i] = 0;
    for (int c = 0; c < 3; c++) {
        encoded[c] = to_bf16(v[c]);
        for (int k = 0; k < degree; k++) {
            float x = ldexpf(v[c], k);
            encoded[3 + 3 * k + c] = to_bf16(sinf(x));
            encoded[3 + 3 * (degree + k) + c] = to_bf16(cosf(x));
        }
    }
    const float unit[2] = {0.0f, 1.0f}, one[1] = {1.0f};
    resample(unit, one, 1, 1.0f, n_samples, jitter, sdist);
    for (int i = 0; i <= n_samples; i++) tdist[i] = normalized_to_metric(sdist[i], warp);
}

static void camera_ray(const float* m, const float* l, float* d) {
    d[0] = m[0] * l[0] + m[1] * l[1] + m[2] * l[2];
    d[1] = m[4] * l[0] + m[5] * l[1] + m[6] * l[2];
    d[2] = m[8] * l[0] + m[9] * l[1] + m[10] * l[2];
}

/* initialize_rays (sampling_api.cu:150-166) */
void oracle_initialize_rays(int64_t seed, const float* directions, int n_rays, int degree, int n_samples, const float* warp, uint16_t* encoded,
                            float* sdist, float* tdist) {
    int width = oracle_direction_block_width(degree);
    for (int r = 0; r < n_rays; r++) {
        float jitter = seed >= 0 ? uniform((uint64_t)seed, 2, (uint64_t)r) : -1.0f;
        new_ray(directions + 3 * (int64_t)r, jitter, degree, n_samples, (const warp_t*)warp, encoded + (int64_t)r * width,
                sdist + (int64_t)r * (n_samples + 1), tdist + (int64_t)r * (n_samples + 1));
    }
}

/* view_rays (sampling_api.cu:120-147) */
void oracle_view_rays(const int64_t* pixels, int n_rays, const float* local, const float* c2w, float radius, int degree, int n_samples,
                      const float* warp, float* origins, float* directions, float* radii, uint16_t* encoded, float* sdist, float* tdist) {
    int width = oracle_direction_block_width(degree);
    for (int r = 0; r < n_rays; r++) {
        float* d = directions + 3 * (int64_t)r;
        camera_ray(c2w, local + 3 * pixels[r], d);
        origins[3 * r] = c2w[3];
        origins[3 * r + 1] = c2w[7];
        origins[3 * r + 2] = c2w[11];
        radii[r] = radius;
        new_ray(d, -1.0f, degree, n_samples, (const warp_t*)warp, encoded + (int64_t)r * width, sdist + (int64_t)r * (n_samples + 1),
                tdist + (int64_t)r * (n_samples + 1));
    }
}

/* generate_rays (sampling_api.cu:72-117) */
void oracle_generate_rays(int64_t seed, int n_rays, const int64_t* view_offsets, int n_views, const int32_t* view_cameras,
                          const int64_t* camera_offsets, const float* local, const float* c2w, const float* camera_radii, const uint8_t* pool_rgb,
                          int64_t n_pixels, int degree, int n_samples, const float* warp, float* origins, float* directions, float* radii,
                          float* rgb, uint16_t* encoded, float* sdist, float* tdist) {
    int width = oracle_direction_block_width(degree);
    for (int r = 0; r < n_rays; r++) {
        int64_t pixel = (int64_t)uniform_int((uint64_t)seed, 0, (uint64_t)r, (uint64_t)n_pixels);
        int view = 0;
        /* the last view whose first pixel is <= pixel (view_offsets ascending; binary search as in the reference) */
        int lo = 0, hi = n_views;
        while (hi - lo > 1) {
            int mid = (lo + hi) / 2;
            if (view_offsets[mid] <= pixel) lo = mid;
            else hi = mid;
        }
        view = lo;
        int camera = view_cameras[view];
        const float* m = c2w + 12 * view;
        float* d = directions + 3 * (int64_t)r;
        camera_ray(m, local + 3 * (camera_offsets[camera] + pixel - view_offsets[view]), d);
        origins[3 * r] = m[3];
        origins[3 * r + 1] = m[7];
        origins[3 * r + 2] = m[11];
        radii[r] = camera_radii[camera];
        for (int c = 0; c < 3; c++) rgb[3 * r + c] = (float)pool_rgb[3 * pixel + c] / 255.0f;
        new_ray(d, uniform((uint64_t)seed, 2, (uint64_t)r), degree, n_samples, (const warp_t*)warp, encoded + (int64_t)r * width,
                sdist + (int64_t)r * (n_samples + 1), tdist + (int64_t)r * (n_samples + 1));
    }
}

/* sample_uniforms (sampling_api.cu:168-172) */
void oracle_sample_uniforms(int64_t seed, int64_t stream, int64_t n, float* values) {
    for (int64_t i = 0; i < n; i++) values[i] = uniform((uint64_t)seed, (uint64_t)stream, (uint64_t)i);
}

/* composite_and_resample (sampling_api.cu:174-196 with composite, ray_ops.cuh:91-99) */
void oracle_composite_and_resample(const float* raw, const float* sdist, const float* tdist, const float* directions, int n_rays, int n, float anneal,
                                   int n_out, int64_t seed, int next_level, const float* warp, float* weights, float* sdist_next, float* tdist_next) {
    for (int r = 0; r < n_rays; r++) {
        const float* t = tdist + (int64_t)r * (n + 1);
        float* w = weights + (int64_t)r * n;
        float scale = norm3(directions + 3 * (int64_t)r), depth = 0.0f;
        for (int i = 0; i < n; i++) {
            float density = expf(fminf(raw[(int64_t)r * n + i] - 1.0f, 88.72283f));
            float x = density * (t[i + 1] - t[i]) * scale;
            w[i] = -expm1f(-x) * expf(-depth);
            depth += x;
        }
        float jitter = seed >= 0 ? uniform((uint64_t)seed, (uint64_t)(2 + next_level), (uint64_t)r) : -1.0f;
        float* s = sdist_next + (int64_t)r * (n_out + 1);
        resample(sdist + (int64_t)r * (n + 1), w, n, anneal, n_out, jitter, s);
        for (int i = 0; i <= n_out; i++) tdist_next[(int64_t)r * (n_out + 1) + i] = normalized_to_metric(s[i], (const warp_t*)warp);
    }
}

/* ------------------------------------------------------------------------------------------------------------------
 * Adam step of one buffer (optimizer_api.cu:43-53 per element, :80-93 the fp16 clamp): params / grads / moments of
 * numel floats; grad_half: grads are fp16 bits; level offsets (n_offsets entries, 0: none) regularize each level with
 * reg_weight / size and add that level's sum of squared updated parameters (double) to level_sums[first_level + i].
 * Gradients are zeroed. Returns nothing; the caller forms magnitudes and the regularizer from level_sums. */
static float half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31, exponent = (h >> 10) & 0x1f, mantissa = h & 0x3ff, bits;
    if (exponent == 0) {
        float value = ldexpf((float)mantissa, -24);
        return sign ? -value : value;
    }
    if (exponent == 31) bits = sign | 0x7f800000u | (mantissa << 13);
    else bits = sign | ((exponent + 112) << 23) | (mantissa << 13);
    float value;
    memcpy(&value, &bits, sizeof(value));
    return value;
}

void oracle_adam_buffer(float* params, void* grads, int grad_half, float* exp_avg, float* exp_avg_sq, int64_t numel, double grad_scale,
                        const int64_t* offsets, int n_offsets, double reg_weight, double beta1_d, double beta2_d, double eps_d, int64_t step, double lr_d,
                        double* level_sums) {
    float beta1 = (float)beta1_d, beta2 = (float)beta2_d, eps = (float)eps_d, lr = (float)lr_d, inv = (float)(1.0 / grad_scale);
    float bc1 = (float)(1.0 - pow((double)beta1, (double)step)), bc2 = (float)(1.0 - pow((double)beta2, (double)step));
    int level = 0;
    for (int64_t i = 0; i < numel; i++) {
        while (n_offsets > 0 && level + 1 < n_offsets - 1 && i >= offsets[level + 1]) level++;
        float reg = n_offsets > 0 ? (float)(reg_weight / (double)(offsets[level + 1] - offsets[level])) : 0.0f;
        float g;
        if (grad_half) {
            g = half_to_float(((uint16_t*)grads)[i]);
            g = fminf(fmaxf(g, -65504.0f), 65504.0f);
        } else {
            g = ((float*)grads)[i];
        }
        float p = params[i];
        g = g * inv + reg * p;
        g = isnan(g) ? 0.0f : fminf(fmaxf(g, -FLT_MAX), FLT_MAX);
        float m = beta1 * exp_avg[i] + (1.0f - beta1) * g;
        float v = beta2 * exp_avg_sq[i] + (1.0f - beta2) * g * g;
        p -= lr * (m / bc1) / (sqrtf(v / bc2) + eps);
        params[i] = p;
        exp_avg[i] = m;
        exp_avg_sq[i] = v;
        if (grad_half) ((uint16_t*)grads)[i] = 0;
        else ((float*)grads)[i] = 0.0f;
        if (n_offsets > 0) level_sums[level] += (double)p * (double)p;
    }
}

/* ------------------------------------------------------------------------------------------------------------------
 * The final level (sampling_api.cu:203-424 with ray_ops.cuh:20-24,91-166): training losses and the gradients of all
 * levels' raw outputs, and the inference compositing. bf16 values are their 16-bit patterns. */
#define NERF_OUTPUTS 8
#define RGB_PADDING 0.001f
#define MAX_PROPOSAL_LEVELS 4

static float from_bf16(uint16_t bits) {
    uint32_t word = (uint32_t)bits << 16;
    float value;
    memcpy(&value, &word, sizeof(value));
    return value;
}

static float ladder(float x, float p, float premult) { /* ray_ops.cuh:20-24 */
    float xp = fabsf(x * premult);
    float y = fabsf(p - 1.0f) / p * (powf(xp / fabsf(p - 1.0f) + 1.0f, p) - 1.0f);
    return copysignf(y, x);
}

static void alpha_composite(const float* density, const float* t, int n, float norm, float* w, float* x) { /* ray_ops.cuh:91-99 */
    float depth = 0.0f;
    for (int i = 0; i < n; i++) {
        float xi = density[i] * (t[i + 1] - t[i]) * norm;
        w[i] = -expm1f(-xi) * expf(-depth);
        depth += xi;
        x[i] = xi;
    }
}

static void alpha_composite_backward(float* grad, const float* x, const float* w, int n) { /* ray_ops.cuh:102-117 */
    float transmittance[MAX_INTERVALS], depth = 0.0f, suffix = 0.0f;
    for (int i = 0; i < n; i++) {
        depth += x[i];
        transmittance[i] = expf(-depth);
    }
    for (int i = n - 1; i >= 0; i--) {
        float g = grad[i];
        grad[i] = g * transmittance[i] - suffix;
        suffix += g * w[i];
    }
}

static float up(float x) { return fabsf(x) < FLT_MIN ? FLT_MIN : nextafterf(x, INFINITY); }
static float down(float x) { return fabsf(x) < FLT_MIN ? -FLT_MIN : nextafterf(x, -INFINITY); }

/* the histogram (t, w) of n bins blurred by a box of half width h, resampled into the nq - 1 bins of tq
 * (ray_ops.cuh:121-166) */
static void blur_resample(const float* tq, int nq, const float* t, const float* w, int n, float h, float* out) {
    float lo[MAX_INTERVALS + 1], hi[MAX_INTERVALS + 1], dslope[MAX_INTERVALS + 1];
    float previous_pdf = 0.0f;
    for (int i = 0; i <= n; i++) {
        float dt = i < n ? t[i + 1] - t[i] : 0.0f;
        float pdf = (i < n && dt >= FLT_MIN) ? w[i] / dt : 0.0f;
        lo[i] = t[i] - h;
        hi[i] = fmaxf(up(t[i]), t[i] + h);
        dslope[i] = (pdf - previous_pdf) / (hi[i] - lo[i]);
        previous_pdf = pdf;
    }
    float knots[2 * (MAX_INTERVALS + 1)], values[2 * (MAX_INTERVALS + 1)];
    int n_knots = 2 * (n + 1), a = 0, b = 0;
    float slope = 0.0f;
    for (int k = 0; k < n_knots; k++) {
        int take_lo = b > n || (a <= n && lo[a] <= hi[b]);
        float knot = take_lo ? lo[a] : hi[b];
        values[k] = (k == 0 || k == n_knots - 1) ? 0.0f : values[k - 1] + (knot - knots[k - 1]) * slope;
        knots[k] = knot;
        if (k < n_knots - 2) slope += take_lo ? dslope[a] : -dslope[b];
        if (take_lo) a++;
        else b++;
    }
    float first = knots[0], last = down(knots[n_knots - 1]), area = 0.0f, previous = 0.0f;
    int k = 0;
    for (int j = 0; j < nq; j++) {
        float q = fminf(fmaxf(tq[j], first), last);
        while (k + 2 < n_knots && knots[k + 1] <= q) {
            area += 0.5f * (knots[k + 1] - knots[k]) * (values[k] + values[k + 1]);
            k++;
        }
        float c = (values[k + 1] - values[k]) / fmaxf(FLT_EPSILON * FLT_EPSILON, 2.0f * (knots[k + 1] - knots[k]));
        float td = q - knots[k];
        float value = (c * td + values[k]) * td + area;
        if (j > 0) out[j - 1] = fmaxf(value - previous, 0.0f);
        previous = value;
    }
}

/* densities, rgb sigmoids, optical depths and weights of one ray of the final level (sampling_api.cu:203-220) */
static void final_level(const uint16_t* outputs, const float* t, int n, float norm, float* density, float* x, float* w, float (*sig)[3]) {
    for (int i = 0; i < n; i++) {
        const uint16_t* raw = outputs + NERF_OUTPUTS * i;
        float r[4] = {from_bf16(raw[0]), from_bf16(raw[1]), from_bf16(raw[2]), from_bf16(raw[3])};
        int valid = isfinite(r[0]) && isfinite(r[1]) && isfinite(r[2]) && isfinite(r[3]);
        density[i] = valid ? expf(fminf(r[0] - 1.0f, 88.72283f)) : 0.0f;
        for (int c = 0; c < 3; c++) sig[i][c] = valid ? 1.0f / (1.0f + expf(-r[c + 1])) : 0.5f;
    }
    alpha_composite(density, t, n, norm, w, x);
}

static float padded(float s) { return s * (1.0f + 2.0f * RGB_PADDING) - RGB_PADDING; }

/* the weights' gradients -> the raw densities (sampling_api.cu:223-229) */
static void weights_to_raw(float* grad, const float* x, const float* w, const float* density, const float* raw, const float* t, int n, float norm) {
    alpha_composite_backward(grad, x, w, n);
    for (int i = 0; i < n; i++) grad[i] = raw[i] - 1.0f > 88.72283f ? 0.0f : grad[i] * (t[i + 1] - t[i]) * norm * density[i];
}

/* train_final (sampling_api.cu:231-376); loss_sums (double [4]) += this batch's sums */
void oracle_train_final(const uint16_t* outputs, const float* sdist, const float* tdist, int n_rays, int n, int n_levels, const int* n_p,
                        const float* const* raw_p, const float* const* sdist_p, const float* const* tdist_p, const float* const* weights_p,
                        float* const* grad_p_out, const float* interlevel_weights, const float* interlevel_blurs, const float* directions,
                        uint64_t seed, const float* rgb_target, float padding, float distortion_weight, float distortion_power,
                        float distortion_premult, uint16_t* outputs_grad, double* loss_sums) {
    float inv_n_rays = 1.0f / (float)n_rays;
    for (int r = 0; r < n_rays; r++) {
        const float* t = tdist + (int64_t)r * (n + 1);
        const float* s = sdist + (int64_t)r * (n + 1);
        float norm = norm3(directions + 3 * (int64_t)r);
        float density[MAX_INTERVALS], x[MAX_INTERVALS], w[MAX_INTERVALS], grad_w[MAX_INTERVALS], sig[MAX_INTERVALS][3];
        final_level(outputs + (int64_t)NERF_OUTPUTS * r * n, t, n, norm, density, x, w, sig);
        float rgb[3] = {0.0f, 0.0f, 0.0f}, acc = 0.0f;
        for (int i = 0; i < n; i++) {
            for (int c = 0; c < 3; c++) rgb[c] += w[i] * padded(sig[i][c]);
            acc += w[i];
        }
        float bg[3], grad_rgb[3];
        for (int c = 0; c < 3; c++) bg[c] = uniform(seed, 1, 3 * (uint64_t)r + (uint64_t)c);
        float background_weight = fmaxf(1.0f - acc, 0.0f);
        for (int c = 0; c < 3; c++) {
            float residual = rgb[c] + background_weight * bg[c] - rgb_target[3 * (int64_t)r + c];
            float q = sqrtf(residual * residual + padding * padding);
            loss_sums[0] += q * inv_n_rays / 3.0f;
            loss_sums[1] += residual * residual * inv_n_rays / 3.0f;
            grad_rgb[c] = residual / q * inv_n_rays / 3.0f;
        }
        float grad_background = 1.0f - acc >= 0.0f ? grad_rgb[0] * bg[0] + grad_rgb[1] * bg[1] + grad_rgb[2] * bg[2] : 0.0f;
        for (int i = 0; i < n; i++) {
            grad_w[i] = grad_rgb[0] * padded(sig[i][0]) + grad_rgb[1] * padded(sig[i][1]) + grad_rgb[2] * padded(sig[i][2]) - grad_background;
        }
        /* distortion loss on the curved distances */
        float u[MAX_INTERVALS], ds[MAX_INTERVALS], prev = ladder(t[0], distortion_power, distortion_premult), w_total = 0.0f, wu_total = 0.0f;
        for (int i = 0; i < n; i++) {
            float next = ladder(t[i + 1], distortion_power, distortion_premult);
            u[i] = 0.5f * (prev + next);
            ds[i] = next - prev;
            prev = next;
            w_total += w[i];
            wu_total += w[i] * u[i];
        }
        float scale = distortion_weight * inv_n_rays, w_before = 0.0f, wu_before = 0.0f, loss = 0.0f;
        for (int i = 0; i < n; i++) {
            float w_after = w_total - w_before - w[i], wu_after = wu_total - wu_before - w[i] * u[i];
            float inter = u[i] * w_before - wu_before + wu_after - u[i] * w_after;
            loss += w[i] * (u[i] * w_before - wu_before) * 2.0f + w[i] * w[i] * ds[i] / 3.0f;
            grad_w[i] += scale * (2.0f * inter + 2.0f / 3.0f * w[i] * ds[i]);
            w_before += w[i];
            wu_before += w[i] * u[i];
        }
        loss_sums[3] += scale * loss;
        /* gradients of the raw outputs */
        float raw[MAX_INTERVALS];
        for (int i = 0; i < n; i++) raw[i] = from_bf16(outputs[(int64_t)NERF_OUTPUTS * ((int64_t)r * n + i)]);
        weights_to_raw(grad_w, x, w, density, raw, t, n, norm);
        for (int i = 0; i < n; i++) {
            uint16_t* g = outputs_grad + (int64_t)NERF_OUTPUTS * ((int64_t)r * n + i);
            float color_scale = w[i] * (1.0f + 2.0f * RGB_PADDING);
            g[0] = to_bf16(grad_w[i]);
            for (int c = 0; c < 3; c++) g[c + 1] = to_bf16(color_scale * grad_rgb[c] * sig[i][c] * (1.0f - sig[i][c]));
            for (int c = 4; c < NERF_OUTPUTS; c++) g[c] = to_bf16(0.0f);
        }
        /* interlevel losses of the proposal levels */
        for (int level = 0; level < n_levels; level++) {
            int m = n_p[level];
            const float* sp = sdist_p[level] + (int64_t)r * (m + 1);
            const float* tp = tdist_p[level] + (int64_t)r * (m + 1);
            const float* wp = weights_p[level] + (int64_t)r * m;
            float gp[MAX_INTERVALS], rawp[MAX_INTERVALS], densityp[MAX_INTERVALS], xp[MAX_INTERVALS];
            blur_resample(sp, m + 1, s, w, n, interlevel_blurs[level], gp);
            float lscale = interlevel_weights[level] * inv_n_rays / (float)(m > 1 ? m : 1);
            for (int i = 0; i < m; i++) {
                float resid = fmaxf(gp[i] - wp[i], 0.0f), denominator = wp[i] + FLT_EPSILON;
                loss_sums[2] += lscale * resid * resid / denominator;
                gp[i] = lscale * (-2.0f * resid / denominator - resid * resid / (denominator * denominator));
                rawp[i] = raw_p[level][(int64_t)r * m + i];
                densityp[i] = expf(fminf(rawp[i] - 1.0f, 88.72283f));
                xp[i] = densityp[i] * (tp[i + 1] - tp[i]) * norm;
            }
            weights_to_raw(gp, xp, wp, densityp, rawp, tp, m, norm);
            for (int i = 0; i < m; i++) grad_p_out[level][(int64_t)r * m + i] = gp[i];
        }
    }
}

/* composite_final (sampling_api.cu:379-424); alpha / depth may be NULL */
void oracle_composite_final(const uint16_t* outputs, const float* tdist, const float* directions, const float* background, const int64_t* pixels,
                            int n_rays, int n, float* rgb, float* alpha, float* depth, int use_median_depth) {
    for (int r = 0; r < n_rays; r++) {
        const float* t = tdist + (int64_t)r * (n + 1);
        float density[MAX_INTERVALS], x[MAX_INTERVALS], w[MAX_INTERVALS], sig[MAX_INTERVALS][3];
        final_level(outputs + (int64_t)NERF_OUTPUTS * r * n, t, n, norm3(directions + 3 * (int64_t)r), density, x, w, sig);
        float color[3] = {0.0f, 0.0f, 0.0f}, acc = 0.0f;
        for (int i = 0; i < n; i++) {
            for (int c = 0; c < 3; c++) color[c] += w[i] * padded(sig[i][c]);
            acc += w[i];
        }
        float background_weight = fmaxf(1.0f - acc, 0.0f);
        int64_t p = pixels[r];
        for (int c = 0; c < 3; c++) rgb[3 * p + c] = color[c] + background_weight * background[c];
        if (alpha) alpha[p] = acc;
        if (!depth) continue;
        if (use_median_depth) {
            float target = 0.5f * acc, cw = 0.0f, median = t[n];
            for (int i = 0; i < n; i++) {
                cw += w[i];
                if (w[i] > 0.0f && cw >= target) {
                    median = t[i];
                    break;
                }
            }
            depth[p] = median;
        } else {
            float weighted = 0.0f;
            for (int i = 0; i < n; i++) weighted += w[i] * logf(0.5f * (t[i] + t[i + 1]));
            depth[p] = fminf(fmaxf(expf(weighted / fmaxf(acc, FLT_EPSILON)), t[0]), t[n]);
        }
    }
}

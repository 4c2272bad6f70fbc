// fz_nerf_mlp_backward.cu -- the NeRF MLP backward on the tcgen05 tensor cores (NerfMlp::backward, nerf_mlp.cu:565-620),
// as two kernels:
//
// fz_nerf_mlp_backward_data_kernel: the data-gradient chain of one 128-sample tile after another (persistent, one CTA
// per SM), the transposed packed weights as B operands (zipnerf_b200.nerf_mlp.pack_transposed):
//   B0  g_v2 = (g_out @ w_rgb) * [v2 > 0]              K = 16 (the 8 outputs, zero padded)
//   B1  g_v1 = (g_v2 @ w_2) * [v1 > 0]
//   B2  g_v0 = (g_v1 @ w_1) * [v0 > 0]
//   B3  g_in = g_v0 @ w_combined + g_out @ w_skip,  g_h = g_in[:, 0:64] * [h > 0]
//   B4  g_features = g_h @ w_density
// The masked gradients stay on the SM as the next layer's A operand and are written to global memory for the weight
// gradients; the masks come from the forward's activations (v0, v1, v2 and h). Warp roles, weight ring, tensor-memory
// regions, chunk barriers and bounded waits as in the forward kernel (fz_nerf_mlp.cu).
//
// fz_nerf_mlp_backward_weight_kernel: one weight gradient dW = G^T V summed over all samples (split over the CTAs by
// 64-sample K-tiles, each CTA accumulating its share in tensor memory and adding it to dW with fp32 atomics at the end),
// G and V read from global memory into shared memory by cp.async and used as MN-major operands (the samples are the
// K dimension of this GEMM); the column sums of G (a bias gradient) on the CUDA cores from the same tiles.
#include "zf_mlp.h"
#include "fz_status.h"
#include "fz_tcgen05.cuh"

namespace zf::nerf_mlp {

namespace bwd {

constexpr int kView = 256;
constexpr int kInputs = 96;
constexpr int kDensity = 64;
constexpr int kFeatures = 56;
constexpr int kOutputs = 8;           // output gradient columns (raw density, 3 rgb logits, 4 zeros)
constexpr int kGoutK = 16;           // the output gradients padded to one MMA K step
constexpr int kSlice = 64;
constexpr int kChunks = kView / kSlice;

constexpr int kMmaWarp = 0;
constexpr int kProducerWarp = 1;
constexpr int kFirstEpilogueWarp = 2;
constexpr int kEpilogueWarps = 8;    // group g (warps 2 + 4g .. 5 + 4g) takes the 64-column chunks g and g + 2
constexpr int kEpilogueThreads = 32 * kEpilogueWarps;
constexpr int kThreads = 32 * (kFirstEpilogueWarp + kEpilogueWarps);
constexpr uint32_t kTmemColumns = 512;
constexpr uint32_t kRegionColumns = 256;

// weight stages per tile: rgb_t, view_2_t x 4, view_1_t x 4, combined_t x 4, skip_t, density_t
constexpr int kStagesPerTile = 15;
constexpr int kRingSlots = 4;
constexpr int kStageBytes = kView * kSlice * 2;     // 32 KB

constexpr int kActBytes = kTileRows * kView * 2;    // 64 KB: g_v2, then g_v1, then g_v0
constexpr int kGoutBytes = kTileRows * kGoutK * 2;  // 4 KB
constexpr int kHiddenBytes = kTileRows * kDensity * 2;  // 16 KB: g_h
constexpr int kActOffset = 0;
constexpr int kGoutOffset = kActOffset + kActBytes;
constexpr int kHiddenOffset = kGoutOffset + kGoutBytes;
constexpr int kRingOffset = kHiddenOffset + kHiddenBytes;
constexpr int kBarOffset = kRingOffset + kRingSlots * kStageBytes;
// full[4], empty[4], acc_full, in_ready, h_ready, chunk[4], drain
constexpr int kNumBarriers = 2 * kRingSlots + 3 + kChunks + 1;
constexpr int kMiscOffset = kBarOffset + kNumBarriers * 8;
constexpr int kSmemBytes = kMiscOffset + 16;
static_assert(kSmemBytes <= 227 * 1024, "one CTA per SM");

// transposed packed weights [inputs x outputs] in K-slices (canonical K-major order per slice)
struct PackedMlpT {
    const uint16_t* rgb_t;       // [256, 16]
    const uint16_t* view_2_t;    // [256, 256], 4 slices of 64
    const uint16_t* view_1_t;    // [256, 256], 4 slices of 64
    const uint16_t* combined_t;  // [96, 256], 4 slices of 64
    const uint16_t* skip_t;      // [96, 16]
    const uint16_t* density_t;   // [64, 64]
};

struct DataArgs {
    const uint16_t* grad_outputs;   // [n, 8]
    const uint16_t* inputs;         // [n, inputs_stride]: h in columns 0-63
    int64_t inputs_stride;
    const uint16_t* activations;    // [3, n, 256]: v0, v1, v2
    uint16_t* grad_activations;     // [3, n, 256] out: g_v0, g_v1, g_v2
    uint16_t* grad_hidden;          // [n, 64] out: g_h
    uint16_t* grad_features;        // [n, features_stride] out: columns 0-55
    int64_t features_stride;
    int64_t n;
};

struct Stage {
    const void* src;
    uint32_t bytes;
};

__device__ __forceinline__ Stage weight_stage(const PackedMlpT& w, const int s) {
    if (s == 0) return {w.rgb_t, kView * kGoutK * 2};
    if (s < 5) return {w.view_2_t + (s - 1) * kView * kSlice, kStageBytes};
    if (s < 9) return {w.view_1_t + (s - 5) * kView * kSlice, kStageBytes};
    if (s < 13) return {w.combined_t + (s - 9) * kInputs * kSlice, kInputs * kSlice * 2};
    if (s == 13) return {w.skip_t, kInputs * kGoutK * 2};
    return {w.density_t, kDensity * kDensity * 2};
}

// N (32 or 64) accumulator columns of this thread's row, times the ReLU mask of mask_row (bf16 values > 0; none: no
// mask), rounded to bf16, into row `row` of a K-major operand at column k_first (when dst is given) and into global
// memory at out_row + k_first (its first out_cols columns, when out_row is given)
template <int N>
__device__ __forceinline__ void masked_columns(const uint32_t taddr, const uint16_t* mask_row, uint8_t* dst, const int row, const int k_total,
                                               const int k_first, uint16_t* out_row, const int out_cols) {
    uint32_t r[N];
    #pragma unroll
    for (int c = 0; c < N; c += 32) issue_load<32>(taddr + c, r + c);
    uint4 m[N / 8];
    #pragma unroll
    for (int j = 0; j < N / 8; j++) m[j] = mask_row != nullptr ? __ldg(reinterpret_cast<const uint4*>(mask_row + k_first) + j) : make_uint4(0, 0, 0, 0);
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    #pragma unroll
    for (int j = 0; j < N / 8; j++) {
        const uint32_t mw[4] = {m[j].x, m[j].y, m[j].z, m[j].w};
        uint32_t words[4];
        #pragma unroll
        for (int q = 0; q < 4; q++) {
            float lo = __uint_as_float(r[8 * j + 2 * q]), hi = __uint_as_float(r[8 * j + 2 * q + 1]);
            if (mask_row != nullptr) {
                if (!(__uint_as_float(mw[q] << 16) > 0.0f)) lo = 0.0f;
                if (!(__uint_as_float(mw[q] & 0xFFFF0000u) > 0.0f)) hi = 0.0f;
            }
            words[q] = pack_bf16x2(lo, hi);
        }
        const uint4 out = make_uint4(words[0], words[1], words[2], words[3]);
        if (dst != nullptr) *reinterpret_cast<uint4*>(dst + canonical_offset(row, k_first + 8 * j, k_total)) = out;
        if (out_row != nullptr && 8 * j < out_cols) *reinterpret_cast<uint4*>(out_row + k_first + 8 * j) = out;
    }
}

__global__ void __launch_bounds__(kThreads, 1) fz_nerf_mlp_backward_data_kernel(const __grid_constant__ PackedMlpT w, const __grid_constant__ DataArgs a,
                                                                             int* status) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* act = smem + kActOffset;
    uint8_t* gout = smem + kGoutOffset;
    uint8_t* gh = smem + kHiddenOffset;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOffset);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kMiscOffset);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + kMiscOffset + 4);
    const uint32_t bar0 = smem_address(bars);
    auto full_bar = [&](const uint32_t slot) { return bar0 + 8u * slot; };
    auto empty_bar = [&](const uint32_t slot) { return bar0 + 8u * (kRingSlots + slot); };
    const uint32_t acc_bar = bar0 + 8u * (2 * kRingSlots);      // a layer's MMAs are done (tcgen05.commit)
    const uint32_t in_bar = acc_bar + 8u;                      // the tile's output gradients are in shared memory
    const uint32_t h_bar = in_bar + 8u;                        // g_h is in shared memory
    auto chunk_bar = [&](const int c) { return h_bar + 8u * (1 + c); };  // 64 columns of the next A operand are written
    const uint32_t drain_bar = h_bar + 8u * (1 + kChunks);
    const uint32_t ring = smem_address(smem + kRingOffset);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int64_t n = a.n;
    const int64_t n_tiles = (n + kTileRows - 1) / kTileRows;

    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_address(tmem_slot)), "r"(kTmemColumns));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (threadIdx.x == 32 * kProducerWarp) {
        for (int s = 0; s < kRingSlots; s++) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(full_bar(s)), "r"(1));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(empty_bar(s)), "r"(1));
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(acc_bar), "r"(1));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(in_bar), "r"(kEpilogueThreads));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(h_bar), "r"(kEpilogueThreads));
        for (int c = 0; c < kChunks; c++) asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(chunk_bar(c)), "r"(kEpilogueThreads / 2));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(drain_bar), "r"(1));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *abort = 0;
    }
    // columns 8-15 of the output-gradient tile stay zero (the K padding of B0 and of the skip term)
    for (int r = threadIdx.x; r < kTileRows; r += kThreads) *reinterpret_cast<uint4*>(gout + canonical_offset(r, 8, kGoutK)) = make_uint4(0, 0, 0, 0);
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;
    uint32_t stages_issued = 0;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            for (int64_t tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                for (int s = 0; s < kStagesPerTile; s++) {
                    const uint32_t slot = stages_issued % kRingSlots;
                    if (stages_issued >= kRingSlots && !wait_phase(empty_bar(slot), (stages_issued / kRingSlots - 1) & 1u, abort)) {
                        ok = false;
                        break;
                    }
                    const Stage st = weight_stage(w, s);
                    expect_bytes(full_bar(slot), st.bytes);
                    bulk_copy(ring + slot * kStageBytes, st.src, st.bytes, full_bar(slot));
                    stages_issued++;
                }
            }
        }
    }
    else if (warp == kMmaWarp) {
        if (lane == 0) {
            uint32_t stage = 0, layer = 0, inputs_seen = 0, hidden_seen = 0;
            uint32_t chunks_seen[kChunks] = {0, 0, 0, 0};
            auto take = [&](uint32_t& address) -> bool {
                const uint32_t slot = stage % kRingSlots;
                if (!wait_phase(full_bar(slot), (stage / kRingSlots) & 1u, abort)) return false;
                address = ring + slot * kStageBytes;
                return true;
            };
            auto release = [&]() {
                commit(empty_bar(stage % kRingSlots));
                stage++;
            };
            auto chunk_ready = [&](const int c) -> bool {
                const bool done = wait_phase(chunk_bar(c), chunks_seen[c] & 1u, abort);
                chunks_seen[c]++;
                fence_after_sync();
                return done;
            };
            const uint32_t a_act = smem_address(act), a_gout = smem_address(gout), a_gh = smem_address(gh);
            for (int64_t tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                uint32_t b = 0;
                // B0: g_out @ w_rgb (N = 256, K = 16)
                uint32_t d = tmem + (layer & 1u) * kRegionColumns;
                ok = wait_phase(in_bar, inputs_seen & 1u, abort);
                inputs_seen++;
                fence_after_sync();
                if (!(ok = ok && take(b))) break;
                mma_chain(d, a_gout, kGoutK, b, kGoutK, kView, kGoutK, false);
                release();
                commit(acc_bar);
                layer++;
                // B1, B2: K-slice j reads chunk j of the previous masked gradient
                for (int k = 1; k <= 2 && ok; k++) {
                    d = tmem + (layer & 1u) * kRegionColumns;
                    for (int j = 0; j < kChunks; j++) {
                        if (!(ok = chunk_ready(j) && take(b))) break;
                        mma_chain(d, a_act + j * (kSlice / 8) * 128, kView, b, kSlice, kView, kSlice, j > 0);
                        release();
                    }
                    if (!ok) break;
                    commit(acc_bar);
                    layer++;
                }
                if (!ok) break;
                // B3: g_v0 @ w_combined + g_out @ w_skip (N = 96)
                d = tmem + (layer & 1u) * kRegionColumns;
                for (int j = 0; j < kChunks; j++) {
                    if (!(ok = chunk_ready(j) && take(b))) break;
                    mma_chain(d, a_act + j * (kSlice / 8) * 128, kView, b, kSlice, kInputs, kSlice, j > 0);
                    release();
                }
                if (!ok) break;
                if (!(ok = take(b))) break;
                mma_chain(d, a_gout, kGoutK, b, kGoutK, kInputs, kGoutK, true);
                release();
                commit(acc_bar);
                layer++;
                // B4: g_h @ w_density (N = 64)
                d = tmem + (layer & 1u) * kRegionColumns;
                ok = wait_phase(h_bar, hidden_seen & 1u, abort);
                hidden_seen++;
                fence_after_sync();
                if (!(ok = ok && take(b))) break;
                mma_chain(d, a_gh, kDensity, b, kDensity, kDensity, kDensity, false);
                release();
                commit(acc_bar);
                layer++;
            }
        }
    }
    else {
        const int e = warp - kFirstEpilogueWarp;
        const int g = e / 4;
        const int quadrant = warp % 4;
        const int row = 32 * quadrant + lane;
        const int tid = threadIdx.x - 32 * kFirstEpilogueWarp;
        const uint32_t lanes = tmem + (static_cast<uint32_t>(32 * quadrant) << 16);
        uint32_t layer = 0;
        auto accumulator_ready = [&]() -> bool {
            const bool done = __all_sync(0xFFFFFFFFu, wait_phase(acc_bar, layer & 1u, abort));
            fence_after_sync();
            return done;
        };
        auto publish = [&](const uint32_t bar) {
            fence_async_shared();
            fence_before_sync();
            arrive(bar);
        };
        // one row of the output gradients per thread of the first half (16 bytes: the 8 outputs)
        static_assert(kOutputs * 2 == sizeof(uint4), "one 16-byte word per output-gradient row");
        auto fetch_gout = [&](const int64_t tile) -> uint4 {
            const int64_t s = tile * kTileRows + tid;
            return tid < kTileRows && s < n ? __ldg(reinterpret_cast<const uint4*>(a.grad_outputs) + s) : make_uint4(0, 0, 0, 0);
        };
        auto store_gout = [&](const uint4 v) {
            if (tid < kTileRows) *reinterpret_cast<uint4*>(gout + canonical_offset(tid, 0, kGoutK)) = v;
        };
        int64_t tile = blockIdx.x;
        uint4 next = make_uint4(0, 0, 0, 0);
        if (tile < n_tiles) {
            store_gout(fetch_gout(tile));
            publish(in_bar);
        }
        for (; tile < n_tiles && ok; tile += gridDim.x) {
            const int64_t sample = tile * kTileRows + row;
            const bool valid = sample < n;
            const bool more = tile + gridDim.x < n_tiles;
            // E0-E2: g_v2, g_v1, g_v0 masked by v2, v1, v0: chunks g and g + 2 -> act and global memory
            for (int k = 0; k < 3 && ok; k++) {
                if (!(ok = accumulator_ready())) break;
                const int index = 2 - k;  // v2, v1, v0
                const uint16_t* mask = valid ? a.activations + (static_cast<int64_t>(index) * n + sample) * kView : nullptr;
                uint16_t* out = valid ? a.grad_activations + (static_cast<int64_t>(index) * n + sample) * kView : nullptr;
                const uint32_t region = lanes + (layer & 1u) * kRegionColumns;
                for (int j = g; j < kChunks; j += 2) {
                    masked_columns<kSlice>(region + kSlice * j, mask, act, row, kView, kSlice * j, out, kSlice);
                    publish(chunk_bar(j));
                }
                layer++;
                if (k == 0 && more) next = fetch_gout(tile + gridDim.x);
            }
            if (!ok) break;
            // E3: g_h = g_in[:, 0:64] masked by h: columns [32 g, 32 g + 32) -> the g_h tile and global memory
            if (!(ok = accumulator_ready())) break;
            masked_columns<32>(lanes + (layer & 1u) * kRegionColumns + 32 * g, valid ? a.inputs + sample * a.inputs_stride : nullptr, gh, row, kDensity,
                               32 * g, valid ? a.grad_hidden + sample * kDensity : nullptr, 32);
            publish(h_bar);
            layer++;
            // E4: g_features, columns [32 g, 32 g + 32) below 56, then the next tile's output gradients
            if (!(ok = accumulator_ready())) break;
            masked_columns<32>(lanes + (layer & 1u) * kRegionColumns + 32 * g, nullptr, nullptr, row, 0, 32 * g,
                               valid ? a.grad_features + sample * a.features_stride : nullptr, kFeatures - 32 * g);
            layer++;
            if (more) {
                store_gout(next);
                publish(in_bar);
            }
        }
    }

    fence_before_sync();
    __syncthreads();
    if (threadIdx.x == 32 * kMmaWarp) {
        commit(drain_bar);
        drain_phase(drain_bar, 0);
    }
    if (threadIdx.x == 32 * kProducerWarp && *abort) {
        for (uint32_t i = stages_issued > kRingSlots ? stages_issued - kRingSlots : 0; i < stages_issued; i++) {
            drain_phase(full_bar(i % kRingSlots), (i / kRingSlots) & 1u);
        }
    }
    if (threadIdx.x == 0 && *abort) atomicExch(status, kWaitTimeout);
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (warp == kMmaWarp) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemColumns));
}

// ---------------------------------------------------------------------------------------------------------------------
// weight gradients: dW[m][k] += sum over samples s of G[s][m] V[s][k], bias[m] += sum over s of G[s][m]

constexpr int kWgradThreads = 256;
constexpr int kKTile = 64;           // samples per K-tile (4 MMA K steps)
constexpr int kWgradStages = 3;
constexpr int kWgradMaxM = 256;      // two M = 128 halves
constexpr int kWgradMaxN = 256;
constexpr int kWgradStageBytes = kKTile * (kWgradMaxM + kWgradMaxN) * 2;  // 64 KB
constexpr int kWgradBarOffset = kWgradStages * kWgradStageBytes;
constexpr int kWgradSmemBytes = kWgradBarOffset + 8 * (kWgradStages + 1) + 16;
static_assert(kWgradSmemBytes <= 227 * 1024, "one CTA per SM");

struct WeightArgs {
    const uint16_t* g;          // [n, g_stride]: the first m_cols columns are G
    int64_t g_stride;
    int m_cols;                 // <= 256
    const uint16_t* v;          // [n, v_stride]: the first k_cols columns are V
    int64_t v_stride;
    int k_cols;                 // <= 256
    int64_t n;
    float* dw;                  // dW[m][k] at dw[m * dw_m_stride + k * dw_k_stride] (+=)
    int64_t dw_m_stride;
    int64_t dw_k_stride;
    float* bias;                // bias[m] (+=), or null
};

// the 16-byte copies of one K-tile of G (m_pad columns) and V (k_pad columns) into a stage, canonical order with
// the samples as rows; columns and samples past the end are zero-filled
__device__ __forceinline__ void load_wgrad_tile(const WeightArgs& a, const int m_pad, const int k_pad, const int64_t first, const uint32_t stage_address,
                                                const int tid) {
    const int gm = m_pad / 8, vk = k_pad / 8;
    const int words = kKTile * (gm + vk);
    for (int q = tid; q < words; q += kWgradThreads) {
        const bool is_g = q < kKTile * gm;
        const int local = is_g ? q : q - kKTile * gm;
        const int per_row = is_g ? gm : vk;
        const int r = local / per_row, c = local % per_row;
        const int64_t s = first + r;
        const int cols = is_g ? a.m_cols : a.k_cols;
        const bool inside = s < a.n && 8 * c < cols;
        const uint16_t* src = (is_g ? a.g + (inside ? s : 0) * a.g_stride : a.v + (inside ? s : 0) * a.v_stride) + (inside ? 8 * c : 0);
        const uint32_t dst = stage_address + (is_g ? 0u : static_cast<uint32_t>(kKTile * m_pad * 2)) + canonical_offset(r, 8 * c, per_row * 8);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(inside ? 16 : 0) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// D[128 x n] (+)= A[128 x 16 k-steps] B[n x ...]^T with A and B MN-major: the stored rows are the K dimension (samples)
// and the 16 bytes of a core-matrix row run along M or N; MN-adjacent core matrices 128 bytes apart, K-adjacent ones
// (width / 8) * 128 bytes apart
__device__ __forceinline__ void mma_chain_mn(const uint32_t d_tmem, const uint32_t a_address, const int a_width, const uint32_t b_address,
                                             const int b_width, const int n, const int k, const bool accumulate) {
    const uint32_t idesc = instr_descriptor(kTileRows, n, true, true);
    const uint32_t a_k = static_cast<uint32_t>(a_width >> 3) * 128, b_k = static_cast<uint32_t>(b_width >> 3) * 128;
    for (int s = 0; s < k / kMmaK; s++) {
        // one K step of 16 samples covers two K-adjacent core matrices
        mma(d_tmem, smem_descriptor(a_address + 2 * s * a_k, a_k, 128), smem_descriptor(b_address + 2 * s * b_k, b_k, 128), idesc,
            (accumulate || s > 0) ? 1u : 0u);
    }
}

__global__ void __launch_bounds__(kWgradThreads, 1) fz_nerf_mlp_backward_weight_kernel(const __grid_constant__ WeightArgs a, int* status) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWgradBarOffset);  // mma_done[stages], drain
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kWgradBarOffset + 8 * (kWgradStages + 1));
    volatile int* abort = reinterpret_cast<volatile int*>(smem + kWgradBarOffset + 8 * (kWgradStages + 1) + 4);
    const uint32_t bar0 = smem_address(bars);
    const uint32_t base = smem_address(smem);
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int m_halves = a.m_cols > 128 ? 2 : 1;
    const int m_pad = 128 * m_halves;
    const int k_pad = (a.k_cols + 15) / 16 * 16;
    const int64_t n_tiles = (a.n + kKTile - 1) / kKTile;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_address(tmem_slot)), "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 32) {
        for (int s = 0; s <= kWgradStages; s++) asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar0 + 8u * s), "r"(1));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *abort = 0;
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    float column_sum = 0.0f;  // this thread's column of G (tid < m_cols), over this CTA's samples
    // prologue: the first stages in flight
    int64_t tile = blockIdx.x;
    for (int s = 0; s < kWgradStages - 1; s++) {
        if (tile + s * gridDim.x < n_tiles) load_wgrad_tile(a, m_pad, k_pad, (tile + s * gridDim.x) * kKTile, base + s * kWgradStageBytes, tid);
        else asm volatile("cp.async.commit_group;" ::: "memory");
    }
    uint32_t step = 0;
    bool ok = true;
    uint32_t mma_phase[kWgradStages] = {0, 0, 0};
    for (; tile < n_tiles; tile += gridDim.x, step++) {
        const uint32_t slot = step % kWgradStages;
        // the stage that the next load reuses must have been read by its MMAs (issued kWgradStages - 1 steps ago)
        const int64_t ahead = tile + (kWgradStages - 1) * static_cast<int64_t>(gridDim.x);
        const uint32_t ahead_slot = (step + kWgradStages - 1) % kWgradStages;
        if (step >= 1 && ahead < n_tiles) {
            const bool done = __syncthreads_and(wait_phase(bar0 + 8u * ahead_slot, mma_phase[ahead_slot] & 1u, abort));
            mma_phase[ahead_slot]++;
            if (!done) {
                ok = false;
                break;
            }
        }
        if (ahead < n_tiles) load_wgrad_tile(a, m_pad, k_pad, ahead * kKTile, base + ahead_slot * kWgradStageBytes, tid);
        else asm volatile("cp.async.commit_group;" ::: "memory");
        // this step's stage has landed (all but the newest kWgradStages - 1 groups are complete)
        asm volatile("cp.async.wait_group %0;" ::"n"(kWgradStages - 1) : "memory");
        fence_async_shared();
        __syncthreads();
        const uint32_t stage = base + slot * kWgradStageBytes;
        if (tid == 0) {
            fence_after_sync();
            const uint32_t b = stage + kKTile * m_pad * 2;
            for (int h = 0; h < m_halves; h++) {
                // M-half h of G: its 16 MN core-matrix columns start 16 * 128 bytes further along M
                mma_chain_mn(tmem + h * k_pad, stage + h * 16 * 128, m_pad, b, k_pad, k_pad, kKTile, step > 0);
            }
            commit(bar0 + 8u * slot);
        }
        // the bias gradient: this thread's column of the K-tile
        if (a.bias != nullptr && tid < a.m_cols) {
            const uint8_t* g_tile = smem + slot * kWgradStageBytes;
            #pragma unroll 8
            for (int r = 0; r < kKTile; r++) {
                const uint16_t bits = *reinterpret_cast<const uint16_t*>(g_tile + canonical_offset(r, tid, m_pad));
                column_sum += __uint_as_float(static_cast<uint32_t>(bits) << 16);
            }
        }
    }
    // every MMA of this CTA is done, then the accumulators go to dW with fp32 atomics (rows of M-half h: warps
    // 4h .. 4h + 3, tensor-memory lane quadrant warp % 4)
    fence_before_sync();
    __syncthreads();
    if (tid == 0) {
        commit(bar0 + 8u * kWgradStages);
        drain_phase(bar0 + 8u * kWgradStages, 0);
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (ok && step > 0) {
        const int h = warp / 4;
        const int m = 128 * h + 32 * (warp % 4) + lane;
        if (h < m_halves) {
            const uint32_t lanes = tmem + (static_cast<uint32_t>(32 * (warp % 4)) << 16) + h * k_pad;
            for (int c = 0; c < k_pad; c += 16) {
                uint32_t r[16];
                issue_load<16>(lanes + c, r);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (m < a.m_cols) {
                    #pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const float value = __uint_as_float(r[j]);
                        if (c + j < a.k_cols && value != 0.0f) atomicAdd(a.dw + m * a.dw_m_stride + (c + j) * a.dw_k_stride, value);
                    }
                }
            }
        }
        if (a.bias != nullptr && tid < a.m_cols && column_sum != 0.0f) atomicAdd(a.bias + tid, column_sum);
    }
    if (tid == 0 && (*abort || !ok)) atomicExch(status, kWaitTimeout);
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}

// launches of one backward: the data-gradient kernel, then the weight gradients of every packed weight
cudaError_t launch_backward(const PackedMlpT& w, const DataArgs& d, const zf_nerf_mlp_grads& grads, const uint16_t* features, int* status,
                            cudaStream_t stream) {
    int device = 0, n_sms = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, device);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(fz_nerf_mlp_backward_data_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(fz_nerf_mlp_backward_weight_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kWgradSmemBytes);
    if (e != cudaSuccess) return e;
    const int64_t n = d.n;
    const int64_t data_tiles = (n + kTileRows - 1) / kTileRows;
    fz_nerf_mlp_backward_data_kernel<<<static_cast<unsigned>(data_tiles < n_sms ? data_tiles : n_sms), kThreads, kSmemBytes, stream>>>(w, d, status);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int64_t k_tiles = (n + kKTile - 1) / kKTile;
    const unsigned grid = static_cast<unsigned>(k_tiles < n_sms ? k_tiles : n_sms);
    const uint16_t* g_v0 = d.grad_activations;
    const uint16_t* g_v1 = d.grad_activations + n * kView;
    const uint16_t* g_v2 = d.grad_activations + 2 * n * kView;
    const uint16_t* v0 = d.activations;
    const uint16_t* v1 = d.activations + n * kView;
    const uint16_t* v2 = d.activations + 2 * n * kView;
    const WeightArgs launches[] = {
        // view_2: g_v2^T v1 (+ bias), view_1: g_v1^T v0 (+ bias), combined: g_v0^T inputs (its bias in the bias lane)
        {g_v2, kView, kView, v1, kView, kView, n, grads.view_2, kView, 1, grads.view_2_bias},
        {g_v1, kView, kView, v0, kView, kView, n, grads.view_1, kView, 1, grads.view_1_bias},
        {g_v0, kView, kView, d.inputs, d.inputs_stride, kInputs, n, grads.combined, kInputs, 1, nullptr},
        // density: g_h^T features (+ bias)
        {d.grad_hidden, kDensity, kDensity, features, d.features_stride, kFeatures, n, grads.density, kDensity, 1, grads.density_bias},
        // rgb and skip, transposed (their 8 output rows as N): v2^T g_out into rgb[o][i], inputs^T g_out into skip[o][i]
        {v2, kView, kView, d.grad_outputs, kOutputs, kOutputs, n, grads.rgb, 1, kView, nullptr},
        {d.inputs, d.inputs_stride, kInputs, d.grad_outputs, kOutputs, kOutputs, n, grads.skip, 1, kInputs, nullptr},
    };
    for (const WeightArgs& a : launches) {
        fz_nerf_mlp_backward_weight_kernel<<<grid, kWgradThreads, kWgradSmemBytes, stream>>>(a, status);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace bwd

}  // namespace zf::nerf_mlp

int64_t zf_nerf_mlp_backward_workspace_size(const int64_t n) {
    using namespace zf::nerf_mlp::bwd;
    return n < 0 ? 0 : n * (3 * kView + kDensity) * 2;
}

int zf_nerf_mlp_backward_tc(const uint16_t* grad_outputs, const uint16_t* features, const int64_t features_stride, const uint16_t* inputs,
                            const int64_t inputs_stride, const uint16_t* activations, const zf_nerf_mlp_weights_t* weights, uint16_t* grad_features,
                            const int64_t grad_features_stride, const zf_nerf_mlp_grads* grads, void* workspace, const int64_t workspace_bytes,
                            const int64_t n, int* status, cudaStream_t stream) {
    using namespace zf::nerf_mlp::bwd;
    if (n < 0 || weights == nullptr || grads == nullptr || status == nullptr) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "invalid nerf mlp backward inputs");
    if (n == 0) return ZF_OK;
    if (workspace_bytes < zf_nerf_mlp_backward_workspace_size(n)) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "nerf mlp backward workspace too small");
    const void* pointers[] = {grad_outputs, features, inputs, activations, grad_features, workspace, weights->rgb_t, weights->view_2_t,
                              weights->view_1_t, weights->combined_t, weights->skip_t, weights->density_t};
    for (const void* p : pointers) {
        if (p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 != 0) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "nerf mlp tensors must be 16-byte aligned");
    }
    const float* grad_pointers[] = {grads->density, grads->density_bias, grads->combined, grads->skip, grads->view_1, grads->view_1_bias,
                                    grads->view_2, grads->view_2_bias, grads->rgb};
    for (const float* p : grad_pointers) {
        if (p == nullptr) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "nerf mlp gradients must be given");
    }
    if (features_stride % 8 != 0 || inputs_stride % 8 != 0 || grad_features_stride % 8 != 0 || features_stride < kFeatures || inputs_stride < kInputs ||
        grad_features_stride < kFeatures) {
        return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "invalid nerf mlp row strides");
    }
    const PackedMlpT w{weights->rgb_t, weights->view_2_t, weights->view_1_t, weights->combined_t, weights->skip_t, weights->density_t};
    uint16_t* ws = static_cast<uint16_t*>(workspace);
    const DataArgs d{grad_outputs, inputs, inputs_stride, activations, ws, ws + 3 * n * kView, grad_features, grad_features_stride, n};
    const cudaError_t e = launch_backward(w, d, *grads, features, status, stream);
    return e == cudaSuccess ? ZF_OK : zf::set_cuda_error(e, "nerf mlp backward");
}

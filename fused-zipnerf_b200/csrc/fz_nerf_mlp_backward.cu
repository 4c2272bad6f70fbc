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

#include <cuda.h>
#include <cudaTypedefs.h>

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
    const uint32_t* masks;          // [3, n, 8]: the ReLU masks of v0, v1, v2 (bit c % 32 of word c / 32)
    const uint32_t* hidden_masks;   // [n, 2]: h's
    uint16_t* grad_activations;     // [3, n, 256] out: g_v0, g_v1, g_v2
    uint16_t* grad_hidden;          // [n, 64] out: g_h
    uint16_t* grad_features;        // [n, grad_features_stride] out: columns 0-55
    int64_t grad_features_stride;
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

// N (32 or 64) accumulator columns of this thread's row, times the ReLU mask bits m (bit c of the 64-bit word: column
// k_first + c positive; all columns when masked is false), rounded to bf16, into row `row` of a K-major operand at
// column k_first (when dst is given) and into global memory at out_row + k_first (its first out_cols columns, when
// out_row is given)
template <int N>
__device__ __forceinline__ void masked_columns(const uint32_t taddr, const bool masked, const uint64_t m, uint8_t* dst, const int row,
                                               const int k_total, const int k_first, uint16_t* out_row, const int out_cols) {
    // 32 columns per tensor-memory load
    #pragma unroll
    for (int c = 0; c < N; c += 32) {
        uint32_t r[32];
        issue_load<32>(taddr + c, r);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        const uint32_t bits = static_cast<uint32_t>(m >> c);
        #pragma unroll
        for (int j = c / 8; j < c / 8 + 4; j++) {
            uint32_t words[4];
            #pragma unroll
            for (int q = 0; q < 4; q++) {
                const int col = 8 * (j - c / 8) + 2 * q;  // within this 32-column load
                float lo = __uint_as_float(r[col]), hi = __uint_as_float(r[col + 1]);
                if (masked) {
                    if (!((bits >> col) & 1u)) lo = 0.0f;
                    if (!((bits >> (col + 1)) & 1u)) hi = 0.0f;
                }
                words[q] = pack_bf16x2(lo, hi);
            }
            const uint4 out = make_uint4(words[0], words[1], words[2], words[3]);
            if (dst != nullptr) *reinterpret_cast<uint4*>(dst + canonical_offset(row, k_first + 8 * j, k_total)) = out;
            if (out_row != nullptr && 8 * j < out_cols) *reinterpret_cast<uint4*>(out_row + k_first + 8 * j) = out;
        }
    }
}

// this thread's mask bits of one tile: chunks g and g + 2 of v2, v1, v0 (64 bits each), then h's columns [32 g, 32 g + 32)
struct TileMasks {
    uint2 v[3][2];
    uint32_t h;
};

__device__ __forceinline__ TileMasks fetch_masks(const DataArgs& a, const int64_t sample, const int g) {
    TileMasks t{};
    if (sample < a.n) {
        #pragma unroll
        for (int k = 0; k < 3; k++) {
            const int index = 2 - k;  // v2, v1, v0
            const uint2* row = reinterpret_cast<const uint2*>(a.masks + (static_cast<int64_t>(index) * a.n + sample) * (kView / 32));
            #pragma unroll
            for (int i = 0; i < 2; i++) t.v[k][i] = __ldg(row + g + 2 * i);
        }
        t.h = __ldg(a.hidden_masks + sample * (kDensity / 32) + g);
    }
    return t;
}

__device__ __forceinline__ uint64_t bits64(const uint2 w) { return static_cast<uint64_t>(w.x) | (static_cast<uint64_t>(w.y) << 32); }

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
        // the ReLU mask bits of the next tile are fetched while this tile's layers run
        int64_t tile = blockIdx.x;
        uint4 next = make_uint4(0, 0, 0, 0);
        TileMasks masks{}, next_masks{};
        if (tile < n_tiles) {
            store_gout(fetch_gout(tile));
            publish(in_bar);
            masks = fetch_masks(a, tile * kTileRows + row, g);
        }
        for (; tile < n_tiles && ok; tile += gridDim.x) {
            const int64_t sample = tile * kTileRows + row;
            const bool valid = sample < n;
            const bool more = tile + gridDim.x < n_tiles;
            // E0-E2: g_v2, g_v1, g_v0 masked by v2, v1, v0: chunks g and g + 2 -> act and global memory
            #pragma unroll
            for (int k = 0; k < 3; k++) {
                if (!(ok = accumulator_ready())) break;
                const int index = 2 - k;  // v2, v1, v0
                uint16_t* out = valid ? a.grad_activations + (static_cast<int64_t>(index) * n + sample) * kView : nullptr;
                const uint32_t region = lanes + (layer & 1u) * kRegionColumns;
                #pragma unroll
                for (int i = 0; i < 2; i++) {
                    const int j = g + 2 * i;
                    masked_columns<kSlice>(region + kSlice * j, true, bits64(masks.v[k][i]), act, row, kView, kSlice * j, out, kSlice);
                    publish(chunk_bar(j));
                }
                layer++;
                if (k == 0 && more) {
                    next = fetch_gout(tile + gridDim.x);
                    next_masks = fetch_masks(a, (tile + gridDim.x) * kTileRows + row, g);
                }
            }
            if (!ok) break;
            // E3: g_h = g_in[:, 0:64] masked by h: columns [32 g, 32 g + 32) -> the g_h tile and global memory
            if (!(ok = accumulator_ready())) break;
            masked_columns<32>(lanes + (layer & 1u) * kRegionColumns + 32 * g, true, masks.h, gh, row, kDensity, 32 * g,
                               valid ? a.grad_hidden + sample * kDensity : nullptr, 32);
            publish(h_bar);
            layer++;
            // E4: g_features, columns [32 g, 32 g + 32) below 56, then the next tile's output gradients
            if (!(ok = accumulator_ready())) break;
            masked_columns<32>(lanes + (layer & 1u) * kRegionColumns + 32 * g, false, 0, nullptr, row, 0, 32 * g,
                               valid ? a.grad_features + sample * a.grad_features_stride : nullptr, kFeatures - 32 * g);
            layer++;
            masks = next_masks;
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

// Persistent CTAs over K-tiles of 32 samples. Warp 0 (one lane) loads each K-tile's G and V with TMA tensor copies
// (no multicast) into a six-slot ring: operands of 64 or more columns as 64-column boxes with the 128-byte swizzle,
// the 8-column output gradients as one 16-column box with the 32-byte swizzle, columns past the matrix and rows past n
// zero-filled. Warp 1 (one lane) issues the MN-major MMAs into tensor memory (two M = 128 halves for m_pad = 256).
// Warps 2-9 sum the bias columns from the same slots, then move the accumulators to dW with vector fp32 atomics.
constexpr int kWgradWarps = 10;
constexpr int kWgradThreads = 32 * kWgradWarps;
constexpr int kWgradFirstSumWarp = 2;
constexpr int kKTile = 32;           // samples per K-tile (2 MMA K steps)
constexpr int kWgradStages = 6;
constexpr int kWgradMaxM = 256;      // two M = 128 halves
constexpr int kWgradMaxN = 256;
constexpr int kBoxCols = 64;         // columns of a 128-byte-swizzled box
constexpr int kBoxBytes = kKTile * kBoxCols * 2;     // 4 KB: the MN-atom stride of a tile
constexpr int kNarrowCols = 16;      // columns of the 32-byte-swizzled box (the output gradients)
constexpr int kNarrowBytes = kKTile * kNarrowCols * 2;
constexpr int kWgradStageBytes = kKTile * (kWgradMaxM + kWgradMaxN) * 2;  // 32 KB
constexpr int kWgradSumOffset = kWgradStages * kWgradStageBytes;           // 8 x 256 fp32 partial bias sums
constexpr int kWgradBarOffset = kWgradSumOffset + 8 * kWgradMaxM * 4;
constexpr int kWgradBars = 2 * kWgradStages + 1;                           // full[stages], empty[stages], done
constexpr int kWgradSmemBytes = 1024 + kWgradBarOffset + 8 * kWgradBars + 16;  // 1024: alignment of the swizzled ring
static_assert(kWgradSmemBytes <= 227 * 1024, "one CTA per SM");

struct WeightArgs {
    CUtensorMap g_map;          // G [n, m_cols] bf16, 64-column boxes of kKTile rows, 128-byte swizzle
    CUtensorMap v_map;          // V [n, k_cols] bf16, 64-column boxes (128-byte swizzle) or one 16-column box (32-byte)
    int m_pad;                  // 128 or 256 (G boxes: m_pad / 64)
    int k_pad;                  // 16 (one narrow box), 64, 128 or 256 (V boxes: k_pad / 64)
    int m_cols;                 // <= m_pad
    int k_cols;                 // <= k_pad
    int64_t n;
    float* dw;                  // dW[m][k] at dw[m * dw_m_stride + k * dw_k_stride] (+=)
    int64_t dw_m_stride;
    int64_t dw_k_stride;
    float* bias;                // bias[m] (+=), or null
};

__device__ __forceinline__ void tma_load_2d(const uint32_t dst, const CUtensorMap* map, const int x, const int y, const uint32_t bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
                 "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void red_add_v4(float* address, const float a, const float b, const float c, const float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(address), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

__device__ __forceinline__ uint64_t wgrad_descriptor(const uint32_t address, const bool narrow) {
    return narrow ? mn_sw32_descriptor(address) : mn_sw128_descriptor(address, kKTile);
}

__global__ void __launch_bounds__(kWgradThreads, 1) fz_nerf_mlp_backward_weight_kernel(const __grid_constant__ WeightArgs a, int* status) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // the swizzle patterns follow shared-memory address bits: the ring starts on a 1024-byte boundary
    uint8_t* smem = smem_raw + ((1024u - (smem_address(smem_raw) & 1023u)) & 1023u);
    const uint32_t base = smem_address(smem);
    const uint32_t bar0 = base + kWgradBarOffset;
    auto full_bar = [&](const uint32_t i) { return bar0 + 8u * i; };
    auto empty_bar = [&](const uint32_t i) { return bar0 + 8u * (kWgradStages + i); };
    const uint32_t done_bar = bar0 + 8u * (2 * kWgradStages);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kWgradBarOffset + 8 * kWgradBars);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + kWgradBarOffset + 8 * kWgradBars + 4);
    float* partial = reinterpret_cast<float*>(smem + kWgradSumOffset);
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const bool narrow = a.k_pad < kBoxCols;
    const int m_halves = a.m_pad / 128;
    const int g_boxes = a.m_pad / kBoxCols, v_boxes = narrow ? 1 : a.k_pad / kBoxCols;
    const uint32_t g_bytes = static_cast<uint32_t>(g_boxes * kBoxBytes);
    const uint32_t stage_bytes = g_bytes + static_cast<uint32_t>(narrow ? kNarrowBytes : v_boxes * kBoxBytes);
    const int64_t n_tiles = (a.n + kKTile - 1) / kKTile;
    const int my_tiles = blockIdx.x < n_tiles ? static_cast<int>((n_tiles - 1 - blockIdx.x) / gridDim.x + 1) : 0;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_address(tmem_slot)), "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 32) {
        for (int i = 0; i < kWgradStages; i++) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(full_bar(i)), "r"(1));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(empty_bar(i)), "r"(1 + kWgradWarps - kWgradFirstSumWarp));
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(done_bar), "r"(1));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *abort = 0;
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    if (warp == 0) {
        // TMA producer
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a.g_map)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a.v_map)) : "memory");
            int issued = 0;
            for (int i = 0; i < my_tiles; i++) {
                const uint32_t slot = i % kWgradStages;
                if (i >= kWgradStages && !wait_phase(empty_bar(slot), (i / kWgradStages - 1) & 1u, abort)) break;
                const int y = static_cast<int>((blockIdx.x + static_cast<int64_t>(i) * gridDim.x) * kKTile);
                const uint32_t stage = base + slot * kWgradStageBytes;
                expect_bytes(full_bar(slot), stage_bytes);
                for (int b = 0; b < g_boxes; b++) tma_load_2d(stage + b * kBoxBytes, &a.g_map, b * kBoxCols, y, full_bar(slot));
                for (int b = 0; b < v_boxes; b++) tma_load_2d(stage + g_bytes + b * kBoxBytes, &a.v_map, b * kBoxCols, y, full_bar(slot));
                issued = i + 1;
            }
            // every copy issued has landed before the CTA's shared memory can go to another CTA
            for (int i = issued > kWgradStages ? issued - kWgradStages : 0; i < issued; i++) drain_phase(full_bar(i % kWgradStages), (i / kWgradStages) & 1u);
        }
    } else if (warp == 1) {
        // MMA issuer
        if (lane == 0) {
            const uint32_t idesc = instr_descriptor(kTileRows, a.k_pad, true, true);
            for (int i = 0; i < my_tiles; i++) {
                const uint32_t slot = i % kWgradStages;
                if (!wait_phase(full_bar(slot), (i / kWgradStages) & 1u, abort)) break;
                fence_after_sync();
                const uint32_t stage = base + slot * kWgradStageBytes;
                for (int h = 0; h < m_halves; h++) {
                    for (int k = 0; k < kKTile / kMmaK; k++) {
                        // M-half h: two 64-column atoms further; K step k: two 8-row groups further
                        const uint32_t a_addr = stage + h * 2 * kBoxBytes + k * 2 * 1024;
                        const uint32_t b_addr = stage + g_bytes + k * 2 * (narrow ? 256 : 1024);
                        mma(tmem + h * a.k_pad, wgrad_descriptor(a_addr, false), wgrad_descriptor(b_addr, narrow), idesc, (i > 0 || k > 0) ? 1u : 0u);
                    }
                }
                commit(empty_bar(slot));
            }
            commit(done_bar);
        }
    } else {
        // bias sums: warp w' = warp - 2 takes rows w' + 8 j of each K-tile, lane l the 8 columns of word l (box l / 8,
        // 16-byte chunk l % 8, stored at chunk (l % 8) ^ w' of its 128-byte row)
        const int wp = warp - kWgradFirstSumWarp;
        const bool sums = a.bias != nullptr && 8 * lane < a.m_cols;
        float column_sum[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        const uint32_t read_offset = (lane / 8) * kBoxBytes + wp * 128 + (((lane % 8) ^ wp) << 4);
        bool ok = true;
        for (int i = 0; i < my_tiles; i++) {
            const uint32_t slot = i % kWgradStages;
            if (!(ok = wait_phase(full_bar(slot), (i / kWgradStages) & 1u, abort))) break;
            if (sums) {
                const uint8_t* tile = smem + slot * kWgradStageBytes + read_offset;
                #pragma unroll
                for (int j = 0; j < kKTile / 8; j++) {
                    const uint4 v = *reinterpret_cast<const uint4*>(tile + j * 1024);
                    const uint32_t words[4] = {v.x, v.y, v.z, v.w};
                    #pragma unroll
                    for (int q = 0; q < 4; q++) {
                        column_sum[2 * q] += __uint_as_float(words[q] << 16);
                        column_sum[2 * q + 1] += __uint_as_float(words[q] & 0xFFFF0000u);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) arrive(empty_bar(slot));
        }
        // every MMA is done: the accumulators go to dW (rows 128 h + 32 (warp % 4) + lane; with two M-halves warp pair
        // p = w' / 4 takes half p, with one both pairs take alternate 16-column chunks)
        ok = ok && (my_tiles == 0 || wait_phase(done_bar, 0, abort));
        ok = __all_sync(0xFFFFFFFFu, ok);  // the tensor-memory loads below are warp-collective
        fence_after_sync();
        const int pair = wp / 4, quadrant = warp % 4;
        const int h = m_halves == 2 ? pair : 0;
        const int m = 128 * h + 32 * quadrant + lane;
        const bool vector = a.dw_k_stride == 1 && (a.dw_m_stride & 3) == 0 && (reinterpret_cast<uintptr_t>(a.dw) & 15) == 0;
        if (ok && my_tiles > 0) {
            const uint32_t lanes = tmem + (static_cast<uint32_t>(32 * quadrant) << 16) + h * a.k_pad;
            for (int c = (m_halves == 2 ? 0 : 16 * pair); c < a.k_pad; c += (m_halves == 2 ? 16 : 32)) {
                uint32_t r[16];
                issue_load<16>(lanes + c, r);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (m < a.m_cols) {
                    float* row = a.dw + m * a.dw_m_stride;
                    #pragma unroll
                    for (int j = 0; j < 16; j += 4) {
                        if (vector && c + j + 4 <= a.k_cols) {
                            red_add_v4(row + c + j, __uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
                        } else {
                            #pragma unroll
                            for (int e = 0; e < 4; e++) {
                                if (c + j + e < a.k_cols) atomicAdd(row + (c + j + e) * a.dw_k_stride, __uint_as_float(r[j + e]));
                            }
                        }
                    }
                }
            }
        }
        // the bias: the 8 row phases' partial sums through shared memory, one atomic per column
        if (a.bias != nullptr) {
            #pragma unroll
            for (int e = 0; e < 8; e++) partial[wp * kWgradMaxM + 8 * lane + e] = column_sum[e];
            asm volatile("bar.sync 1, %0;" ::"n"(32 * (kWgradWarps - kWgradFirstSumWarp)) : "memory");
            const int column = tid - 32 * kWgradFirstSumWarp;
            if (ok && my_tiles > 0 && column < a.m_cols) {
                float total = 0.0f;
                #pragma unroll
                for (int w = 0; w < kWgradWarps - kWgradFirstSumWarp; w++) total += partial[w * kWgradMaxM + column];
                atomicAdd(a.bias + column, total);
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (tid == 32 && my_tiles > 0) drain_phase(done_bar, 0);  // no MMA still writes the tensor memory freed below
    if (tid == 0 && *abort) atomicExch(status, kWaitTimeout);
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}

// cuTensorMapEncodeTiled from the driver through the runtime (the library links no driver library)
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess) p = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// the tensor map of a [n, cols] bf16 matrix with row stride `stride` elements, boxes of kKTile rows and 64 (128-byte
// swizzle) or 16 (32-byte swizzle) columns
bool encode_operand(CUtensorMap* map, const uint16_t* base, const int cols, const int64_t stride, const int64_t n, const bool narrow) {
    const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (encode == nullptr) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(n)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(narrow ? kNarrowCols : kBoxCols), static_cast<cuuint32_t>(kKTile)};
    const cuuint32_t element_strides[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(base), dims, strides, box, element_strides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, narrow ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_backward(const PackedMlpT& w, const DataArgs& d, const zf_nerf_mlp_grads& grads, const uint16_t* features,
                            const int64_t features_stride, const uint16_t* activations, int* status, cudaStream_t stream) {
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
    const uint16_t* v0 = activations;
    const uint16_t* v1 = activations + n * kView;
    const uint16_t* v2 = activations + 2 * n * kView;
    struct Gemm {
        const uint16_t* g;
        int64_t g_stride;
        int m_cols;
        const uint16_t* v;
        int64_t v_stride;
        int k_cols;
        float* dw;
        int64_t dw_m_stride, dw_k_stride;
        float* bias;
    };
    const Gemm gemms[] = {
        // view_2: g_v2^T v1 (+ bias), view_1: g_v1^T v0 (+ bias), combined: g_v0^T inputs (its bias in the bias lane)
        {g_v2, kView, kView, v1, kView, kView, grads.view_2, kView, 1, grads.view_2_bias},
        {g_v1, kView, kView, v0, kView, kView, grads.view_1, kView, 1, grads.view_1_bias},
        {g_v0, kView, kView, d.inputs, d.inputs_stride, kInputs, grads.combined, kInputs, 1, nullptr},
        // density: g_h^T features (+ bias)
        {d.grad_hidden, kDensity, kDensity, features, features_stride, kFeatures, grads.density, kDensity, 1, grads.density_bias},
        // rgb and skip, transposed (their 8 output rows as N): v2^T g_out into rgb[o][i], inputs^T g_out into skip[o][i]
        {v2, kView, kView, d.grad_outputs, kOutputs, kOutputs, grads.rgb, 1, kView, nullptr},
        {d.inputs, d.inputs_stride, kInputs, d.grad_outputs, kOutputs, kOutputs, grads.skip, 1, kInputs, nullptr},
    };
    for (const Gemm& gemm : gemms) {
        WeightArgs a{};
        a.m_pad = gemm.m_cols > 128 ? 256 : 128;
        a.k_pad = gemm.k_cols <= kNarrowCols ? kNarrowCols : (gemm.k_cols + kBoxCols - 1) / kBoxCols * kBoxCols;
        a.m_cols = gemm.m_cols;
        a.k_cols = gemm.k_cols;
        a.n = n;
        a.dw = gemm.dw;
        a.dw_m_stride = gemm.dw_m_stride;
        a.dw_k_stride = gemm.dw_k_stride;
        a.bias = gemm.bias;
        if (!encode_operand(&a.g_map, gemm.g, gemm.m_cols, gemm.g_stride, n, false) ||
            !encode_operand(&a.v_map, gemm.v, gemm.k_cols, gemm.v_stride, n, a.k_pad == kNarrowCols)) {
            return cudaErrorInvalidValue;
        }
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
    // the weight gradients' tensor copies address samples with 32-bit coordinates
    if (n > INT32_MAX - 64) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "nerf mlp backward: too many samples");
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
    const uint32_t* masks = reinterpret_cast<const uint32_t*>(activations + 3 * n * kView);
    const DataArgs d{grad_outputs, inputs, inputs_stride, masks, masks + 3 * n * (kView / 32), ws, ws + 3 * n * kView, grad_features, grad_features_stride, n};
    const cudaError_t e = launch_backward(w, d, *grads, features, features_stride, activations, status, stream);
    return e == cudaSuccess ? ZF_OK : zf::set_cuda_error(e, "nerf mlp backward");
}

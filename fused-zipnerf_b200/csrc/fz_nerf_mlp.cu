// fz_nerf_mlp.cu -- the NeRF MLP forward on the tcgen05 tensor cores: a persistent kernel, one CTA per SM walking over
// 128-sample tiles, bf16 operands in shared memory, fp32 accumulators in tensor memory. Per tile it runs the layer
// chain of NerfMlp::forward (nerf_mlp.h:35-45) on the packed (folded) weights:
//   L0  h  = relu(features @ w_density^T + b_density)      -> columns 0-63 of the inputs tile (and of the global inputs)
//   L1  v0 = relu(inputs @ w_combined^T)                    inputs = [h | encoded direction | 1], bias in the bias lane
//   L2  v1 = relu(v0 @ w_1^T + b_1)
//   L3  v2 = relu(v1 @ w_2^T + b_2)
//   L4  out = inputs @ w_skip^T + v2 @ w_rgb^T               8 outputs
// The activations never leave the SM: each layer's epilogue reads its accumulator rows from tensor memory, applies bias
// and ReLU and writes bf16 back to shared memory as the next layer's A operand.
//
// Warp roles (576 threads): warp 0 issues the MMAs (one thread), warp 1 streams the weights (one thread), warps 2-17 run
// the epilogues (one warp per tensor-memory lane quadrant and 64-column chunk) and load the input tiles. The weights are packed as K-slices of 64 input columns with all output rows
// (zipnerf_b200.nerf_mlp.pack), so every MMA runs at the full N of its layer; the slices arrive by bulk copies
// (cp.async.bulk, no multicast) through a four-slot ring, four slices ahead of the MMAs. Tensor memory holds two
// 256-column accumulator regions used by alternate layers. An epilogue publishes its layer's activations 64 columns at
// a time (one mbarrier per 64-column chunk), and the next layer's MMAs over K-slice j start as soon as chunk j is in
// shared memory, so epilogue and MMAs overlap. The next tile's inputs are loaded into registers while the current
// tile's layers run and stored to shared memory once its last MMAs are done.
//
// Every wait is bounded: a wait that runs out raises the CTA's abort flag, which ends every role's loop; the CTA then
// waits (bounded) for its own MMAs and weight copies in flight, frees its tensor memory and sets *status. A status of 1
// leaves this launch's outputs undefined.
//
// Shared-memory operands use the canonical K-major layout without swizzle: 8-row x 16-byte core matrices stored
// contiguously (128 bytes), K-adjacent core matrices 128 bytes apart (leading byte offset), 8-row groups
// (K / 8) * 128 bytes apart (stride byte offset), K the operand's stored width (a weight slice: its own width).
#include "zf_mlp.h"
#include "fz_status.h"
#include "fz_tcgen05.cuh"

#include <cuda_runtime.h>

#include <cstdint>

namespace zf::nerf_mlp {

constexpr int kFeatures = 56;        // NeRF features per sample: 10 levels x (4 + 1) = 50, padded to 56
constexpr int kFeaturesK = 64;       // padded to the MMA K step of 16
constexpr int kDensity = 64;         // density width = hidden columns of the inputs
constexpr int kInputs = 96;          // hidden 64 + direction block 32 (its last column the bias lane 1.0)
constexpr int kView = 256;
constexpr int kOutputs = 8;          // raw density, 3 rgb logits, 4 padding
constexpr int kOutputsN = 16;        // the smallest N of an M = 128 MMA
// the training record behind the activations v0, v1, v2 ([3, n, 256] bf16): their ReLU masks, [3, n, 8] words (bit
// c % 32 of word c / 32: column c positive), then h's, [n, 2] words
constexpr int kMaskWords = kView / 32;
constexpr int kHiddenMaskWords = kDensity / 32;

// warp roles
constexpr int kMmaWarp = 0;
constexpr int kProducerWarp = 1;
constexpr int kFirstEpilogueWarp = 2;
// whether one lane per epilogue warp polls the accumulator barrier (the others take its outcome)
#ifndef ZF_MLP_POLL_LANE0
#define ZF_MLP_POLL_LANE0 0
#endif
#ifndef ZF_MLP_EPILOGUE_WARPS
#define ZF_MLP_EPILOGUE_WARPS 8
#endif
constexpr int kEpilogueWarps = ZF_MLP_EPILOGUE_WARPS;  // 4 x the chunk groups: a group of 4 warps covers the 128 lanes
constexpr int kChunkGroups = kEpilogueWarps / 4;
static_assert(kChunkGroups == 1 || kChunkGroups == 2 || kChunkGroups == 4, "each group takes whole 64-column chunks");
constexpr int kEpilogueThreads = 32 * kEpilogueWarps;
constexpr int kThreads = 32 * (kFirstEpilogueWarp + kEpilogueWarps);

constexpr uint32_t kTmemColumns = 512;   // two accumulator regions of 256 columns
constexpr uint32_t kRegionColumns = 256;

// weight stages: K-slices of 64 input columns (the combined layer's last slice 32), all output rows each
constexpr int kSlice = 64;
constexpr int kChunks = kView / kSlice;                        // 64-column chunks of a 256-wide activation
constexpr int kStagesPerTile = 12;                             // density, combined x 2, view_1 x 4, view_2 x 4, skip + rgb
constexpr int kRingSlots = 4;
constexpr int kStageBytes = kView * kSlice * 2;                // 32 KB
constexpr int kSkipBytes = kOutputsN * kInputs * 2;            // skip weights at the start of the last stage
constexpr int kRgbStageOffset = kSkipBytes;                    // rgb weights behind them
static_assert(kRgbStageOffset % 16 == 0 && kRgbStageOffset + kOutputsN * kView * 2 <= kStageBytes, "skip and rgb share one stage");

// shared-memory carve-up (bytes)
constexpr int kActBytes = kTileRows * kView * 2;               // 64 KB: features tile, then v0, v1, v2
constexpr int kInBytes = kTileRows * kInputs * 2;              // 24 KB: the inputs tile
constexpr int kBiasFloats = kDensity + 2 * kView;              // density, view_1 and view_2 biases
constexpr int kActOffset = 0;
constexpr int kInOffset = kActOffset + kActBytes;
constexpr int kRingOffset = kInOffset + kInBytes;
constexpr int kBiasOffset = kRingOffset + kRingSlots * kStageBytes;
constexpr int kBarOffset = kBiasOffset + kBiasFloats * 4;
// full[4], empty[4], acc_full, in_ready, h_ready, chunk[4], drain
constexpr int kNumBarriers = 2 * kRingSlots + 3 + kChunks + 1;
constexpr int kMiscOffset = kBarOffset + kNumBarriers * 8;     // tensor-memory slot, abort flag
constexpr int kSmemBytes = kMiscOffset + 16;
static_assert(kBarOffset % 8 == 0, "mbarriers are 8-byte aligned");
static_assert(kSmemBytes <= 227 * 1024, "one CTA per SM");

// per-thread share of a tile's inputs: features 128 rows x 8 16-byte words (56 columns + zero padding) and direction
// blocks 128 rows x 4 words
constexpr int kInputWords = kTileRows * (kFeaturesK / 8 + 4) / kEpilogueThreads;
static_assert(kInputWords * kEpilogueThreads == kTileRows * (kFeaturesK / 8 + 4), "the input words divide evenly");

// packed weights: bf16 [out x in] with zero padding in the canonical K-major order, fp32 biases
struct PackedMlp {
    const uint16_t* density;      // [64, 64]: features 56 -> 64 zero columns
    const float* density_bias;    // [64]
    const uint16_t* combined;     // [256, 96]: folded bottleneck and first view layer, bias in column 95
    const uint16_t* skip;         // [16, 96]: rows 0-3 density and rgb skip terms, rows 4-15 zero
    const uint16_t* view_1;       // [256, 256]
    const float* view_1_bias;     // [256]
    const uint16_t* view_2;       // [256, 256]
    const float* view_2_bias;     // [256]
    const uint16_t* rgb;          // [16, 256]: rows 1-3 the rgb weights of v2, the others zero
};

// N accumulator columns of this thread's row (N = 16, or a multiple of 32 loaded 32 at a time with one wait) + bias
// (shared memory, or none), ReLU, bf16, into row `row` of a K-major operand at column k_first (and into global memory
// at `global_row` when given; and, when mask_words is given, bit c % 32 of word c / 32 set where column c came out
// positive, N a multiple of 32)
template <int N, bool kMasks = false>
__device__ __forceinline__ void relu_columns(const uint32_t taddr, const float* bias, uint8_t* dst, const int row, const int k_total, const int k_first,
                                             uint16_t* global_row, uint32_t* mask_words = nullptr) {
    uint32_t bits[N / 32 > 0 ? N / 32 : 1] = {};
    uint32_t r[N];
    if constexpr (N == 16) {
        issue_load<16>(taddr, r);
    }
    else {
        #pragma unroll
        for (int c = 0; c < N; c += 32) issue_load<32>(taddr + c, r + c);
    }
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    #pragma unroll
    for (int j = 0; j < N; j += 8) {
        uint32_t words[4];
        #pragma unroll
        for (int q = 0; q < 4; q++) {
            float lo = __uint_as_float(r[j + 2 * q]), hi = __uint_as_float(r[j + 2 * q + 1]);
            if (bias != nullptr) {
                lo += bias[j + 2 * q];
                hi += bias[j + 2 * q + 1];
            }
            words[q] = pack_bf16x2_relu(lo, hi);
            if constexpr (kMasks && N >= 32) {
                const uint32_t pair = (__uint_as_float(words[q] << 16) > 0.0f ? 1u : 0u) | (__uint_as_float(words[q] & 0xFFFF0000u) > 0.0f ? 2u : 0u);
                bits[(j + 2 * q) / 32] |= pair << ((j + 2 * q) % 32);
            }
        }
        const uint4 out = make_uint4(words[0], words[1], words[2], words[3]);
        *reinterpret_cast<uint4*>(dst + canonical_offset(row, k_first + j, k_total)) = out;
        if (global_row != nullptr) *reinterpret_cast<uint4*>(global_row + k_first + j) = out;
    }
    if constexpr (kMasks && N == 32) {
        if (mask_words != nullptr) *mask_words = bits[0];
    }
    else if constexpr (kMasks && N == 64) {
        if (mask_words != nullptr) *reinterpret_cast<uint2*>(mask_words) = make_uint2(bits[0], bits[1]);
    }
}

// input word i of this epilogue thread (tid) for the tile at `first`: its source in global memory (null for a zero
// word) and its destination in shared memory (act: features with the K-major layout of 64 columns; in: the direction
// block, columns 64-95)
__device__ __forceinline__ void input_word(const int i, const int tid, const uint16_t* __restrict__ features, const int64_t features_stride,
                                           const uint16_t* inputs, const int64_t inputs_stride, const int64_t first, const int64_t n,
                                           const uint4*& src, uint32_t& dst_offset, bool& to_act) {
    const int q = tid + i * kEpilogueThreads;
    constexpr int kFeatureWords = kTileRows * (kFeaturesK / 8);
    src = nullptr;
    if (q < kFeatureWords) {
        // eight consecutive words: one 16-byte chunk of eight consecutive rows, which is one core matrix (128
        // contiguous bytes of shared memory, all 32 banks)
        const int r = (q / (8 * (kFeaturesK / 8))) * 8 + q % 8, c = (q / 8) % (kFeaturesK / 8);
        if (first + r < n && c < kFeatures / 8) src = reinterpret_cast<const uint4*>(features + (first + r) * features_stride) + c;
        dst_offset = canonical_offset(r, 8 * c, kFeaturesK);
        to_act = true;
    }
    else {
        const int r = (q - kFeatureWords) / 4, c = (q - kFeatureWords) % 4;
        if (first + r < n) src = reinterpret_cast<const uint4*>(inputs + (first + r) * inputs_stride + kDensity) + c;
        dst_offset = canonical_offset(r, kDensity + 8 * c, kInputs);
        to_act = false;
    }
}

// this thread's words of the tile's inputs (zeros for rows past n) into registers
__device__ __forceinline__ void fetch_inputs(uint4 (&words)[kInputWords], const int tid, const uint16_t* __restrict__ features, const int64_t features_stride,
                                             const uint16_t* inputs, const int64_t inputs_stride, const int64_t first, const int64_t n) {
    #pragma unroll
    for (int i = 0; i < kInputWords; i++) {
        const uint4* src;
        uint32_t offset;
        bool to_act;
        input_word(i, tid, features, features_stride, inputs, inputs_stride, first, n, src, offset, to_act);
        words[i] = src != nullptr ? __ldg(src) : make_uint4(0, 0, 0, 0);
    }
}

// the fetched words into the features tile (act) and the direction block (in)
__device__ __forceinline__ void store_inputs(const uint4 (&words)[kInputWords], const int tid, uint8_t* act, uint8_t* in) {
    #pragma unroll
    for (int i = 0; i < kInputWords; i++) {
        const uint4* src;
        uint32_t offset;
        bool to_act;
        input_word(i, tid, nullptr, 0, nullptr, 0, 0, 0, src, offset, to_act);
        *reinterpret_cast<uint4*>((to_act ? act : in) + offset) = words[i];
    }
}

// source and size of weight stage s of a tile (the second part only for the last stage)
struct Stage {
    const void* src0;
    uint32_t bytes0;
    const void* src1;
    uint32_t bytes1;
};

__device__ __forceinline__ Stage weight_stage(const PackedMlp& w, const int s) {
    if (s == 0) return {w.density, kDensity * kFeaturesK * 2, nullptr, 0};
    if (s == 1) return {w.combined, kView * kSlice * 2, nullptr, 0};
    if (s == 2) return {w.combined + kView * kSlice, kView * (kInputs - kSlice) * 2, nullptr, 0};
    if (s < 7) return {w.view_1 + (s - 3) * kView * kSlice, kStageBytes, nullptr, 0};
    if (s < 11) return {w.view_2 + (s - 7) * kView * kSlice, kStageBytes, nullptr, 0};
    return {w.skip, kSkipBytes, w.rgb, kOutputsN * kView * 2};
}

// features [n, 56] bf16 (row stride features_stride), inputs [n, 96] bf16 (row stride inputs_stride; the direction
// block in columns 64-95 is read, the hidden layer written to columns 0-63), outputs [n, 8] bf16
// kRecord: the training forward, which writes the record (activations non-null); the inference forward compiles
// without the mask bits' work in its epilogues
template <bool kRecord>
__global__ void __launch_bounds__(kThreads, 1)
    fz_nerf_mlp_forward_kernel(const uint16_t* __restrict__ features, const int64_t features_stride, uint16_t* __restrict__ inputs,
                               const int64_t inputs_stride, const PackedMlp w, uint16_t* __restrict__ outputs, uint16_t* __restrict__ activations,
                               const int64_t n, int* status) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint32_t* masks = activations != nullptr ? reinterpret_cast<uint32_t*>(activations + 3 * n * kView) : nullptr;
    uint8_t* act = smem + kActOffset;
    uint8_t* in = smem + kInOffset;
    float* bias = reinterpret_cast<float*>(smem + kBiasOffset);  // density [64], view_1 [256], view_2 [256]
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOffset);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kMiscOffset);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + kMiscOffset + 4);
    const uint32_t bar0 = smem_address(bars);
    auto full_bar = [&](const uint32_t slot) { return bar0 + 8u * slot; };
    auto empty_bar = [&](const uint32_t slot) { return bar0 + 8u * (kRingSlots + slot); };
    const uint32_t acc_bar = bar0 + 8u * (2 * kRingSlots);      // a layer's MMAs are done (tcgen05.commit)
    const uint32_t in_bar = acc_bar + 8u;                      // the tile's inputs are in shared memory
    const uint32_t h_bar = in_bar + 8u;                        // the hidden layer h is in the inputs tile
    auto chunk_bar = [&](const int c) { return h_bar + 8u * (1 + c); };  // 64 columns of the next A operand are written
    const uint32_t drain_bar = h_bar + 8u * (1 + kChunks);
    const uint32_t ring = smem_address(smem + kRingOffset);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
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
        for (int c = 0; c < kChunks; c++) asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(chunk_bar(c)), "r"(128));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(drain_bar), "r"(1));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *abort = 0;
    }
    for (int i = threadIdx.x; i < kBiasFloats; i += kThreads) {
        bias[i] = i < kDensity ? __ldg(w.density_bias + i) : i < kDensity + kView ? __ldg(w.view_1_bias + i - kDensity)
                                                                                   : __ldg(w.view_2_bias + i - kDensity - kView);
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;
    uint32_t stages_issued = 0;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            // the weight stages of every tile of this CTA, up to a ring's worth ahead of the MMAs
            for (int64_t tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                for (int s = 0; s < kStagesPerTile; s++) {
                    const uint32_t slot = stages_issued % kRingSlots;
                    if (stages_issued >= kRingSlots && !wait_phase(empty_bar(slot), (stages_issued / kRingSlots - 1) & 1u, abort)) {
                        ok = false;
                        break;
                    }
                    const Stage st = weight_stage(w, s);
                    expect_bytes(full_bar(slot), st.bytes0 + st.bytes1);
                    bulk_copy(ring + slot * kStageBytes, st.src0, st.bytes0, full_bar(slot));
                    if (st.bytes1 != 0) bulk_copy(ring + slot * kStageBytes + kRgbStageOffset, st.src1, st.bytes1, full_bar(slot));
                    stages_issued++;
                }
            }
        }
    }
    else if (warp == kMmaWarp) {
        if (lane == 0) {
            uint32_t stage = 0, layer = 0, inputs_seen = 0, hidden_seen = 0;
            uint32_t chunks_seen[kChunks] = {0, 0, 0, 0};
            // the next weight stage (waits for it to land); release() commits its slot's empty barrier
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
            // chunk c of the next A operand is in shared memory (the epilogue of the previous layer)
            auto chunk_ready = [&](const int c) -> bool {
                const bool done = wait_phase(chunk_bar(c), chunks_seen[c] & 1u, abort);
                chunks_seen[c]++;
                fence_after_sync();
                return done;
            };
            const uint32_t a_act = smem_address(act), a_in = smem_address(in);
            for (int64_t tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                uint32_t b = 0;
                // L0: h = features @ density^T (N = 64)
                uint32_t d = tmem + (layer & 1u) * kRegionColumns;
                ok = wait_phase(in_bar, inputs_seen & 1u, abort);
                inputs_seen++;
                fence_after_sync();
                if (!(ok = ok && take(b))) break;
                mma_chain(d, a_act, kFeaturesK, b, kFeaturesK, kDensity, kFeaturesK, false);
                release();
                commit(acc_bar);
                layer++;
                // L1: v0 = inputs @ combined^T: K-slice 0 reads h (every epilogue thread has written its part), K-slice 1
                // the direction block
                d = tmem + (layer & 1u) * kRegionColumns;
                ok = wait_phase(h_bar, hidden_seen & 1u, abort);
                hidden_seen++;
                fence_after_sync();
                if (!(ok = ok && take(b))) break;
                mma_chain(d, a_in, kInputs, b, kSlice, kView, kSlice, false);
                release();
                if (!(ok = take(b))) break;
                mma_chain(d, a_in + (kSlice / 8) * 128, kInputs, b, kInputs - kSlice, kView, kInputs - kSlice, true);
                release();
                commit(acc_bar);
                layer++;
                // L2, L3: K-slice j of the view layers reads chunk j of the previous activation
                for (int k = 2; k <= 3 && ok; k++) {
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
                // L4: out = inputs @ skip^T + v2 @ rgb^T (N = 16), after every chunk of v2
                d = tmem + (layer & 1u) * kRegionColumns;
                for (int j = 0; j < kChunks && ok; j++) ok = chunk_ready(j);
                if (!(ok = ok && take(b))) break;
                mma_chain(d, a_in, kInputs, b, kInputs, kOutputsN, kInputs, false);
                mma_chain(d, a_act, kView, b + kRgbStageOffset, kView, kOutputsN, kView, true);
                release();
                commit(acc_bar);
                layer++;
            }
        }
    }
    else {
        // epilogue warps: the rows of this warp's tensor-memory lane quadrant; group c (warps 2 + 4c .. 5 + 4c) takes the
        // 64-column chunks c, c + groups, ... of each 256-wide layer, so the low chunks are published first
        const int e = warp - kFirstEpilogueWarp;
        const int c = e / 4;
        constexpr int kHiddenColumns = kDensity / kChunkGroups;  // this group's columns of h
        static_assert(kHiddenColumns == 32, "the training record keeps h's ReLU mask as one word per chunk group (8 epilogue warps)");
        const int quadrant = warp % 4;
        const int row = 32 * quadrant + lane;
        const int tid = threadIdx.x - 32 * kFirstEpilogueWarp;
        const uint32_t lanes = tmem + (static_cast<uint32_t>(32 * quadrant) << 16);
        uint32_t layer = 0;
        // warp-uniform outcome: the tensor-memory loads that follow need every lane of the warp
        auto accumulator_ready = [&]() -> bool {
#if ZF_MLP_POLL_LANE0
            bool done = true;
            if (lane == 0) done = wait_phase(acc_bar, layer & 1u, abort);
            done = __shfl_sync(0xFFFFFFFFu, done, 0);
#else
            const bool done = __all_sync(0xFFFFFFFFu, wait_phase(acc_bar, layer & 1u, abort));
#endif
            fence_after_sync();
            return done;
        };
        auto publish = [&](const uint32_t bar) {
            fence_async_shared();
            fence_before_sync();
            arrive(bar);
        };
        uint4 next[kInputWords];
        int64_t tile = blockIdx.x;
        if (tile < n_tiles) {
            fetch_inputs(next, tid, features, features_stride, inputs, inputs_stride, tile * kTileRows, n);
            store_inputs(next, tid, act, in);
            publish(in_bar);
        }
        for (; tile < n_tiles && ok; tile += gridDim.x) {
            const int64_t sample = tile * kTileRows + row;
            const bool valid = sample < n;
            const bool more = tile + gridDim.x < n_tiles;
            // E0: h + b_density, ReLU -> this group's columns of h in the inputs (shared and global)
            if (!(ok = accumulator_ready())) break;
            relu_columns<kHiddenColumns, kRecord>(lanes + (layer & 1u) * kRegionColumns + kHiddenColumns * c, bias + kHiddenColumns * c, in, row, kInputs,
                                         kHiddenColumns * c, valid ? inputs + sample * inputs_stride : nullptr,
                                         masks != nullptr && valid ? masks + 3 * n * kMaskWords + sample * kHiddenMaskWords + c : nullptr);
            publish(h_bar);
            layer++;
            // the next tile's inputs, into registers while this tile's layers run
            if (more) fetch_inputs(next, tid, features, features_stride, inputs, inputs_stride, (tile + gridDim.x) * kTileRows, n);
            // E1-E3: v0 (no bias), v1 (+ b_1), v2 (+ b_2) -> act, this group's 64-column chunks
            for (int k = 1; k <= 3 && ok; k++) {
                if (!(ok = accumulator_ready())) break;
                const float* b = k == 1 ? nullptr : bias + kDensity + (k - 2) * kView;
                // the training forward also keeps v0, v1, v2 in global memory for the backward
                uint16_t* kept = activations != nullptr && valid ? activations + (static_cast<int64_t>(k - 1) * n + sample) * kView : nullptr;
                uint32_t* kept_mask = masks != nullptr && valid ? masks + (static_cast<int64_t>(k - 1) * n + sample) * kMaskWords : nullptr;
                for (int j = c; j < kChunks; j += kChunkGroups) {
                    relu_columns<kSlice, kRecord>(lanes + (layer & 1u) * kRegionColumns + kSlice * j, b != nullptr ? b + kSlice * j : nullptr, act, row, kView,
                                         kSlice * j, kept, kept_mask != nullptr ? kept_mask + 2 * j : nullptr);
                    publish(chunk_bar(j));
                }
                layer++;
            }
            if (!ok) break;
            // E4: the outputs (chunk-0 warps), then the next tile's inputs
            if (!(ok = accumulator_ready())) break;
            if (c == 0) {
                float v[8];
                load_columns8(lanes + (layer & 1u) * kRegionColumns, v);
                if (valid) {
                    uint4 out;
                    out.x = pack_bf16x2(v[0], v[1]);
                    out.y = pack_bf16x2(v[2], v[3]);
                    out.z = pack_bf16x2(v[4], v[5]);
                    out.w = pack_bf16x2(v[6], v[7]);
                    *reinterpret_cast<uint4*>(outputs + sample * kOutputs) = out;
                }
            }
            layer++;
            if (more) {
                store_inputs(next, tid, act, in);
                publish(in_bar);
            }
        }
    }

    // teardown: every role has left its loop; on an abort, the MMAs and weight copies already issued finish before the
    // tensor memory is freed
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

// one CTA per SM over the 128-sample tiles; features, inputs, outputs and weights 16-byte aligned, row strides multiples
// of 8 elements
cudaError_t launch_forward(const uint16_t* features, const int64_t features_stride, uint16_t* inputs, const int64_t inputs_stride, const PackedMlp& w,
                           uint16_t* outputs, uint16_t* activations, const int64_t n, int* status, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const auto kernel = activations != nullptr ? fz_nerf_mlp_forward_kernel<true> : fz_nerf_mlp_forward_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    int device = 0, n_sms = 0;
    e = cudaGetDevice(&device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return e;
    const int64_t n_tiles = (n + kTileRows - 1) / kTileRows;
    const unsigned int blocks = static_cast<unsigned int>(n_tiles < n_sms ? n_tiles : n_sms);
    kernel<<<blocks, kThreads, kSmemBytes, stream>>>(features, features_stride, inputs, inputs_stride, w, outputs, activations, n, status);
    return cudaGetLastError();
}

}  // namespace zf::nerf_mlp

int64_t zf_nerf_mlp_activations_size(const int64_t n) {
    using namespace zf::nerf_mlp;
    return n < 0 ? 0 : n * (3 * kView * 2 + 3 * kMaskWords * 4 + kHiddenMaskWords * 4);
}

int zf_nerf_mlp_forward_tc(const uint16_t* features, const int64_t features_stride, uint16_t* inputs, const int64_t inputs_stride,
                           const zf_nerf_mlp_weights* weights, uint16_t* outputs, uint16_t* activations, const int64_t n, int* status,
                           cudaStream_t stream) {
    using namespace zf::nerf_mlp;
    if (n < 0 || weights == nullptr || status == nullptr) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "invalid nerf mlp inputs");
    if (n == 0) return ZF_OK;
    const void* pointers[] = {features, inputs, outputs, weights->density, weights->density_bias, weights->combined, weights->skip,
                              weights->view_1, weights->view_1_bias, weights->view_2, weights->view_2_bias, weights->rgb};
    for (const void* p : pointers) {
        if (p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 != 0) return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "nerf mlp tensors must be 16-byte aligned");
    }
    if (features_stride % 8 != 0 || inputs_stride % 8 != 0 || features_stride < kFeatures || inputs_stride < kInputs) {
        return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "invalid nerf mlp row strides");
    }
    const PackedMlp w{weights->density, weights->density_bias, weights->combined, weights->skip, weights->view_1,
                      weights->view_1_bias, weights->view_2, weights->view_2_bias, weights->rgb};
    if (activations != nullptr && reinterpret_cast<uintptr_t>(activations) % 16 != 0) {
        return zf::set_error(ZF_ERROR_INVALID_ARGUMENT, "nerf mlp activations must be 16-byte aligned");
    }
    const cudaError_t e = launch_forward(features, features_stride, inputs, inputs_stride, w, outputs, activations, n, status, stream);
    return e == cudaSuccess ? ZF_OK : zf::set_cuda_error(e, "nerf mlp forward");
}

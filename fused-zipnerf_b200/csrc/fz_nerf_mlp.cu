// fz_nerf_mlp.cu -- the NeRF MLP forward of one 128-sample tile per CTA on the tcgen05 tensor cores (bf16 operands in
// shared memory, fp32 accumulators in tensor memory), the layer chain of NerfMlp::forward (nerf_mlp.h:35-45):
//   h  = relu(features @ w_density^T + b_density)      -> the first 64 columns of inputs (global) and of the A tile
//   v0 = relu(inputs @ w_combined^T)                    inputs = [h | encoded direction | 1], bias in the bias lane
//   out = inputs @ w_skip^T                             8 outputs, accumulated in tensor memory
//   v1 = relu(v0 @ w_1^T + b_1), v2 = relu(v1 @ w_2^T + b_2)
//   out += v2 @ w_rgb^T
// The activations never leave the SM: each layer's epilogue reads its accumulator rows from tensor memory, applies
// bias and ReLU and writes bf16 back to shared memory as the next layer's A operand.
//
// The weights arrive already in the MMAs' shared-memory order, one bulk copy (cp.async.bulk, no multicast) per tensor
// on a weight mbarrier; the next layer's copy is issued as soon as a layer's MMAs have finished reading the weight
// buffer, so it lands while that layer's epilogue runs. MMAs and epilogues of one CTA still run one after another.
//
// Shared-memory operands use the canonical K-major layout without swizzle: 8-row x 16-byte core matrices stored
// contiguously (128 bytes), K-adjacent core matrices 128 bytes apart (leading byte offset), 8-row groups
// (K / 8) * 128 bytes apart (stride byte offset). Every wait on an mbarrier is bounded; a wait that runs out sets
// *status and the CTA skips to freeing its tensor memory.
#include "zf_mlp.h"
#include "fz_status.h"

#include <cuda_runtime.h>

#include <cstdint>

namespace zf::nerf_mlp {

constexpr int kTileRows = 128;       // M of every MMA: one accumulator row per tensor-memory lane
constexpr int kThreads = 128;        // 4 warps: warp w owns tensor-memory lanes 32w .. 32w + 31
constexpr int kFeatures = 56;        // NeRF features per sample: 10 levels x (4 + 1) = 50, padded to 56
constexpr int kFeaturesK = 64;       // padded to the MMA K step of 16
constexpr int kDensity = 64;         // density width = hidden columns of the inputs
constexpr int kInputs = 96;          // hidden 64 + direction block 32 (its last column the bias lane 1.0)
constexpr int kView = 256;
constexpr int kOutputs = 8;          // raw density, 3 rgb logits, 4 padding
constexpr int kOutputsN = 16;        // the smallest N of an M = 128 MMA
constexpr int kMmaK = 16;            // K of one kind::f16 MMA
constexpr uint32_t kTmemColumns = 512;  // accumulator 0..255, outputs 256..271; allocations are powers of two
constexpr uint32_t kOutColumn = 256;
constexpr uint32_t kWaitLimit = 1u << 22;  // try_wait polls; a layer's MMAs take microseconds

// shared-memory carve-up (bytes)
constexpr int kActBytes = kTileRows * kView * 2;       // 64 KB: features tile, then v0, v1, v2
constexpr int kInBytes = kTileRows * kInputs * 2;      // 24 KB: the inputs tile
constexpr int kWeightBytes = kView * kView * 2;        // 128 KB: one layer's weights (combined and skip together)
constexpr int kSkipOffset = kView * kInputs * 2;       // skip weights behind the combined weights
constexpr int kSmemBytes = kActBytes + kInBytes + kWeightBytes + 32;  // + the MMA and weight mbarriers, the tensor-memory slot
static_assert(kSkipOffset + kOutputsN * kInputs * 2 <= kWeightBytes, "combined and skip weights share one buffer");
static_assert(kSmemBytes <= 227 * 1024, "one CTA per SM");

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

enum Status : int { kOk = 0, kWaitTimeout = 1 };

__device__ __forceinline__ uint32_t smem_address(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// byte offset of element (row, k) of a K-major operand with k_total columns
__host__ __device__ __forceinline__ uint32_t canonical_offset(const int row, const int k, const int k_total) {
    return static_cast<uint32_t>(((row >> 3) * (k_total >> 3) + (k >> 3)) * 128 + (row & 7) * 16 + (k & 7) * 2);
}

// shared-memory matrix descriptor (tcgen05 format): start, leading and stride byte offsets in 16-byte units, version 1
// in bits 46-47, base offset 0, no swizzle (layout type 0 in bits 61-63)
__host__ __device__ __forceinline__ uint64_t smem_descriptor(const uint32_t address, const uint32_t leading_bytes, const uint32_t stride_bytes) {
    uint64_t d = static_cast<uint64_t>((address & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((leading_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((stride_bytes >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    return d;
}

// instruction descriptor of kind::f16: fp32 accumulator (bits 4-5 = 1), bf16 A and B (bits 7-9, 10-12 = 1), both
// K-major (bits 15, 16 = 0), N / 8 in bits 17-22, M / 16 in bits 24-28
__host__ __device__ constexpr uint32_t instr_descriptor(const int m, const int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma(const uint32_t d_tmem, const uint64_t a, const uint64_t b, const uint32_t idesc, const uint32_t accumulate) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// D[128 x n] (+)= A[128 x k] B[n x k]^T from K-major operands, k / 16 MMAs
__device__ __forceinline__ void mma_chain(const uint32_t d_tmem, const uint32_t a_address, const uint32_t b_address, const int n, const int k,
                                          const bool accumulate) {
    const uint32_t idesc = instr_descriptor(kTileRows, n);
    const uint32_t stride = static_cast<uint32_t>(k >> 3) * 128;
    for (int s = 0; s < k / kMmaK; s++) {
        // one K step covers two core matrices: start at chunk 2s, the second chunk one leading offset further
        const uint32_t step = static_cast<uint32_t>(2 * s) * 128;
        mma(d_tmem, smem_descriptor(a_address + step, 128, stride), smem_descriptor(b_address + step, 128, stride), idesc,
            (accumulate || s > 0) ? 1u : 0u);
    }
}

__device__ __forceinline__ void commit(const uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// bounded wait for the given phase parity; false if the limit ran out
__device__ __forceinline__ bool wait_phase(const uint32_t bar, const uint32_t parity) {
    for (uint32_t i = 0; i < kWaitLimit; i++) {
        uint32_t done;
        asm volatile(
            "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// generic-proxy shared-memory writes become visible to the tensor cores' reads
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 consecutive fp32 accumulator columns of this thread's lane
__device__ __forceinline__ void load_columns(const uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, "
        "%19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]),
          "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
          "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void load_columns8(const uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t pack_bf16x2(const float lo, const float hi) {
    uint32_t out;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(out) : "f"(hi), "f"(lo));
    return out;
}

// the weight mbarrier expects `bytes` more bytes in its current phase (the arrival of its one thread)
__device__ __forceinline__ void expect_bytes(const uint32_t bar, const uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// one bulk copy (no multicast) of a weight stored in the canonical order in global memory into shared memory, completing
// on the weight mbarrier; addresses 16-byte aligned, bytes a multiple of 16
__device__ __forceinline__ void bulk_copy(const uint32_t dst, const void* src, const uint32_t bytes, const uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst), "l"(src), "r"(bytes),
                 "r"(bar)
                 : "memory");
}

// this thread's accumulator row (columns 0 .. width - 1) + bias, ReLU, bf16 into row `row` of a K-major operand
template <int kWidth>
__device__ __forceinline__ void relu_epilogue(const uint32_t tmem_row, const float* __restrict__ bias, uint8_t* dst, const int row, const int k_total,
                                              const int k_first) {
    for (int c = 0; c < kWidth; c += 32) {
        float v[32];
        load_columns(tmem_row + static_cast<uint32_t>(c), v);
        for (int j = 0; j < 32; j += 8) {
            uint4 out;
            uint32_t* words = reinterpret_cast<uint32_t*>(&out);
            for (int q = 0; q < 4; q++) {
                float lo = v[j + 2 * q], hi = v[j + 2 * q + 1];
                if (bias != nullptr) {
                    lo += __ldg(bias + c + j + 2 * q);
                    hi += __ldg(bias + c + j + 2 * q + 1);
                }
                words[q] = pack_bf16x2(fmaxf(lo, 0.0f), fmaxf(hi, 0.0f));
            }
            *reinterpret_cast<uint4*>(dst + canonical_offset(row, k_first + c + j, k_total)) = out;
        }
    }
}

// features [n, 56] bf16 (row stride features_stride), inputs [n, 96] bf16 (row stride inputs_stride; the direction
// block in columns 64-95 is read, the hidden layer written to columns 0-63), outputs [n, 8] bf16
__global__ void __launch_bounds__(kThreads, 1)
    fz_nerf_mlp_forward_kernel(const uint16_t* __restrict__ features, const int64_t features_stride, uint16_t* __restrict__ inputs,
                               const int64_t inputs_stride, const PackedMlp w, uint16_t* __restrict__ outputs, const int64_t n, int* status) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* act = smem;
    uint8_t* in = smem + kActBytes;
    uint8_t* weights = in + kInBytes;
    uint64_t* bar = reinterpret_cast<uint64_t*>(weights + kWeightBytes);  // MMA completion
    uint64_t* wbar = bar + 1;                                                // weight copies landed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 2);
    const int warp = threadIdx.x / 32;
    const int row = threadIdx.x;  // accumulator row = tensor-memory lane of this thread
    const int64_t first = static_cast<int64_t>(blockIdx.x) * kTileRows;
    const int64_t sample = first + row;
    const bool valid = sample < n;
    const uint32_t bar_address = smem_address(bar), wbar_address = smem_address(wbar), weights_address = smem_address(weights);

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_address(tmem_slot)), "r"(kTmemColumns));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar_address), "r"(1));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(wbar_address), "r"(1));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        expect_bytes(wbar_address, kDensity * kFeaturesK * 2);
        bulk_copy(weights_address, w.density, kDensity * kFeaturesK * 2, wbar_address);
    }

    // features (56 columns + 8 zero columns) into act, the direction block into columns 64-95 of in, density weights
    for (int q = threadIdx.x; q < kTileRows * (kFeaturesK / 8); q += kThreads) {
        const int r = q / (kFeaturesK / 8), c = q % (kFeaturesK / 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (first + r < n && c < kFeatures / 8) v = __ldg(reinterpret_cast<const uint4*>(features + (first + r) * features_stride) + c);
        *reinterpret_cast<uint4*>(act + canonical_offset(r, 8 * c, kFeaturesK)) = v;
    }
    for (int q = threadIdx.x; q < kTileRows * 4; q += kThreads) {
        const int r = q / 4, c = q % 4;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (first + r < n) v = __ldg(reinterpret_cast<const uint4*>(inputs + (first + r) * inputs_stride + kDensity) + c);
        *reinterpret_cast<uint4*>(in + canonical_offset(r, kDensity + 8 * c, kInputs)) = v;
    }
    fence_async_shared();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tmem_row = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    uint32_t parity = 0, wparity = 0;
    bool ok = true;  // the same in every thread: each wait's outcome is combined over the block
    ok = __syncthreads_and(wait_phase(wbar_address, wparity));
    wparity ^= 1;
    if (!ok) goto done;

    // layer 0: h = relu(features @ w_density^T + b_density)
    if (threadIdx.x == 0) {
        mma_chain(tmem, smem_address(act), smem_address(weights), kDensity, kFeaturesK, false);
        commit(bar_address);
    }
    ok = __syncthreads_and(wait_phase(bar_address, parity));
    parity ^= 1;
    if (!ok) goto done;
    fence_after_sync();
    if (threadIdx.x == 0) {  // the weight buffer is free: the next layer's weights arrive during this epilogue
        expect_bytes(wbar_address, (kView + kOutputsN) * kInputs * 2);
        bulk_copy(weights_address, w.combined, kView * kInputs * 2, wbar_address);
        bulk_copy(weights_address + kSkipOffset, w.skip, kOutputsN * kInputs * 2, wbar_address);
    }
    relu_epilogue<kDensity>(tmem_row, w.density_bias, in, row, kInputs, 0);
    if (valid) {  // the hidden layer is part of the inputs the backward reads
        for (int c = 0; c < kDensity / 8; c++) {
            *reinterpret_cast<uint4*>(inputs + sample * inputs_stride + 8 * c) = *reinterpret_cast<const uint4*>(in + canonical_offset(row, 8 * c, kInputs));
        }
    }
    fence_async_shared();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    ok = __syncthreads_and(wait_phase(wbar_address, wparity));
    wparity ^= 1;
    if (!ok) goto done;

    // layer 1: v0 = relu(inputs @ w_combined^T); outputs = inputs @ w_skip^T
    if (threadIdx.x == 0) {
        mma_chain(tmem, smem_address(in), smem_address(weights), kView, kInputs, false);
        mma_chain(tmem + kOutColumn, smem_address(in), smem_address(weights + kSkipOffset), kOutputsN, kInputs, false);
        commit(bar_address);
    }
    ok = __syncthreads_and(wait_phase(bar_address, parity));
    parity ^= 1;
    if (!ok) goto done;
    fence_after_sync();
    if (threadIdx.x == 0) {
        expect_bytes(wbar_address, kView * kView * 2);
        bulk_copy(weights_address, w.view_1, kView * kView * 2, wbar_address);
    }
    relu_epilogue<kView>(tmem_row, nullptr, act, row, kView, 0);
    fence_async_shared();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    ok = __syncthreads_and(wait_phase(wbar_address, wparity));
    wparity ^= 1;
    if (!ok) goto done;

    // layer 2: v1 = relu(v0 @ w_1^T + b_1)
    if (threadIdx.x == 0) {
        mma_chain(tmem, smem_address(act), smem_address(weights), kView, kView, false);
        commit(bar_address);
    }
    ok = __syncthreads_and(wait_phase(bar_address, parity));
    parity ^= 1;
    if (!ok) goto done;
    fence_after_sync();
    if (threadIdx.x == 0) {
        expect_bytes(wbar_address, kView * kView * 2);
        bulk_copy(weights_address, w.view_2, kView * kView * 2, wbar_address);
    }
    relu_epilogue<kView>(tmem_row, w.view_1_bias, act, row, kView, 0);
    fence_async_shared();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    ok = __syncthreads_and(wait_phase(wbar_address, wparity));
    wparity ^= 1;
    if (!ok) goto done;

    // layer 3: v2 = relu(v1 @ w_2^T + b_2)
    if (threadIdx.x == 0) {
        mma_chain(tmem, smem_address(act), smem_address(weights), kView, kView, false);
        commit(bar_address);
    }
    ok = __syncthreads_and(wait_phase(bar_address, parity));
    parity ^= 1;
    if (!ok) goto done;
    fence_after_sync();
    if (threadIdx.x == 0) {
        expect_bytes(wbar_address, kOutputsN * kView * 2);
        bulk_copy(weights_address, w.rgb, kOutputsN * kView * 2, wbar_address);
    }
    relu_epilogue<kView>(tmem_row, w.view_2_bias, act, row, kView, 0);
    fence_async_shared();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    ok = __syncthreads_and(wait_phase(wbar_address, wparity));
    wparity ^= 1;
    if (!ok) goto done;

    // layer 4: outputs += v2 @ w_rgb^T
    if (threadIdx.x == 0) {
        mma_chain(tmem + kOutColumn, smem_address(act), smem_address(weights), kOutputsN, kView, true);
        commit(bar_address);
    }
    ok = __syncthreads_and(wait_phase(bar_address, parity));
    if (!ok) goto done;
    fence_after_sync();
    {
        float v[8];
        load_columns8(tmem_row + kOutColumn, v);
        if (valid) {
            uint4 out;
            out.x = pack_bf16x2(v[0], v[1]);
            out.y = pack_bf16x2(v[2], v[3]);
            out.z = pack_bf16x2(v[4], v[5]);
            out.w = pack_bf16x2(v[6], v[7]);
            *reinterpret_cast<uint4*>(outputs + sample * kOutputs) = out;
        }
    }

done:
    if (!ok && threadIdx.x == 0) atomicExch(status, kWaitTimeout);
    fence_before_sync();
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemColumns));
}

// one CTA per 128 samples; features, inputs, outputs and weights 16-byte aligned, row strides multiples of 8 elements
cudaError_t launch_forward(const uint16_t* features, const int64_t features_stride, uint16_t* inputs, const int64_t inputs_stride, const PackedMlp& w,
                           uint16_t* outputs, const int64_t n, int* status, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(fz_nerf_mlp_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    const unsigned int blocks = static_cast<unsigned int>((n + kTileRows - 1) / kTileRows);
    fz_nerf_mlp_forward_kernel<<<blocks, kThreads, kSmemBytes, stream>>>(features, features_stride, inputs, inputs_stride, w, outputs, n, status);
    return cudaGetLastError();
}

}  // namespace zf::nerf_mlp

int zf_nerf_mlp_forward_tc(const uint16_t* features, const int64_t features_stride, uint16_t* inputs, const int64_t inputs_stride,
                           const zf_nerf_mlp_weights* weights, uint16_t* outputs, const int64_t n, int* status, cudaStream_t stream) {
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
    const cudaError_t e = launch_forward(features, features_stride, inputs, inputs_stride, w, outputs, n, status, stream);
    return e == cudaSuccess ? ZF_OK : zf::set_cuda_error(e, "nerf mlp forward");
}

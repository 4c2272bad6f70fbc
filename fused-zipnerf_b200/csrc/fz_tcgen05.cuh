// fz_tcgen05.cuh -- the tcgen05 building blocks of the NeRF MLP kernels (forward and backward): shared-memory matrix and
// instruction descriptors, MMA chains over operands in the canonical no-swizzle layouts, tensor-memory loads, mbarrier
// waits with a time bound, bulk copies of packed weights (no multicast).
//
// Canonical K-major layout without swizzle: 8-row x 16-byte core matrices stored contiguously (128 bytes), K-adjacent
// core matrices 128 bytes apart, 8-row groups (K / 8) * 128 bytes apart, K the operand's stored width.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace zf::nerf_mlp {

constexpr int kTileRows = 128;       // M of every MMA: one accumulator row per tensor-memory lane
constexpr int kMmaK = 16;            // K of one kind::f16 MMA
// bounded waits: a waiting thread is suspended in mbarrier.try_wait for up to kSuspendNs at a time (woken when the phase
// completes), and gives up after kWaitNs in total; a layer takes microseconds
constexpr uint32_t kSuspendNs = 20000;
constexpr uint64_t kWaitNs = 2000000000ull;

enum Status : int { kOk = 0, kWaitTimeout = 1 };

__device__ __forceinline__ uint32_t smem_address(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// byte offset of element (row, k) of a K-major operand with k_total columns
__host__ __device__ __forceinline__ uint32_t canonical_offset(const int row, const int k, const int k_total) {
    return static_cast<uint32_t>(((row >> 3) * (k_total >> 3) + (k >> 3)) * 128 + (row & 7) * 16 + (k & 7) * 2);
}

// shared-memory matrix descriptor (tcgen05 format): start, leading and stride byte offsets in 16-byte units, version 1
// in bits 46-47, base offset 0, the layout type in bits 61-63 (0: no swizzle, 2: 128-byte swizzle, 6: 32-byte swizzle)
__host__ __device__ __forceinline__ uint64_t smem_descriptor(const uint32_t address, const uint32_t leading_bytes, const uint32_t stride_bytes,
                                                             const uint32_t layout = 0) {
    uint64_t d = static_cast<uint64_t>((address & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((leading_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((stride_bytes >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(layout & 7u) << 61;
    return d;
}

// MN-major tiles of `rows` K rows as TMA writes them: with the 128-byte swizzle, 64-column atoms rows * 128 bytes apart
// (leading offset) and 8-row K groups 1024 bytes apart (stride offset); with the 32-byte swizzle one 16-column atom,
// 8-row K groups 256 bytes apart
__host__ __device__ __forceinline__ uint64_t mn_sw128_descriptor(const uint32_t address, const uint32_t rows) {
    return smem_descriptor(address, rows * 128, 1024, 2);
}
__host__ __device__ __forceinline__ uint64_t mn_sw32_descriptor(const uint32_t address) { return smem_descriptor(address, 0, 256, 6); }

// instruction descriptor of kind::f16: fp32 accumulator (bits 4-5 = 1), bf16 A and B (bits 7-9, 10-12 = 1), A and B
// K-major (bits 15, 16 = 0) or MN-major (= 1), N / 8 in bits 17-22, M / 16 in bits 24-28
__host__ __device__ constexpr uint32_t instr_descriptor(const int m, const int n, const bool a_mn = false, const bool b_mn = false) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (a_mn ? 1u << 15 : 0u) | (b_mn ? 1u << 16 : 0u) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma(const uint32_t d_tmem, const uint64_t a, const uint64_t b, const uint32_t idesc, const uint32_t accumulate) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// D[128 x n] (+)= A[128 x k] B[n x k]^T from K-major operands stored with a_k_total and b_k_total columns, k / 16 MMAs
__device__ __forceinline__ void mma_chain(const uint32_t d_tmem, const uint32_t a_address, const int a_k_total, const uint32_t b_address,
                                          const int b_k_total, const int n, const int k, const bool accumulate) {
    const uint32_t idesc = instr_descriptor(kTileRows, n);
    const uint32_t a_stride = static_cast<uint32_t>(a_k_total >> 3) * 128, b_stride = static_cast<uint32_t>(b_k_total >> 3) * 128;
    for (int s = 0; s < k / kMmaK; s++) {
        // one K step covers two core matrices: start at chunk 2s, the second chunk one leading offset further
        const uint32_t step = static_cast<uint32_t>(2 * s) * 128;
        mma(d_tmem, smem_descriptor(a_address + step, 128, a_stride), smem_descriptor(b_address + step, 128, b_stride), idesc,
            (accumulate || s > 0) ? 1u : 0u);
    }
}

// the mbarrier tracks the completion of every tcgen05 operation this thread has issued so far
__device__ __forceinline__ void commit(const uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// whether the phase with the given parity has completed; the thread may be suspended (up to kSuspendNs) until it does
__device__ __forceinline__ bool try_wait(const uint32_t bar, const uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(kSuspendNs)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// bounded wait for the completion of the phase with the given parity; false if the CTA's abort flag went up or the
// time limit ran out (which raises the flag)
__device__ __forceinline__ bool wait_phase(const uint32_t bar, const uint32_t parity, volatile int* abort) {
    if (try_wait(bar, parity)) return true;
    const uint64_t start = global_ns();
    while (true) {
        if (try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (global_ns() - start > kWaitNs) break;
    }
    *abort = 1;
    return false;
}

// bounded wait that ignores the abort flag (the teardown's wait for work already in flight)
__device__ __forceinline__ void drain_phase(const uint32_t bar, const uint32_t parity) {
    const uint64_t start = global_ns();
    while (!try_wait(bar, parity) && global_ns() - start <= kWaitNs) {
    }
}

__device__ __forceinline__ void arrive(const uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
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

// round to bf16 pairs with negative values (ReLU) set to zero
__device__ __forceinline__ uint32_t pack_bf16x2_relu(const float lo, const float hi) {
    uint32_t out;
    asm("cvt.rn.relu.bf16x2.f32 %0, %1, %2;" : "=r"(out) : "f"(hi), "f"(lo));
    return out;
}

// the mbarrier expects `bytes` more bytes in its current phase (the arrival of its one thread)
__device__ __forceinline__ void expect_bytes(const uint32_t bar, const uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// one bulk copy (no multicast) of packed weights from global into shared memory, completing on the mbarrier; addresses
// 16-byte aligned, bytes a multiple of 16
__device__ __forceinline__ void bulk_copy(const uint32_t dst, const void* src, const uint32_t bytes, const uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst), "l"(src), "r"(bytes),
                 "r"(bar)
                 : "memory");
}

// tcgen05.ld of N (16 or 32) consecutive fp32 accumulator columns of this thread's lane into r (no wait)
template <int N>
__device__ __forceinline__ void issue_load(const uint32_t taddr, uint32_t* r) {
    if constexpr (N == 16) {
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]),
              "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
            : "r"(taddr));
    }
    else {
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, "
            "%19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]),
              "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
              "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
              "=r"(r[31])
            : "r"(taddr));
    }
}

}  // namespace zf::nerf_mlp

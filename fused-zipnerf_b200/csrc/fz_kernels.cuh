// fz_kernels.cuh -- featurization kernels: forward (optionally with the fused density MLP), NeRF-level backward, and
// proposal-level backward with the MLP recomputation.
//
// The reference compiles one kernel per grid at runtime with the layout, level count and feature count as constants
// (featurizer.cu:157-184). Here kernels are compiled ahead of time for sm_100a, templated only on the features per level
// F (and, with the MLP, on the MLP input width rounded up to a multiple of 4); the level loop runs over the layout in
// the kernel parameters, with one level's multisample / corner / gather body unrolled. Per-thread feature rows are
// staged in shared memory, so outputs leave the SM as coalesced warp-wide stores.
#pragma once

#include <type_traits>

#include "fz_device.cuh"

namespace zf {

constexpr int kBlock = 128;
// minimum resident blocks per SM each kernel's register allocation must allow (__launch_bounds__), from sweeps on the
// B200: the kernels are latency bound and gain from resident warps up to where registers spill or shared memory runs
// out (the cooperative forward and the scatter: shared memory for 6 blocks; the MLP kernel: 2 blocks of 256 threads;
// the per-lane forward of 3-4 features: 6, 7 with its MLP)
#ifndef ZF_MIN_BLOCKS_FORWARD
#define ZF_MIN_BLOCKS_FORWARD 6
#endif
#ifndef ZF_MIN_BLOCKS_FORWARD_MLP
#define ZF_MIN_BLOCKS_FORWARD_MLP 7
#endif
// the cooperative forward (1-2 features per level): its shared memory allows 6 blocks per SM
#ifndef ZF_MIN_BLOCKS_FORWARD_COOP
#define ZF_MIN_BLOCKS_FORWARD_COOP 6
#endif
#ifndef ZF_MIN_BLOCKS_BACKWARD
#define ZF_MIN_BLOCKS_BACKWARD 6
#endif
#ifndef ZF_MIN_BLOCKS_BACKWARD_MLP
#define ZF_MIN_BLOCKS_BACKWARD_MLP 2
#endif
constexpr int kWarps = kBlock / 32;

// odd row stride (in floats) of per-thread rows in shared memory: lanes writing the same column hit distinct banks
__host__ __device__ constexpr int staged_stride(const int n_out) { return n_out | 1; }
// n (a multiple of 4) or n + 4: an odd number of 16-byte words, so the 16-byte accesses of 8 consecutive lanes to rows
// of this stride fall into distinct bank quads
__host__ __device__ constexpr int odd_quads(const int n) { return (n / 4) % 2 == 1 ? n : n + 4; }

// ---------------------------------------------------------------------------------------------------------------------
// forward

struct ForwardArgs {
    RayInputs in;
    const float* table;             // [rows, F]
    const float* scale_magnitudes;  // [L]
    const float* w0;                // [W, n_out]
    const float* b0;                // [W]
    const float* w1;                // [W]
    const float* b1;                // [1]
    int mlp_width;
    float* raw_density;             // [n_samples] or null (requires the MLP)
    float* features_float;          // [n_samples, n_out] or null
    uint16_t* features_bf16;        // [n_samples, features_bf16_width] or null
    int features_bf16_width;
    const uint16_t* encoded_directions;  // [n_rays, encoded_width]
    uint16_t* nerf_inputs;          // [n_samples, nerf_inputs_width] or null (last encoded_width columns written)
    int nerf_inputs_width;
    int encoded_width;
    uint32_t interleave_rays;       // 0: consecutive threads take consecutive samples; else the same interval of this many rays
    uint32_t level_begin;           // the levels of this launch (a pass; without the MLP a forward may take several)
    uint32_t level_end;
    bool bf16_pairs;                // features_bf16 allows 4-byte (pair) stores: even width, 4-byte aligned
    bool inputs_vectors;            // nerf_inputs / encoded_directions allow 16-byte copies
    bool w0_vectors;                // w0 rows allow 16-byte loads: 16-byte aligned, n_out a multiple of 4
};

template <int F>
struct GatherRows {
    const float* table;
    float value[F];

    __device__ __forceinline__ void operator()(const uint32_t row, const float weight) {
        if (weight == 0.0f) return;
        // fused multiply-adds, as the reference's feature gather (featurize_common.cuh:179-198)
        if constexpr (F == 4) {
            const float4 t = __ldg(reinterpret_cast<const float4*>(table) + row);
            value[0] = __fmaf_rn(weight, t.x, value[0]);
            value[1] = __fmaf_rn(weight, t.y, value[1]);
            value[2] = __fmaf_rn(weight, t.z, value[2]);
            value[3] = __fmaf_rn(weight, t.w, value[3]);
        }
        else if constexpr (F == 2) {
            const float2 t = __ldg(reinterpret_cast<const float2*>(table) + row);
            value[0] = __fmaf_rn(weight, t.x, value[0]);
            value[1] = __fmaf_rn(weight, t.y, value[1]);
        }
        else {
            #pragma unroll
            for (int f = 0; f < F; f++) value[f] = __fmaf_rn(weight, __ldg(table + row * F + f), value[f]);
        }
    }
};

// sample of a thread: consecutive samples, or (interleave) the same interval of up to R consecutive rays per warp run
// (featurize_forward.cu:49-58)
__device__ __forceinline__ uint32_t thread_sample(const uint32_t t, const RayInputs& in, const uint32_t interleave_rays) {
    if (interleave_rays == 0) return t;
    const uint32_t n = in.n_intervals;
    const uint32_t group = t / (interleave_rays * n), offset = t % (interleave_rays * n);
    const uint32_t group_rays = min(interleave_rays, in.n_samples / n - interleave_rays * group);
    return (interleave_rays * group + offset % group_rays) * n + offset / group_rays;
}

__device__ __forceinline__ void multisamples(const Frustum& fr, float3 (&x)[kMultisamples], float (&scale)[kMultisamples]) {
    #pragma unroll
    for (uint32_t j = 0; j < kMultisamples; j++) multisample(fr, j, x[j], scale[j]);
}

// ---------------------------------------------------------------------------------------------------------------------
// warp-cooperative corner groups (featurize_common.cuh:123-198)
//
// The corner work of an interval is one task per merged corner group, 1 to 6 per level. A lane that loops over its own
// groups keeps the warp busy for the largest group count of its 32 intervals (coarse levels: one group for most
// intervals, several for a few), and pays for selecting its group's leader out of registers. Here every lane publishes
// its multisample records of the level to shared memory and lists its groups in the warp's task list; the warp then
// works through the list 32 tasks at a time, each lane taking whichever group comes next. The merged corner weights
// are formed exactly as in visit_level (the leader's weights, then the other members' in multisample order). Tasks are
// listed group-index-major (every lane's first group, then every lane's second group, ...), so a lane's groups come in
// its own order, which the forward's accumulation needs.

// Per-warp records of the current level, cells packed into 16-bit fields (exact for cells in [-1, 65534], i.e. level
// sizes up to kMaxPackedSize), which keeps the kernels' shared memory within 6 blocks per SM. Lane-major records (the
// scatter's lane-major task lists, where neighbouring lanes read one lane's groups) sit at [l 7 + j]: with stride 7 the
// 16-byte records of 8 consecutive lanes fall into distinct bank quads. Multisample-major records (the forward's
// group-major task lists, where neighbouring lanes read different lanes' records) sit at [j 32 + l].
constexpr int kRecordStride = 7;
constexpr uint32_t kMaxPackedSize = 65534;
struct PackedRecords {
    float4 frac[kMultisamples * 32];   // (fx, fy, fz, weighting) of every multisample
    uint2 cell[kMultisamples * 32];    // (cx + 1 | (cy + 1) << 16, cz + 1 | member mask << 16) of every group leader
    uint8_t task[32 * kMultisamples];  // one byte per group: owner lane | leader multisample << 5

    static __device__ __forceinline__ int at(const uint32_t lane, const uint32_t j) { return static_cast<int>(j * 32 + lane); }
    __device__ __forceinline__ void put_cell(const int i, const int cx, const int cy, const int cz, const uint32_t members) {
        cell[i] = make_uint2((static_cast<uint32_t>(cx + 1) & 0xFFFFu) | (static_cast<uint32_t>(cy + 1) << 16),
                             (static_cast<uint32_t>(cz + 1) & 0xFFFFu) | (members << 16));
    }
    __device__ __forceinline__ int4 get_cell(const int i) const {
        const uint2 c = cell[i];
        return make_int4(static_cast<int>(c.x & 0xFFFFu) - 1, static_cast<int>(c.x >> 16) - 1, static_cast<int>(c.y & 0xFFFFu) - 1,
                         static_cast<int>(c.y >> 16));
    }
};
// lane-major records with packed cells (the scatter of 1-2 features per level)
struct LaneMajorPackedRecords {
    float4 frac[32 * kRecordStride];
    uint2 cell[32 * kRecordStride];
    uint8_t task[32 * kMultisamples];

    static __device__ __forceinline__ int at(const uint32_t lane, const uint32_t j) { return static_cast<int>(lane * kRecordStride + j); }
    __device__ __forceinline__ void put_cell(const int i, const int cx, const int cy, const int cz, const uint32_t members) {
        cell[i] = make_uint2((static_cast<uint32_t>(cx + 1) & 0xFFFFu) | (static_cast<uint32_t>(cy + 1) << 16),
                             (static_cast<uint32_t>(cz + 1) & 0xFFFFu) | (members << 16));
    }
    __device__ __forceinline__ int4 get_cell(const int i) const {
        const uint2 c = cell[i];
        return make_int4(static_cast<int>(c.x & 0xFFFFu) - 1, static_cast<int>(c.x >> 16) - 1, static_cast<int>(c.y & 0xFFFFu) - 1,
                         static_cast<int>(c.y >> 16));
    }
};
static_assert(sizeof(PackedRecords) % 16 == 0 && sizeof(LaneMajorPackedRecords) % 16 == 0, "records stay 16-byte aligned per warp");
// the scatter's records: lane-major with packed cells (level sizes up to kMaxPackedSize)
using ScatterRecords = LaneMajorPackedRecords;

// a warp's staged feature gradients, row r, column c: fp32 rows already scaled, or bf16 bits scaled on reading by
// feature_scale * grad_scale (the product first, as the reference's feature_scale * grad_scale * g,
// featurize_backward.cu:24)
template <typename T>
struct StagedRows {
    const T* rows;
    int stride;
    float scale;
    __device__ __forceinline__ float operator()(const uint32_t r, const int c) const {
        if constexpr (std::is_same_v<T, float>) return rows[r * stride + c];
        else return scale * bf16_bits_to_f32(rows[r * stride + c]);
    }
};

// writes one interval's multisample records of a level; returns the mask of group leaders (the lowest multisample of
// every set of multisamples that share a cell)
template <typename Records>
__device__ __forceinline__ uint32_t publish_level(const uint32_t size, const float3* x, const float* weighting, Records& gr, const int lane) {
    int cx[kMultisamples], cy[kMultisamples], cz[kMultisamples];
    #pragma unroll
    for (uint32_t j = 0; j < kMultisamples; j++) {
        float fx, fy, fz;
        level_cell(x[j].x, size, cx[j], fx);
        level_cell(x[j].y, size, cy[j], fy);
        level_cell(x[j].z, size, cz[j], fz);
        gr.frac[Records::at(lane, j)] = make_float4(fx, fy, fz, weighting[j]);
    }
    uint32_t members[kMultisamples];
    uint32_t followers = 0u;
    #pragma unroll
    for (uint32_t j = 0; j < kMultisamples; j++) members[j] = 1u << j;
    #pragma unroll
    for (uint32_t j = 0; j < kMultisamples; j++) {
        #pragma unroll
        for (uint32_t k = j + 1; k < kMultisamples; k++) {
            if (cx[j] == cx[k] && cy[j] == cy[k] && cz[j] == cz[k]) {
                members[j] |= 1u << k;
                followers |= 1u << k;
            }
        }
    }
    const uint32_t leaders = ((1u << kMultisamples) - 1u) & ~followers;
    #pragma unroll
    for (uint32_t j = 0; j < kMultisamples; j++) {
        if ((leaders >> j) & 1u) gr.put_cell(Records::at(lane, j), cx[j], cy[j], cz[j], members[j]);
    }
    return leaders;
}

// lists the groups of every lane, group-index-major; slot[i] = the task index of this lane's i-th group (for i below
// its group count). Returns the warp's task count. Every lane of the warp must call this.
template <typename Records>
__device__ __forceinline__ uint32_t list_tasks(const uint32_t leaders, const int lane, Records& gr, uint32_t (&slot)[kMultisamples]) {
    const uint32_t lanes_below = (1u << lane) - 1u;
    const uint32_t n = __popc(leaders);
    uint32_t base = 0u, rest = leaders;
    #pragma unroll
    for (uint32_t i = 0; i < kMultisamples; i++) slot[i] = 0u;
    #pragma unroll
    for (uint32_t i = 0; i < kMultisamples; i++) {
        const uint32_t mask = __ballot_sync(0xFFFFFFFFu, n > i);
        if (mask == 0u) break;  // no lane has an i-th group (warp-uniform)
        slot[i] = base + __popc(mask & lanes_below);
        if (n > i) {
            gr.task[slot[i]] = static_cast<uint8_t>(lane | ((__ffs(rest) - 1) << 5));
            rest &= rest - 1u;
        }
        base += __popc(mask);
    }
    return base;
}

// lists the groups of every lane, lane-major (a lane's groups next to each other: the lanes of a round then touch the
// corners of fewer distinct intervals at a time, so fewer of a warp's atomics hit the same row). Returns the warp's
// task count. Every lane of the warp must call this.
template <typename Records>
__device__ __forceinline__ uint32_t list_tasks_by_lane(const uint32_t leaders, const int lane, Records& gr) {
    const uint32_t lanes_below = (1u << lane) - 1u;
    const uint32_t n = __popc(leaders);
    // this lane's first slot: exclusive prefix of the 0..6 group counts, one ballot per count bit
    uint32_t first = 0u, n_tasks = 0u;
    #pragma unroll
    for (int b = 0; b < 3; b++) {
        const uint32_t bits = __ballot_sync(0xFFFFFFFFu, (n >> b) & 1u);
        first += static_cast<uint32_t>(__popc(bits & lanes_below)) << b;
        n_tasks += static_cast<uint32_t>(__popc(bits)) << b;
    }
    #pragma unroll
    for (uint32_t j = 0; j < kMultisamples; j++) {
        if ((leaders >> j) & 1u) gr.task[first + __popc(leaders & ((1u << j) - 1u))] = static_cast<uint8_t>(lane | (j << 5));
    }
    return n_tasks;
}

// merged corner weights and cell of task t's group
template <typename Records>
__device__ __forceinline__ void task_group(const Records& gr, const uint32_t t, float (&corner_weights)[8], int4& cell, uint32_t& owner) {
    const uint32_t task = gr.task[t];
    owner = task & 31u;
    const uint32_t leader = task >> 5;
    const float4 q = gr.frac[Records::at(owner, leader)];
    cell = gr.get_cell(Records::at(owner, leader));
    #pragma unroll
    for (uint32_t corner = 0; corner < 8; corner++) {
        const float wx = corner & 4u ? q.x : 1.0f - q.x;
        const float wy = corner & 2u ? q.y : 1.0f - q.y;
        const float wz = corner & 1u ? q.z : 1.0f - q.z;
        corner_weights[corner] = __fmaf_rn(q.w, __fmul_rn(__fmul_rn(wx, wy), wz), 0.0f);
    }
    uint32_t others = static_cast<uint32_t>(cell.w) & ~(1u << leader);
    while (others != 0u) {
        const uint32_t m = __ffs(others) - 1u;
        others &= others - 1u;
        const float4 qm = gr.frac[Records::at(owner, m)];
        #pragma unroll
        for (uint32_t corner = 0; corner < 8; corner++) {
            const float wx = corner & 4u ? qm.x : 1.0f - qm.x;
            const float wy = corner & 2u ? qm.y : 1.0f - qm.y;
            const float wz = corner & 1u ? qm.z : 1.0f - qm.z;
            corner_weights[corner] = __fmaf_rn(qm.w, __fmul_rn(__fmul_rn(wx, wy), wz), corner_weights[corner]);
        }
    }
}


template <int F>
__device__ __forceinline__ void load_row(const float* __restrict__ table, const uint32_t row, float (&v)[F]) {
    if constexpr (F == 4) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(table) + row);
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    }
    else if constexpr (F == 2) {
        const float2 t = __ldg(reinterpret_cast<const float2*>(table) + row);
        v[0] = t.x; v[1] = t.y;
    }
    else {
        #pragma unroll
        for (int f = 0; f < F; f++) v[f] = __ldg(table + static_cast<size_t>(row) * F + f);
    }
}

// floats per warp of the forward's per-round gather results: (weight, F values) of 8 corners for 32 tasks
template <int F>
__host__ __device__ constexpr int gather_result_floats() { return 32 * 8 * (F + 1); }

// The forward gathers cooperatively for 1-2 features per level. With more, the per-warp records and results take the
// shared memory that the latency-bound gathers of wide hashed tables need for resident warps (measured on the B200 for
// 4 features: 2 instead of 6 blocks per SM, 2.3x slower), and each lane loops over its own groups (visit_level).
__host__ __device__ constexpr bool cooperative_forward(const int n_features) { return n_features <= 2; }

// all level features of a warp's intervals into their shared-memory rows (lane l's row: row[l (F + 1) + f] grid
// features, row[l (F + 1) + F] the scale feature; featurize_common.cuh:174-227). A round's tasks gather their 8 corner
// rows into s_result (component-major, lane-minor); then every owner accumulates its tasks of the round, in its own
// group order, corner by corner, with the fused multiply-adds of the reference's gather, so the features are the
// reference's bit for bit. Every lane of the warp must call this; inactive lanes add no tasks and write no row.
template <int F>
__device__ __forceinline__ void featurize_warp(const GridParams& gp, const Frustum& fr, const bool active, const float* __restrict__ table,
                                               const float* __restrict__ scale_magnitudes, float* row, const int lane, PackedRecords& gr,
                                               float* s_result, const uint32_t level_begin, const uint32_t level_end) {
    float3 x[kMultisamples];
    float scale[kMultisamples];
    if (active) multisamples(fr, x, scale);
    #pragma unroll 1
    for (uint32_t level = level_begin; level < level_end; level++) {
        const uint32_t size = gp.size[level];
        float scale_feature = 0.0f;
        uint32_t leaders = 0u;
        if (active) {
            float weighting[kMultisamples];
            #pragma unroll
            for (uint32_t j = 0; j < kMultisamples; j++) {
                weighting[j] = level_weighting(size, scale[j]);
                scale_feature += 2.0f * weighting[j] - 1.0f;
            }
            leaders = publish_level(size, x, weighting, gr, lane);
        }
        uint32_t slot[kMultisamples];
        const uint32_t n_tasks = list_tasks(leaders, lane, gr, slot);
        const uint32_t n_groups = __popc(leaders);
        __syncwarp();
        float value[F];
        #pragma unroll
        for (int f = 0; f < F; f++) value[f] = 0.0f;
        for (uint32_t first = 0; first < n_tasks; first += 32) {
            const uint32_t t = first + lane;
            if (t < n_tasks) {
                float w[8];
                int4 c;
                uint32_t owner;
                task_group(gr, t, w, c, owner);
                float v[8][F];
                uint32_t rows[8];
                cell_rows(gp, level, c.x, c.y, c.z, rows, w);
                #pragma unroll
                for (uint32_t corner = 0; corner < 8; corner++) {
                    if (w[corner] != 0.0f) load_row<F>(table, rows[corner], v[corner]);
                    else {
                        #pragma unroll
                        for (int f = 0; f < F; f++) v[corner][f] = 0.0f;
                    }
                }
                #pragma unroll
                for (uint32_t corner = 0; corner < 8; corner++) {
                    if constexpr (F == 1) {
                        reinterpret_cast<float2*>(s_result)[corner * 32 + lane] = make_float2(w[corner], v[corner][0]);
                    }
                    else {
                        s_result[(corner * (F + 1)) * 32 + lane] = w[corner];
                        #pragma unroll
                        for (int f = 0; f < F; f++) s_result[(corner * (F + 1) + 1 + f) * 32 + lane] = v[corner][f];
                    }
                }
            }
            __syncwarp();
            #pragma unroll
            for (uint32_t i = 0; i < kMultisamples; i++) {
                const uint32_t src = slot[i] - first;
                if (i < n_groups && src < 32u) {
                    #pragma unroll
                    for (uint32_t corner = 0; corner < 8; corner++) {
                        if constexpr (F == 1) {
                            const float2 wv = reinterpret_cast<const float2*>(s_result)[corner * 32 + src];
                            if (wv.x != 0.0f) value[0] = __fmaf_rn(wv.x, wv.y, value[0]);
                        }
                        else {
                            const float weight = s_result[(corner * (F + 1)) * 32 + src];
                            if (weight != 0.0f) {
                                #pragma unroll
                                for (int f = 0; f < F; f++) value[f] = __fmaf_rn(weight, s_result[(corner * (F + 1) + 1 + f) * 32 + src], value[f]);
                            }
                        }
                    }
                }
            }
            __syncwarp();
        }
        if (active) {
            #pragma unroll
            for (int f = 0; f < F; f++) row[level * (F + 1) + f] = kFeatureScale * value[f];
            row[level * (F + 1) + F] = kFeatureScale * scale_feature * __ldg(scale_magnitudes + level);
        }
    }
}

// all level features of one interval into a shared-memory row: row[l (F + 1) + f] grid features (averaged over the
// multisamples and preconditioned), row[l (F + 1) + F] the scale feature (featurize_common.cuh:207-227)
template <int F>
__device__ __forceinline__ void featurize_to_row(const GridParams& gp, const Frustum& fr, const float* __restrict__ table,
                                                 const float* __restrict__ scale_magnitudes, float* row, const uint32_t level_begin,
                                                 const uint32_t level_end) {
    float3 x[kMultisamples];
    float scale[kMultisamples];
    multisamples(fr, x, scale);
    #pragma unroll 1
    for (uint32_t level = level_begin; level < level_end; level++) {
        float weighting[kMultisamples];
        float scale_feature = 0.0f;
        #pragma unroll
        for (uint32_t j = 0; j < kMultisamples; j++) {
            weighting[j] = level_weighting(gp.size[level], scale[j]);
            scale_feature += 2.0f * weighting[j] - 1.0f;
        }
        GatherRows<F> gather{table, {}};
        #pragma unroll
        for (int f = 0; f < F; f++) gather.value[f] = 0.0f;
        visit_level(gp, level, x, weighting, gather);
        #pragma unroll
        for (int f = 0; f < F; f++) row[level * (F + 1) + f] = kFeatureScale * gather.value[f];
        row[level * (F + 1) + F] = kFeatureScale * scale_feature * __ldg(scale_magnitudes + level);
    }
}

// (row, column) of the elements e = first, first + step, ... of a row-major [rows, cols] block (step 32: a warp's
// lanes, kBlock: a block's threads), advanced without a division per element
struct LaneWalk {
    int r, c, dr, dc, cols;
    __device__ __forceinline__ LaneWalk(const int first, const int n_cols, const int step = 32) : cols(n_cols) {
        r = first / n_cols;
        c = first - r * n_cols;
        dr = step / n_cols;
        dc = step - dr * n_cols;
    }
    __device__ __forceinline__ void next() {
        r += dr;
        c += dc;
        if (c >= cols) {
            c -= cols;
            r++;
        }
    }
};

// warp-cooperative copy of the warp's staged rows to row-major global outputs (rows of samples s_sample[...]); the
// outputs are written once and read by a later kernel, so they are stored with the evict-first (streaming) policy
// and do not push the grid tables out of L2
// (columns [c0, c1) of the rows: a pass writes the columns of its levels; columns at or past n_out are zero padding)
__device__ __forceinline__ void store_rows_float(const float* s_rows, const int stride, const uint32_t* s_sample, const int n_rows, const int n_out,
                                                 const int c0, const int c1, float* __restrict__ out, const int lane) {
    for (LaneWalk w(lane, c1 - c0); w.r < n_rows; w.next()) {
        const int c = c0 + w.c;
        __stcs(out + static_cast<size_t>(s_sample[w.r]) * n_out + c, s_rows[w.r * stride + c]);
    }
}

__device__ __forceinline__ void store_rows_bf16(const float* s_rows, const int stride, const uint32_t* s_sample, const int n_rows, const int n_out,
                                                const int c0, const int c1, uint16_t* __restrict__ out, const int width, const bool pairs, const int lane) {
    auto bits = [&](const int r, const int c) -> uint32_t { return c < n_out ? f32_to_bf16_bits(s_rows[r * stride + c]) : 0u; };
    if (pairs) {
        // 4-byte column pairs; a pair half outside [c0, c1) belongs to another pass and is not written
        const int p0 = c0 / 2;
        for (LaneWalk w(lane, (c1 + 1) / 2 - p0); w.r < n_rows; w.next()) {
            const int r = w.r, c = 2 * (p0 + w.c);
            uint16_t* row = out + static_cast<size_t>(s_sample[r]) * width;
            if (c >= c0 && c + 1 < c1) __stcs(reinterpret_cast<unsigned int*>(row + c), bits(r, c) | (bits(r, c + 1) << 16));
            else if (c >= c0) __stcs(row + c, static_cast<unsigned short>(bits(r, c)));
            else __stcs(row + c + 1, static_cast<unsigned short>(bits(r, c + 1)));
        }
    }
    else {
        for (LaneWalk w(lane, c1 - c0); w.r < n_rows; w.next()) {
            const int c = c0 + w.c;
            __stcs(out + static_cast<size_t>(s_sample[w.r]) * width + c, static_cast<unsigned short>(bits(w.r, c)));
        }
    }
}

// the encoded view direction in the last columns of the NeRF MLP inputs, its last column the bias lane (bf16 1.0)
// (featurize_forward.cu:86-92)
template <typename Args>
__device__ __forceinline__ void store_inputs_tail(const Args& a, const uint32_t* s_sample, const int n_rows, const int lane) {
    const int E = a.encoded_width;
    if (a.inputs_vectors) {
        const int nv = E / 8;
        for (LaneWalk w(lane, nv); w.r < n_rows; w.next()) {
            const int r = w.r, v = w.c;
            const uint32_t sample = s_sample[r];
            const uint4* src = reinterpret_cast<const uint4*>(a.encoded_directions + static_cast<size_t>(sample / a.in.n_intervals) * E);
            uint4 value = __ldg(src + v);
            if (v == nv - 1) value.w = (value.w & 0x0000FFFFu) | 0x3f800000u;
            __stcs(reinterpret_cast<uint4*>(a.nerf_inputs + static_cast<size_t>(sample + 1) * a.nerf_inputs_width - E) + v, value);
        }
    }
    else {
        for (LaneWalk w(lane, E); w.r < n_rows; w.next()) {
            const int r = w.r, c = w.c;
            const uint32_t sample = s_sample[r];
            const uint16_t value = c == E - 1 ? static_cast<uint16_t>(0x3f80) : a.encoded_directions[static_cast<size_t>(sample / a.in.n_intervals) * E + c];
            __stcs(a.nerf_inputs + static_cast<size_t>(sample + 1) * a.nerf_inputs_width - E + c, value);
        }
    }
}

// staged-row stride of the forward: the cooperative forward's rows are read as 16-byte words by its MLP (a multiple of
// 4 with an odd word count); the per-lane forward writes its rows column by column (odd)
__host__ __device__ constexpr int forward_row_stride(const int n_features, const int n_out) {
    return cooperative_forward(n_features) ? odd_quads((n_out + 3) / 4 * 4) : staged_stride(n_out);
}

// Forward. NOUT_PAD == 0: no MLP; otherwise the fused density MLP n_out -> W (ReLU) -> 1 runs for raw_density, with
// the features in registers (NOUT_PAD >= n_out) and the reference's accumulation order (featurize_forward.cu:65-73);
// its weights are read through the L1 (every lane reads the same row).
template <int F, int NOUT_PAD>
__global__ void __launch_bounds__(kBlock, cooperative_forward(F) ? ZF_MIN_BLOCKS_FORWARD_COOP : (NOUT_PAD > 0 ? ZF_MIN_BLOCKS_FORWARD_MLP : ZF_MIN_BLOCKS_FORWARD)) fz_forward_kernel(const __grid_constant__ GridParams gp, const __grid_constant__ ForwardArgs a) {
    const int n_out = static_cast<int>(gp.n_levels) * (F + 1);
    const int stride = forward_row_stride(F, n_out);
    extern __shared__ __align__(16) float smem[];
    float* s_rows = smem;                                      // [kBlock, stride]
    // the cooperative forward: the warps' group records and gather results (16-byte aligned); the per-lane forward: the
    // threads' sample indices
    PackedRecords* s_groups = reinterpret_cast<PackedRecords*>(smem + kBlock * stride);
    float* s_results = reinterpret_cast<float*>(s_groups + kWarps);  // [kWarps, gather_result_floats<F>()]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // the warp's sample indices for the output stores (the cooperative forward keeps them in its gather results, which
    // are free once the levels are done)
    uint32_t* warp_samples = cooperative_forward(F) ? reinterpret_cast<uint32_t*>(s_results + warp * gather_result_floats<F>())
                                                    : reinterpret_cast<uint32_t*>(smem + kBlock * stride) + warp * 32;
    const uint32_t warp_first = blockIdx.x * kBlock + warp * 32;
    if (warp_first >= a.in.n_samples) return;
    const int n_rows = min(32, static_cast<int>(a.in.n_samples - warp_first));
    const bool active = lane < n_rows;
    const uint32_t sample = active ? thread_sample(warp_first + lane, a.in, a.interleave_rays) : 0u;
    float* row = s_rows + threadIdx.x * stride;
    if constexpr (cooperative_forward(F)) {
        Frustum fr;
        if (active) fr = setup_frustum(a.in, gp.pattern_stream, sample);
        featurize_warp<F>(gp, fr, active, a.table, a.scale_magnitudes, row, lane, s_groups[warp], s_results + warp * gather_result_floats<F>(),
                          a.level_begin, a.level_end);
        __syncwarp();
        warp_samples[lane] = sample;
    }
    else {
        warp_samples[lane] = sample;
        if (active) {
            const Frustum fr = setup_frustum(a.in, gp.pattern_stream, sample);
            featurize_to_row<F>(gp, fr, a.table, a.scale_magnitudes, row, a.level_begin, a.level_end);
        }
    }
    if constexpr (NOUT_PAD > 0) {
        if (active) {
            float f[NOUT_PAD];
            if constexpr (cooperative_forward(F)) {
                #pragma unroll
                for (int q = 0; q < NOUT_PAD / 4; q++) {
                    const float4 v = reinterpret_cast<const float4*>(row)[q];
                    f[4 * q] = v.x;
                    f[4 * q + 1] = v.y;
                    f[4 * q + 2] = v.z;
                    f[4 * q + 3] = v.w;
                }
                #pragma unroll
                for (int i = 0; i < NOUT_PAD; i++) f[i] = i < n_out ? f[i] : 0.0f;
            }
            else {
                #pragma unroll
                for (int i = 0; i < NOUT_PAD; i++) f[i] = i < n_out ? row[i] : 0.0f;
            }
            float raw = __ldg(a.b1);
            if (a.w0_vectors) {
                // two hidden units at a time: independent chains in the reference's input order, added to raw in unit
                // order
                int j = 0;
                for (; j + 1 < a.mlp_width; j += 2) {
                    float pre0 = __ldg(a.b0 + j), pre1 = __ldg(a.b0 + j + 1);
                    const float4* w = reinterpret_cast<const float4*>(a.w0 + j * n_out);
                    const float4* v = reinterpret_cast<const float4*>(a.w0 + (j + 1) * n_out);
                    #pragma unroll
                    for (int q = 0; q < NOUT_PAD / 4; q++) {
                        const float4 wq = __ldg(w + q), vq = __ldg(v + q);
                        pre0 = __fmaf_rn(wq.x, f[4 * q], pre0);
                        pre1 = __fmaf_rn(vq.x, f[4 * q], pre1);
                        pre0 = __fmaf_rn(wq.y, f[4 * q + 1], pre0);
                        pre1 = __fmaf_rn(vq.y, f[4 * q + 1], pre1);
                        pre0 = __fmaf_rn(wq.z, f[4 * q + 2], pre0);
                        pre1 = __fmaf_rn(vq.z, f[4 * q + 2], pre1);
                        pre0 = __fmaf_rn(wq.w, f[4 * q + 3], pre0);
                        pre1 = __fmaf_rn(vq.w, f[4 * q + 3], pre1);
                    }
                    raw = __fmaf_rn(__ldg(a.w1 + j), fmaxf(pre0, 0.0f), raw);
                    raw = __fmaf_rn(__ldg(a.w1 + j + 1), fmaxf(pre1, 0.0f), raw);
                }
                for (; j < a.mlp_width; j++) {
                    float pre = __ldg(a.b0 + j);
                    const float4* w = reinterpret_cast<const float4*>(a.w0 + j * n_out);
                    #pragma unroll
                    for (int q = 0; q < NOUT_PAD / 4; q++) {
                        const float4 wq = __ldg(w + q);
                        pre = __fmaf_rn(wq.x, f[4 * q], pre);
                        pre = __fmaf_rn(wq.y, f[4 * q + 1], pre);
                        pre = __fmaf_rn(wq.z, f[4 * q + 2], pre);
                        pre = __fmaf_rn(wq.w, f[4 * q + 3], pre);
                    }
                    raw = __fmaf_rn(__ldg(a.w1 + j), fmaxf(pre, 0.0f), raw);
                }
            }
            else {
                for (int j = 0; j < a.mlp_width; j++) {
                    float pre = __ldg(a.b0 + j);
                    #pragma unroll
                    for (int i = 0; i < NOUT_PAD; i++) {
                        if (i < n_out) pre = __fmaf_rn(__ldg(a.w0 + j * n_out + i), f[i], pre);
                    }
                    raw = __fmaf_rn(__ldg(a.w1 + j), fmaxf(pre, 0.0f), raw);
                }
            }
            __stcs(a.raw_density + sample, raw);
        }
    }
    __syncwarp();
    const float* warp_rows = s_rows + warp * 32 * stride;
    // this pass's columns; the last pass also writes the zero padding of the bf16 rows and the NeRF-input tail
    const bool last_pass = a.level_end == gp.n_levels;
    const int c0 = static_cast<int>(a.level_begin) * (F + 1), c1 = static_cast<int>(a.level_end) * (F + 1);
    if (a.features_float != nullptr) store_rows_float(warp_rows, stride, warp_samples, n_rows, n_out, c0, c1, a.features_float, lane);
    if (a.features_bf16 != nullptr) {
        store_rows_bf16(warp_rows, stride, warp_samples, n_rows, n_out, c0, last_pass ? static_cast<int>(a.features_bf16_width) : c1, a.features_bf16,
                        a.features_bf16_width, a.bf16_pairs, lane);
    }
    if (a.nerf_inputs != nullptr && last_pass) store_inputs_tail(a, warp_samples, n_rows, lane);
}

// dynamic shared memory of fz_forward_kernel in floats: staged rows, then the cooperative forward's group records and
// gather results (16-byte aligned), or the per-lane forward's sample indices
__host__ __device__ constexpr int forward_smem_floats(const int n_out, const int n_features) {
    return kBlock * forward_row_stride(n_features, n_out) +
           (cooperative_forward(n_features) ? kWarps * (static_cast<int>(sizeof(PackedRecords) / sizeof(float)) + 32 * 8 * (n_features + 1)) : kBlock);
}

// ---------------------------------------------------------------------------------------------------------------------
// row gradient atomics (featurize_common.cuh:230-268)

template <int F>
__device__ __forceinline__ void add_row_f32(float* __restrict__ grad_table, const uint32_t row, const float weight, const float* g) {
    float* p = grad_table + static_cast<size_t>(row) * F;
    if constexpr (F == 4) {
        asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" :: "l"(p), "f"(weight * g[0]), "f"(weight * g[1]),
                     "f"(weight * g[2]), "f"(weight * g[3]) : "memory");
    }
    else {
        #pragma unroll
        for (int f = 0; f < F; f++) {
            if (g[f] != 0.0f) atomicAdd(p + f, weight * g[f]);
        }
    }
}

template <int F>
__device__ __forceinline__ void add_row_f16(uint16_t* __restrict__ grad_table, const uint32_t row, const float weight, const float* g) {
    uint16_t* p = grad_table + static_cast<size_t>(row) * F;
    if constexpr (F == 4) {
        const uint32_t p0 = pack_half2(weight * g[0], weight * g[1]);
        const uint32_t p1 = pack_half2(weight * g[2], weight * g[3]);
        asm volatile("red.global.add.noftz.v2.f16x2 [%0], {%1, %2};" :: "l"(p), "r"(p0), "r"(p1) : "memory");
    }
    else if constexpr (F % 2 == 0) {
        #pragma unroll
        for (int q = 0; q < F / 2; q++) {
            const uint32_t pair = pack_half2(weight * g[2 * q], weight * g[2 * q + 1]);
            asm volatile("red.global.add.noftz.f16x2 [%0], %1;" :: "l"(p + 2 * q), "r"(pair) : "memory");
        }
    }
    else {
        #pragma unroll
        for (int f = 0; f < F; f++) {
            if (g[f] != 0.0f) asm volatile("red.global.add.noftz.f16 [%0], %1;" :: "l"(p + f), "h"(f32_to_half_bits(weight * g[f])) : "memory");
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------------
// warp-cooperative gradient scatter (featurize_common.cuh:123-173, 273-291): the corner groups of a warp's intervals as
// one task list (above); the atomics are order-free

// Runs of tasks with the same cell in consecutive lanes are common on coarse levels, where neighbouring intervals of a
// ray share cells; one atomic per run and corner instead of per lane keeps the L2 atomic units from serialising on a few
// hot rows (how much that costs otherwise depends on where the table's rows fall among the L2 slices: up to 1.2 ms per
// proposal backward at 65,536 rays on a B200). A round takes this path when at least kMinRunLanes of its 32 lanes
// continue a run (swept 4-28: fewer pays the scan on rounds that gain little, more leaves hot rows unmerged).
constexpr int kMinRunLanes = 20;

// inclusive sums of v over the lanes from run_start to this lane (a segmented scan)
template <int F>
__device__ __forceinline__ void sum_run(float (&v)[F], const int lane, const int run_start) {
    #pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        #pragma unroll
        for (int f = 0; f < F; f++) {
            const float y = __shfl_up_sync(0xFFFFFFFFu, v[f], d);
            if (lane - d >= run_start) v[f] += y;
        }
    }
}

// works through the warp's task list of one level: merged corner weights of each group, its 8 rows, and the atomics of
// the owner's gradient (fp32 table, or fp16 table with rows re-based at row_base). fp32 contributions of runs of equal
// cells are summed over the run first; fp16 contributions are always rounded and added one by one, as the reference
// does.
template <int F, bool HALF, typename Rows>
__device__ __forceinline__ void scatter_tasks(const GridParams& gp, const uint32_t level, const uint32_t level_begin, const ScatterRecords& gr,
                                              const uint32_t n_tasks, const int lane, const Rows& staged, float* __restrict__ grad_table,
                                              uint16_t* __restrict__ grad_table_half, const uint32_t row_base) {
    for (uint32_t first = 0; first < n_tasks; first += 32) {
        const bool valid = first + lane < n_tasks;
        float weights[8];
        uint32_t rows[8];
        float g[F];
        int4 c = make_int4(0, 0, 0, 0);
        if (valid) {
            uint32_t owner;
            task_group(gr, first + lane, weights, c, owner);
            #pragma unroll
            for (int f = 0; f < F; f++) g[f] = staged(owner, static_cast<int>(level - level_begin) * (F + 1) + f);
            cell_rows(gp, level, c.x, c.y, c.z, rows, weights);
        }
        else {
            #pragma unroll
            for (uint32_t corner = 0; corner < 8; corner++) {
                weights[corner] = 0.0f;
                rows[corner] = 0u;
            }
            #pragma unroll
            for (int f = 0; f < F; f++) g[f] = 0.0f;
        }
        if constexpr (!HALF) {
            // lanes that continue the run of the lane before them (same cell; every lane takes part in the shuffles)
            const int lx = __shfl_up_sync(0xFFFFFFFFu, c.x, 1), ly = __shfl_up_sync(0xFFFFFFFFu, c.y, 1), lz = __shfl_up_sync(0xFFFFFFFFu, c.z, 1);
            const bool continues = valid && lane > 0 && lx == c.x && ly == c.y && lz == c.z;
            const uint32_t continuing = __ballot_sync(0xFFFFFFFFu, continues);
            if (__popc(continuing) >= kMinRunLanes) {
                const uint32_t heads = ~continuing;
                const int run_start = 31 - __clz(heads & (0xFFFFFFFFu >> (31 - lane)));
                const bool run_end = lane == 31 || !((continuing >> (lane + 1)) & 1u);
                #pragma unroll
                for (uint32_t corner = 0; corner < 8; corner++) {
                    float v[F];
                    #pragma unroll
                    for (int f = 0; f < F; f++) v[f] = weights[corner] != 0.0f ? weights[corner] * g[f] : 0.0f;
                    sum_run<F>(v, lane, run_start);
                    bool any = false;
                    #pragma unroll
                    for (int f = 0; f < F; f++) any |= v[f] != 0.0f;
                    if (valid && run_end && any) add_row_f32<F>(grad_table, rows[corner], 1.0f, v);
                }
                continue;
            }
        }
        if (valid) {
            #pragma unroll
            for (uint32_t corner = 0; corner < 8; corner++) {
                if (weights[corner] == 0.0f) continue;
                if constexpr (HALF) add_row_f16<F>(grad_table_half, rows[corner] - row_base, weights[corner], g);
                else add_row_f32<F>(grad_table, rows[corner], weights[corner], g);
            }
        }
    }
}

// scatters the feature gradients of levels [level_begin, level_end) of a warp's intervals (row of lane l at
// warp_rows[l stride], column (level - level_begin) (F + 1) + f; scale features carry none) into the grid gradient:
// levels below n_fp32 into grad_table (fp32), the others into grad_table_half (fp16, rows re-based at the first fp16
// level). Inactive lanes and all-zero level gradients add no tasks. Every lane of the warp must call this.
template <int F, typename Rows>
__device__ __forceinline__ void scatter_warp(const GridParams& gp, const Frustum& fr, const bool active, const Rows& staged, const int lane,
                                             const uint32_t n_fp32, float* __restrict__ grad_table, uint16_t* __restrict__ grad_table_half,
                                             ScatterRecords& gr, const uint32_t level_begin, const uint32_t level_end) {
    float3 x[kMultisamples];
    float scale[kMultisamples];
    if (active) multisamples(fr, x, scale);
    const uint32_t half_base = gp.offset[min(n_fp32, gp.n_levels)];
    #pragma unroll 1
    for (uint32_t level = level_begin; level < level_end; level++) {
        const uint32_t size = gp.size[level];
        uint32_t leaders = 0u;
        if (active) {
            bool any = false;
            #pragma unroll
            for (int f = 0; f < F; f++) any |= staged(static_cast<uint32_t>(lane), static_cast<int>(level - level_begin) * (F + 1) + f) != 0.0f;
            if (any) {
                float weighting[kMultisamples];
                #pragma unroll
                for (uint32_t j = 0; j < kMultisamples; j++) weighting[j] = level_weighting(size, scale[j]);
                leaders = publish_level(size, x, weighting, gr, lane);
            }
        }
        const uint32_t n_tasks = list_tasks_by_lane(leaders, lane, gr);
        __syncwarp();
        if (level < n_fp32) scatter_tasks<F, false>(gp, level, level_begin, gr, n_tasks, lane, staged, grad_table, grad_table_half, 0u);
        else scatter_tasks<F, true>(gp, level, level_begin, gr, n_tasks, lane, staged, grad_table, grad_table_half, half_base);
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------------------------------------------------
// NeRF-level backward: bf16 feature gradients -> grid gradient scaled by grad_scale (featurize_backward.cu:19-26)

struct BackwardArgs {
    RayInputs in;
    const uint16_t* grad_features;  // bf16 [n_samples, >= n_out], row stride grad_stride (NeRF level)
    long long grad_stride;
    float grad_scale;
    const float* grad_rows;         // or: fp32 [n_samples, n_out] feature gradients, already scaled (proposal levels)
    const float* skip_if_zero;      // optional [n_samples]: samples whose value is 0 are not scattered
    uint32_t n_fp32_levels;         // leading levels scattered into grad_table (fp32), the rest into grad_table_half
    float* grad_table;              // fp32 [n_fp32_rows, F]
    uint16_t* grad_table_half;      // fp16 [rows - n_fp32_rows, F]
    uint32_t level_begin;           // the levels of this launch (a pass)
    uint32_t level_end;
};

template <int F>
__global__ void __launch_bounds__(kBlock, ZF_MIN_BLOCKS_BACKWARD) fz_backward_kernel(const __grid_constant__ GridParams gp, const __grid_constant__ BackwardArgs a) {
    const int n_out = static_cast<int>(gp.n_levels) * (F + 1);
    // the columns of this pass's levels
    const int c0 = static_cast<int>(a.level_begin) * (F + 1), n_cols = static_cast<int>(a.level_end - a.level_begin) * (F + 1);
    const int stride = staged_stride(n_cols);
    extern __shared__ __align__(16) float smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t warp_first = blockIdx.x * kBlock + warp * 32;
    if (warp_first >= a.in.n_samples) return;
    const int n_rows = min(32, static_cast<int>(a.in.n_samples - warp_first));
    // the warps' group records, then the gradient rows of this pass's columns (fp32 or bf16, as given)
    ScatterRecords& gr = reinterpret_cast<ScatterRecords*>(smem)[warp];
    unsigned char* rows_base = reinterpret_cast<unsigned char*>(smem) + kWarps * sizeof(ScatterRecords);
    const uint32_t sample = warp_first + lane;
    bool active = lane < n_rows;
    if (active && a.skip_if_zero != nullptr && __ldcs(a.skip_if_zero + sample) == 0.0f) active = false;
    Frustum fr;
    if (active) fr = setup_frustum(a.in, gp.pattern_stream, sample);
    // coalesced load of the warp's gradient rows
    if (a.grad_rows != nullptr) {
        float* warp_rows = reinterpret_cast<float*>(rows_base) + warp * 32 * stride;
        for (LaneWalk w(lane, n_cols); w.r < n_rows; w.next()) {
            warp_rows[w.r * stride + w.c] = __ldcs(a.grad_rows + static_cast<size_t>(warp_first + w.r) * n_out + c0 + w.c);
        }
        __syncwarp();
        scatter_warp<F>(gp, fr, active, StagedRows<float>{warp_rows, stride, 1.0f}, lane, a.n_fp32_levels, a.grad_table, a.grad_table_half, gr,
                        a.level_begin, a.level_end);
    }
    else {
        uint16_t* warp_rows = reinterpret_cast<uint16_t*>(rows_base) + warp * 32 * stride;
        for (LaneWalk w(lane, n_cols); w.r < n_rows; w.next()) {
            warp_rows[w.r * stride + w.c] = __ldcs(a.grad_features + static_cast<size_t>(warp_first + w.r) * a.grad_stride + c0 + w.c);
        }
        __syncwarp();
        scatter_warp<F>(gp, fr, active, StagedRows<uint16_t>{warp_rows, stride, kFeatureScale * a.grad_scale}, lane, a.n_fp32_levels, a.grad_table,
                        a.grad_table_half, gr, a.level_begin, a.level_end);
    }
}

// dynamic shared memory of fz_backward_kernel in bytes for passes of at most n_cols gradient columns of row_bytes each
// (4: fp32 rows, 2: bf16 rows): the warps' scatter records, then the staged gradient rows
__host__ __device__ constexpr int backward_smem_bytes(const int n_cols, const int row_bytes) {
    return kWarps * static_cast<int>(sizeof(ScatterRecords)) + kBlock * staged_stride(n_cols) * row_bytes;
}

// ---------------------------------------------------------------------------------------------------------------------
// proposal-level backward, MLP part (featurize_backward_mlp.cu:79-147 without the scatter): recomputes the fused MLP
// from the stored fp32 features, writes the scaled input gradient of every sample to grad_rows (the scatter kernel
// adds it to the grid gradient), and reduces the MLP parameter gradients
//
// with a_j = [pre_j > 0] g: grad_w0[j][i] = w1_j sum a_j f_i, grad_b0[j] = w1_j sum a_j, grad_w1[j] = sum g relu(pre_j),
// grad_b1 = sum g

struct BackwardMlpArgs {
    RayInputs in;
    const float* features;          // [n_samples, n_out]
    const float* grad_raw_density;  // [n_samples]
    const float* w0;                // [W, n_out]
    const float* b0;                // [W]
    const float* w1;                // [W]
    int mlp_width;
    float* grad_rows;               // out: [n_samples, n_out] feature gradients times feature_scale
    float* grad_w0;
    float* grad_b0;
    float* grad_w1;
    float* grad_b1;
};

// The kernel runs warps independently: each takes 32 samples at a time (a chunk) through
//   phase 1 (lane = sample): the MLP recomputation in the forward's accumulation order (the same ReLU mask as the
//           forward), its input gradient (written to grad_rows) and the pre-activations (to shared memory), then
//   phase 2 (lane = 4-row tiles of grad_w0, with the row sums of grad_b0 and grad_w1): the chunk's sums in sample
//           order, added to the block's sums with shared-memory atomics.
// Chunk rows in shared memory have a stride of an odd number of 16-byte words, so the lanes' 16-byte stores of phase 1
// are bank-conflict free, and phase 2 reads one row (broadcast) per sample.
#ifndef ZF_MLP_WARPS
#define ZF_MLP_WARPS 8
#endif
// Paired fp32 arithmetic (sm_100): two lanes' worth of fused multiply-adds or adds in one instruction, each element
// rounded as the scalar fma.rn / add.rn with flush-to-zero (what __fmaf_rn and __fadd_rn are under --use_fast_math), so
// a pair of sequential chains gives the scalar chains' results bit for bit.
__device__ __forceinline__ uint64_t pair_of(const float lo, const float hi) {
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
    return d;
}
__device__ __forceinline__ float2 split_pair(const uint64_t d) {
    float2 v;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(d));
    return v;
}
__device__ __forceinline__ uint64_t fma_pair(const uint64_t a, const uint64_t b, const uint64_t c) {
    uint64_t d;
    asm("fma.rn.ftz.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t add_pair(const uint64_t a, const uint64_t b) {
    uint64_t d;
    asm("add.rn.ftz.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

constexpr int kMlpWarps = ZF_MLP_WARPS;
constexpr int kMlpBlock = 32 * kMlpWarps;
// hidden units padded to whole steps of the recomputation (kMlpChains pairs; zero weights and bias beyond the width)
constexpr int kMlpChains = 4;
__host__ __device__ constexpr int mlp_rows_pad(const int width) { return (width + 2 * kMlpChains - 1) / (2 * kMlpChains) * (2 * kMlpChains); }
__host__ __device__ constexpr int mlp_block_floats(const int n_out, const int nout_pad, const int width) {
    return mlp_rows_pad(width) * nout_pad + 2 * mlp_rows_pad(width)                  // weights (w0 rows padded to nout_pad), b0, w1
        + (n_out * (mlp_rows_pad(width) + 1) + 2 * width + 1 + 3) / 4 * 4            // the block's parameter gradient sums
        + mlp_rows_pad(width) * nout_pad;                                             // w0 with row pairs interleaved
}
__host__ __device__ constexpr int mlp_warp_floats(const int nout_pad, const int width) {
    return 32 * odd_quads(mlp_rows_pad(width)) + 32 * odd_quads(nout_pad) + 32;  // pre-activations, features, upstream gradient
}
__host__ __device__ constexpr int backward_mlp_smem_floats(const int n_out, const int nout_pad, const int width) {
    return mlp_block_floats(n_out, nout_pad, width) + kMlpWarps * mlp_warp_floats(nout_pad, width);
}

template <int F, int NOUT_PAD>
__global__ void __launch_bounds__(kMlpBlock, ZF_MIN_BLOCKS_BACKWARD_MLP) fz_backward_mlp_kernel(const __grid_constant__ GridParams gp, const __grid_constant__ BackwardMlpArgs a) {
    const int n_out = static_cast<int>(gp.n_levels) * (F + 1);
    const int W = a.mlp_width;
    const int w_pad = mlp_rows_pad(W);
    const int n_w0 = W * n_out;
    const int n_params = n_w0 + 2 * W + 1;
    const int ps = odd_quads(w_pad), fs = odd_quads(NOUT_PAD);
    extern __shared__ __align__(16) float smem[];
    float* s_w0 = smem;                        // [w_pad, NOUT_PAD]
    float* s_b0 = s_w0 + w_pad * NOUT_PAD;     // [w_pad]
    float* s_w1 = s_b0 + w_pad;                // [w_pad]
    // the block's sums: grad_w0 column-major [n_out][w_pad + 1] (the lanes' shared-memory atomics of one tile entry
    // then fall on distinct banks, but for pairs), then grad_b0 [W], grad_w1 [W], grad_b1
    float* s_acc = s_w1 + w_pad;
    const int acc_stride = w_pad + 1;
    const int acc_b0 = n_out * acc_stride, acc_w1 = acc_b0 + W, acc_b1 = acc_w1 + W, n_acc = acc_b1 + 1;
    // w0 again with rows 2 k and 2 k + 1 interleaved: element (j, i) at (j / 2) 2 NOUT_PAD + 2 i + j % 2, so one float4
    // holds two rows' weights of two consecutive inputs (the paired forward recomputation)
    float* s_w0p = smem + mlp_block_floats(n_out, NOUT_PAD, W) - w_pad * NOUT_PAD;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float* s_pre = smem + mlp_block_floats(n_out, NOUT_PAD, W) + warp * mlp_warp_floats(NOUT_PAD, W);  // [32, ps]
    float* s_feat = s_pre + 32 * ps;           // [32, fs]
    float* s_g = s_feat + 32 * fs;             // [32]
    // padding rows (j >= W) and columns (i >= n_out) are zero: their pre-activations are 0 and select no gradient
    for (int i = threadIdx.x; i < w_pad * NOUT_PAD; i += kMlpBlock) {
        const int j = i / NOUT_PAD, c = i - j * NOUT_PAD;
        const float w = j < W && c < n_out ? __ldg(a.w0 + j * n_out + c) : 0.0f;
        s_w0[i] = w;
        s_w0p[(j / 2) * 2 * NOUT_PAD + 2 * c + (j % 2)] = w;
    }
    for (int i = threadIdx.x; i < w_pad; i += kMlpBlock) {
        s_b0[i] = i < W ? __ldg(a.b0 + i) : 0.0f;
        s_w1[i] = i < W ? __ldg(a.w1 + i) : 0.0f;
    }
    for (int i = threadIdx.x; i < n_acc; i += kMlpBlock) s_acc[i] = 0.0f;
    for (int i = lane; i < 32 * fs; i += 32) s_feat[i] = 0.0f;
    __syncthreads();
    // grad_w0 tiles of 4 rows x TI columns: half the padded inputs up to 24 (a 64-wide MLP then gives every lane one
    // tile), else 4
    constexpr int TI = NOUT_PAD <= 24 ? NOUT_PAD / 2 : 4;
    constexpr int n_itiles = NOUT_PAD / TI;
    const int n_tiles = (w_pad / 4) * n_itiles;
    const bool vector_rows = n_out % 4 == 0;

    // warp-uniform loop bound
    for (uint32_t base = (blockIdx.x * kMlpWarps + warp) * 32u; base < a.in.n_samples; base += gridDim.x * kMlpBlock) {
        const int n_rows = min(32, static_cast<int>(a.in.n_samples - base));
        // the chunk's features (coalesced) and upstream gradients
        for (LaneWalk w(lane, n_out); w.r < n_rows; w.next()) s_feat[w.r * fs + w.c] = __ldcs(a.features + static_cast<size_t>(base + w.r) * n_out + w.c);
        s_g[lane] = lane < n_rows ? __ldcs(a.grad_raw_density + base + lane) : 0.0f;
        {
            // L2 prefetch of this warp's next chunk (its feature rows, 128 bytes per lane, and upstream gradients)
            const uint32_t next = base + gridDim.x * kMlpBlock;
            if (next < a.in.n_samples) {
                const size_t first = static_cast<size_t>(next) * n_out, end = static_cast<size_t>(min(next + 32u, a.in.n_samples)) * n_out;
                if (first + lane * 32u < end) asm volatile("prefetch.global.L2 [%0];" :: "l"(a.features + first + lane * 32u));
                if (lane == 0) asm volatile("prefetch.global.L2 [%0];" :: "l"(a.grad_raw_density + next));
            }
        }
        __syncwarp();

        // phase 1, one sample per lane: MLP recomputation and its input gradient (featurize_backward_mlp.cu:82-105), two
        // hidden units per paired instruction in the recomputation and two inputs per paired instruction in the gradient
        float grad_f[NOUT_PAD];
        {
            uint64_t ff[NOUT_PAD];  // (f_i, f_i)
            #pragma unroll
            for (int q = 0; q < NOUT_PAD / 4; q++) {
                const float4 v = *reinterpret_cast<const float4*>(s_feat + lane * fs + 4 * q);
                ff[4 * q] = pair_of(v.x, v.x);
                ff[4 * q + 1] = pair_of(v.y, v.y);
                ff[4 * q + 2] = pair_of(v.z, v.z);
                ff[4 * q + 3] = pair_of(v.w, v.w);
            }
            const float g = s_g[lane];
            uint64_t gf[NOUT_PAD / 2];  // (grad_f_2k, grad_f_2k+1)
            #pragma unroll
            for (int k = 0; k < NOUT_PAD / 2; k++) gf[k] = pair_of(0.0f, 0.0f);
            // kMlpChains pairs of hidden units at a time: their recomputations are independent chains, interleaved
            for (int j0 = 0; j0 < w_pad; j0 += 2 * kMlpChains) {
                // rows j0 + 2 h and j0 + 2 h + 1 in the forward's accumulation order; the padding columns (zero weight,
                // zero feature) add +0, which changes at most the sign of a zero and so neither the ReLU mask nor
                // relu(pre)
                uint64_t p[kMlpChains];
                #pragma unroll
                for (int h = 0; h < kMlpChains; h++) p[h] = pair_of(s_b0[j0 + 2 * h], s_b0[j0 + 2 * h + 1]);
                const float4* wp = reinterpret_cast<const float4*>(s_w0p + (j0 / 2) * 2 * NOUT_PAD);
                #pragma unroll
                for (int q = 0; q < NOUT_PAD / 2; q++) {
                    #pragma unroll
                    for (int h = 0; h < kMlpChains; h++) {
                        const float4 w2 = wp[h * NOUT_PAD / 2 + q];  // (w[j][2q], w[j+1][2q], w[j][2q+1], w[j+1][2q+1])
                        p[h] = fma_pair(pair_of(w2.x, w2.y), ff[2 * q], p[h]);
                        p[h] = fma_pair(pair_of(w2.z, w2.w), ff[2 * q + 1], p[h]);
                    }
                }
                float pre[2 * kMlpChains];
                #pragma unroll
                for (int h = 0; h < kMlpChains; h++) {
                    const float2 pv = split_pair(p[h]);
                    pre[2 * h] = pv.x;
                    pre[2 * h + 1] = pv.y;
                }
                // branch-free: a zero pre-activation gradient adds +0 (the warp has some positive lane anyway)
                #pragma unroll
                for (int r = 0; r < 2 * kMlpChains; r++) {
                    const float grad_pre = pre[r] > 0.0f ? __fmul_rn(g, s_w1[j0 + r]) : 0.0f;
                    const uint64_t gp = pair_of(grad_pre, grad_pre);
                    const float4* w = reinterpret_cast<const float4*>(s_w0 + (j0 + r) * NOUT_PAD);
                    #pragma unroll
                    for (int q = 0; q < NOUT_PAD / 4; q++) {
                        const float4 wq = w[q];
                        gf[2 * q] = fma_pair(gp, pair_of(wq.x, wq.y), gf[2 * q]);
                        gf[2 * q + 1] = fma_pair(gp, pair_of(wq.z, wq.w), gf[2 * q + 1]);
                    }
                }
                #pragma unroll
                for (int h = 0; h < kMlpChains / 2; h++) {
                    *reinterpret_cast<float4*>(s_pre + lane * ps + j0 + 4 * h) = make_float4(pre[4 * h], pre[4 * h + 1], pre[4 * h + 2], pre[4 * h + 3]);
                }
            }
            #pragma unroll
            for (int k = 0; k < NOUT_PAD / 2; k++) {
                const float2 v = split_pair(gf[k]);
                grad_f[2 * k] = v.x;
                grad_f[2 * k + 1] = v.y;
            }
        }
        {
            // this sample's scaled feature gradient to grad_rows (read by the scatter kernel)
            if (lane < n_rows) {
                float* out = a.grad_rows + static_cast<size_t>(base + lane) * n_out;
                if (vector_rows) {
                    #pragma unroll
                    for (int q = 0; q < NOUT_PAD / 4; q++) {
                        if (4 * q < n_out) {
                            __stcs(reinterpret_cast<float4*>(out) + q, make_float4(__fmul_rn(grad_f[4 * q], kFeatureScale), __fmul_rn(grad_f[4 * q + 1], kFeatureScale),
                                                                                  __fmul_rn(grad_f[4 * q + 2], kFeatureScale), __fmul_rn(grad_f[4 * q + 3], kFeatureScale)));
                        }
                    }
                }
                else {
                    #pragma unroll
                    for (int i = 0; i < NOUT_PAD; i++) {
                        if (i < n_out) __stcs(out + i, __fmul_rn(grad_f[i], kFeatureScale));
                    }
                }
            }
        }
        __syncwarp();

        // phase 2: the chunk's parameter gradient sums in sample order per output (as the reference's
        // featurize_backward_mlp.cu:110-135): tiles of 4 x TI of grad_w0 (a register-blocked outer product of
        // [pre > 0] g with the features); the tiles of the first columns also sum grad_b0 and grad_w1 of their rows
        for (int tile = lane; tile < n_tiles; tile += 32) {
            const int j0 = (tile / n_itiles) * 4, i0 = (tile % n_itiles) * TI;
            // paired sums: sum2[r][k] = (sum[r][2k], sum[r][2k+1]), b0s / w1s = rows (0, 1) and (2, 3)
            uint64_t sum2[4][TI / 2];
            #pragma unroll
            for (int r = 0; r < 4; r++) {
                #pragma unroll
                for (int k = 0; k < TI / 2; k++) sum2[r][k] = pair_of(0.0f, 0.0f);
            }
            uint64_t b0s[2] = {pair_of(0.0f, 0.0f), pair_of(0.0f, 0.0f)}, w1s[2] = {pair_of(0.0f, 0.0f), pair_of(0.0f, 0.0f)};
            for (int s = 0; s < n_rows; s++) {
                const float4 p = *reinterpret_cast<const float4*>(s_pre + s * ps + j0);
                uint64_t fc[TI / 2];
                #pragma unroll
                for (int k = 0; k < TI / 2; k++) {
                    const float2 v = *reinterpret_cast<const float2*>(s_feat + s * fs + i0 + 2 * k);
                    fc[k] = pair_of(v.x, v.y);
                }
                const float gs = s_g[s];
                const float av[4] = {p.x > 0.0f ? gs : 0.0f, p.y > 0.0f ? gs : 0.0f, p.z > 0.0f ? gs : 0.0f, p.w > 0.0f ? gs : 0.0f};
                #pragma unroll
                for (int r = 0; r < 4; r++) {
                    const uint64_t a2 = pair_of(av[r], av[r]);
                    #pragma unroll
                    for (int k = 0; k < TI / 2; k++) sum2[r][k] = fma_pair(a2, fc[k], sum2[r][k]);
                }
                const uint64_t g2 = pair_of(gs, gs);
                b0s[0] = add_pair(b0s[0], pair_of(av[0], av[1]));
                b0s[1] = add_pair(b0s[1], pair_of(av[2], av[3]));
                w1s[0] = fma_pair(g2, pair_of(fmaxf(p.x, 0.0f), fmaxf(p.y, 0.0f)), w1s[0]);
                w1s[1] = fma_pair(g2, pair_of(fmaxf(p.z, 0.0f), fmaxf(p.w, 0.0f)), w1s[1]);
            }
            float sum[4][TI], sum_b0[4], sum_w1[4];
            #pragma unroll
            for (int r = 0; r < 4; r++) {
                #pragma unroll
                for (int k = 0; k < TI / 2; k++) {
                    const float2 v = split_pair(sum2[r][k]);
                    sum[r][2 * k] = v.x;
                    sum[r][2 * k + 1] = v.y;
                }
            }
            #pragma unroll
            for (int h = 0; h < 2; h++) {
                const float2 b = split_pair(b0s[h]), w = split_pair(w1s[h]);
                sum_b0[2 * h] = b.x;
                sum_b0[2 * h + 1] = b.y;
                sum_w1[2 * h] = w.x;
                sum_w1[2 * h + 1] = w.y;
            }
            #pragma unroll
            for (int r = 0; r < 4; r++) {
                const int j = j0 + r;
                #pragma unroll
                for (int c = 0; c < TI; c++) {
                    const int i = i0 + c;
                    if (j < W && i < n_out && sum[r][c] != 0.0f) atomicAdd(s_acc + i * acc_stride + j, sum[r][c]);
                }
                if (i0 == 0 && j < W) {
                    if (sum_b0[r] != 0.0f) atomicAdd(s_acc + acc_b0 + j, sum_b0[r]);
                    if (sum_w1[r] != 0.0f) atomicAdd(s_acc + acc_w1 + j, sum_w1[r]);
                }
            }
        }
        if (lane == 0) {
            float sum = 0.0f;
            for (int s = 0; s < n_rows; s++) sum = __fadd_rn(sum, s_g[s]);
            if (sum != 0.0f) atomicAdd(s_acc + acc_b1, sum);
        }
        __syncwarp();
    }
    __syncthreads();

    // one atomic per parameter and block, with w1 applied late (featurize_backward_mlp.cu:139-147)
    for (int q = threadIdx.x; q < n_params; q += kMlpBlock) {
        if (q < n_w0) {
            const int j = q / n_out, i = q - j * n_out;
            const float acc = s_acc[i * acc_stride + j];
            if (acc != 0.0f) atomicAdd(a.grad_w0 + q, s_w1[j] * acc);
        }
        else if (q < n_w0 + W) {
            const float acc = s_acc[acc_b0 + q - n_w0];
            if (acc != 0.0f) atomicAdd(a.grad_b0 + (q - n_w0), s_w1[q - n_w0] * acc);
        }
        else if (q < n_w0 + 2 * W) {
            const float acc = s_acc[acc_w1 + q - n_w0 - W];
            if (acc != 0.0f) atomicAdd(a.grad_w1 + (q - n_w0 - W), acc);
        }
        else if (s_acc[acc_b1] != 0.0f) atomicAdd(a.grad_b1, s_acc[acc_b1]);
    }
}

// ---------------------------------------------------------------------------------------------------------------------
// numerics self-check: approx_erf over a range of float bit patterns; counts the arguments whose value is not exactly
// 1.0f and records the largest such bit pattern (atomicMax on the bits orders non-negative floats)

template <int kUnused>
__global__ void fz_check_erf_kernel(const uint32_t first_bits, const uint32_t count, unsigned long long* n_not_one, uint32_t* max_bits) {
    unsigned long long local = 0;
    uint32_t local_max = 0;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
        const uint32_t bits = first_bits + i;
        if (approx_erf(__uint_as_float(bits)) != 1.0f) {
            local++;
            local_max = max(local_max, bits);
        }
    }
    if (local != 0) {
        atomicAdd(n_not_one, local);
        atomicMax(max_bits, local_max);
    }
}

// ---------------------------------------------------------------------------------------------------------------------
// debug: intermediate values of single intervals (positions, contraction flags, merged corner rows and weights)

struct DebugArgs {
    RayInputs in;
    const uint32_t* samples;  // [n_debug] sample indices
    uint32_t n_debug;
    float* x;                 // [n_debug, 6, 3]
    float* scale;             // [n_debug, 6]
    int32_t* contracted;      // [n_debug, 6]
    int32_t* n_groups;        // [n_debug, L]
    uint32_t* rows;           // [n_debug, L, 6, 8]
    float* weights;           // [n_debug, L, 6, 8]
};

// (a template only so that the header defines no non-inline kernel; instantiated once, as fz_debug_kernel<0>)
template <int kUnused>
__global__ void fz_debug_kernel(const __grid_constant__ GridParams gp, const __grid_constant__ DebugArgs a) {
    const uint32_t d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= a.n_debug) return;
    const uint32_t sample = a.samples[d];
    const uint32_t L = gp.n_levels;
    const Frustum fr = setup_frustum(a.in, gp.pattern_stream, sample);
    float3 x[kMultisamples];
    float scale[kMultisamples];
    #pragma unroll
    for (uint32_t j = 0; j < kMultisamples; j++) {
        bool contracted;
        multisample(fr, j, x[j], scale[j], &contracted);
        a.x[(d * kMultisamples + j) * 3] = x[j].x;
        a.x[(d * kMultisamples + j) * 3 + 1] = x[j].y;
        a.x[(d * kMultisamples + j) * 3 + 2] = x[j].z;
        a.scale[d * kMultisamples + j] = scale[j];
        a.contracted[d * kMultisamples + j] = contracted;
    }
    #pragma unroll 1
    for (uint32_t level = 0; level < L; level++) {
        float weighting[kMultisamples];
        #pragma unroll
        for (uint32_t j = 0; j < kMultisamples; j++) weighting[j] = level_weighting(gp.size[level], scale[j]);
        uint32_t n = 0;
        const size_t base = (static_cast<size_t>(d) * L + level) * kMultisamples * 8;
        auto visitor = [&](const uint32_t row, const float weight) {
            a.rows[base + n] = row;
            a.weights[base + n] = weight;
            n++;
        };
        visit_level(gp, level, x, weighting, visitor);
        for (uint32_t k = n; k < kMultisamples * 8; k++) {
            a.rows[base + k] = 0u;
            a.weights[base + k] = 0.0f;
        }
        a.n_groups[d * L + level] = static_cast<int32_t>(n / 8);
    }
}

}  // namespace zf

#pragma once

// Shared machinery for row-wise kernels (softmax, layer_norm, rms_norm).
//
// A row is owned by a "group" of threads: one warp for rows up to 1024
// floats (no __syncthreads at all), or a 256-thread block for longer rows.
// The row is loaded ONCE into registers (kSlots 16-byte vectors per thread),
// reduced in registers and written once: one HBM read + one HBM write per
// element, where the SIMT original re-read each row two or three times.
// Rows too long for registers (> 8192 floats) use a streaming variant.

#include "../../core/block_reduce.cuh"
#include "../../core/cuda_utils.cuh"

namespace opworks::detail {

// Reductions over the threads that own one row.
template <int kGroup> struct RowGroup;

template <> struct RowGroup<32> {
    __device__ __forceinline__ static int rank() { return threadIdx.x % kWarpSize; }
    __device__ __forceinline__ static float sum(float v) { return warp_reduce<ReduceSum>(v); }
    __device__ __forceinline__ static float max(float v) { return warp_reduce<ReduceMax>(v); }
};

template <> struct RowGroup<kThreads> {
    __device__ __forceinline__ static int rank() { return threadIdx.x; }
    __device__ __forceinline__ static float sum(float v) { return block_reduce_all<ReduceSum>(v); }
    __device__ __forceinline__ static float max(float v) { return block_reduce_all<ReduceMax>(v); }
};

// Row index handled by this thread's group; warps of a block take
// consecutive rows when kGroup == 32.
template <int kGroup> __device__ __forceinline__ int64_t row_of_group() {
    if constexpr (kGroup == 32)
        return static_cast<int64_t>(blockIdx.x) * (blockDim.x / kWarpSize) + threadIdx.x / kWarpSize;
    else
        return blockIdx.x;
}

// Vector access helpers: V is float4 (aligned rows, cols % 4 == 0) or float.
template <typename V> struct VecTraits;
template <> struct VecTraits<float4> {
    static constexpr int kWidth = 4;
    __device__ __forceinline__ static float get(const float4 &v, int i) {
        return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
    }
    __device__ __forceinline__ static void set(float4 &v, int i, float x) {
        if (i == 0)
            v.x = x;
        else if (i == 1)
            v.y = x;
        else if (i == 2)
            v.z = x;
        else
            v.w = x;
    }
};
template <> struct VecTraits<float> {
    static constexpr int kWidth = 1;
    __device__ __forceinline__ static float get(const float &v, int) { return v; }
    __device__ __forceinline__ static void set(float &v, int, float x) { v = x; }
};

// Launch geometry for a row kernel on `rows` rows of `cols` floats.
struct RowPlan {
    int group;  // 32 or kThreads
    int slots;  // vectors per thread (register tile); 0 = streaming
    bool vec;   // float4 path
};

inline RowPlan plan_rows(int cols, bool aligned) {
    RowPlan p;
    p.vec = aligned && cols % 4 == 0;
    const int width = p.vec ? 4 : 1;
    const int vecs = (cols + width - 1) / width;
    if (vecs <= 32 * 8) { // warp per row, <= 8 vectors per lane
        p.group = 32;
        p.slots = (vecs + 31) / 32;
    } else if (vecs <= kThreads * 8) {
        p.group = kThreads;
        p.slots = (vecs + kThreads - 1) / kThreads;
    } else {
        p.group = kThreads;
        p.slots = 0;
    }
    // round slots up to a compiled instantiation
    if (p.slots > 4)
        p.slots = 8;
    else if (p.slots > 2)
        p.slots = 4;
    return p;
}

inline int row_grid(int rows, int group) {
    if (group == 32) {
        const int rows_per_block = kThreads / kWarpSize;
        return rows / rows_per_block + (rows % rows_per_block != 0 ? 1 : 0);
    }
    return rows;
}

inline bool aligned16(const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

// Warps per SM of the row-walking (warp per row, next row prefetched) grid
// of softmax; OPWORKS_ROW_WARPS_PER_SM overrides the measured default.
inline int row_walk_warps_per_sm() {
    static const int v = [] {
        const char *e = std::getenv("OPWORKS_ROW_WARPS_PER_SM");
        const int w = e ? std::atoi(e) : 16;
        return w >= 8 && w <= 64 ? w : 16;
    }();
    return v;
}

// Blocks of kThreads in a row-walking grid of `rows` rows (one warp per row):
// at most one resident wave, at most row_walk_warps_per_sm() warps per SM
// (the kernel's occupancy, queried once per device, may allow fewer).
template <auto Kernel> inline int row_walk_grid(int64_t rows) {
    static thread_local int per_sm[16] = {0};
    const DeviceFacts &f = device_facts();
    int &slot = per_sm[f.device % 16];
    if (slot == 0) {
        int occ = 0;
        OPWORKS_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, Kernel, kThreads, 0));
        const int want = row_walk_warps_per_sm() / (kThreads / kWarpSize);
        slot = occ < want ? (occ > 0 ? occ : 1) : (want > 0 ? want : 1);
    }
    const int per_block = kThreads / kWarpSize;
    const int64_t need = (rows + per_block - 1) / per_block;
    const int64_t cap = static_cast<int64_t>(f.sm_count) * slot;
    return static_cast<int>(need < cap ? need : cap);
}

} // namespace opworks::detail

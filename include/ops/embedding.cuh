#pragma once

// ops::embedding — out[t, :] = table[ids[t], :] for a [vocab, hidden] table
// (fp32 or bf16), fp32 output (OpWorks include/ops/embedding.cuh:24-34).
// ids are not range-checked on the device; callers validate them.
//
// B200 kernel: 16-byte gathers (4 fp32 or 8 bf16 table entries per load).

#include <cuda_bf16.h>

#include "../core/cuda_utils.cuh"

namespace opworks::detail {

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename WT>
__global__ void embedding_vec_kernel(const WT *__restrict__ table, const int *__restrict__ ids, float *__restrict__ out,
                                     int hidden, int n) {
    constexpr int kPer = 16 / sizeof(WT); // table entries per 16-byte load
    const int per_row = hidden / kPer;
    OPWORKS_GRID_LOOP(i, static_cast<int64_t>(n) * per_row) {
        const int64_t row = i / per_row;
        const int64_t col = (i % per_row) * kPer;
        const uint4 raw = *reinterpret_cast<const uint4 *>(table + static_cast<int64_t>(ids[row]) * hidden + col);
        float4 *dst = reinterpret_cast<float4 *>(out + row * hidden + col);
        if constexpr (sizeof(WT) == 4) {
            dst[0] = *reinterpret_cast<const float4 *>(&raw);
        } else {
            const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&raw);
            const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
            const float2 c = __bfloat1622float2(h[2]), d = __bfloat1622float2(h[3]);
            dst[0] = make_float4(a.x, a.y, b.x, b.y);
            dst[1] = make_float4(c.x, c.y, d.x, d.y);
        }
    }
}

template <typename WT>
__global__ void embedding_scalar_kernel(const WT *__restrict__ table, const int *__restrict__ ids,
                                        float *__restrict__ out, int hidden, int n) {
    OPWORKS_GRID_LOOP(i, static_cast<int64_t>(n) * hidden) {
        const int64_t row = i / hidden;
        out[i] = to_f32(table[static_cast<int64_t>(ids[row]) * hidden + (i % hidden)]);
    }
}

} // namespace opworks::detail

namespace opworks::ops {

template <typename WT>
inline void embedding(const WT *table, const int *ids, float *out, int n, int hidden, cudaStream_t stream = nullptr) {
    detail::validate_size(n);
    detail::validate_size(hidden);
    if (n == 0)
        return;
    detail::require(hidden > 0 && table && ids && out, "embedding requires positive width and non-null pointers");
    constexpr int kPer = 16 / sizeof(WT);
    const bool vec = hidden % kPer == 0 && reinterpret_cast<uintptr_t>(table) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(out) % 16 == 0;
    const int64_t work = vec ? static_cast<int64_t>(n) * (hidden / kPer) : static_cast<int64_t>(n) * hidden;
    const int64_t blocks = (work + kThreads - 1) / kThreads;
    const int grid = static_cast<int>(blocks < detail::device_facts().max_grid_blocks
                                          ? blocks
                                          : detail::device_facts().max_grid_blocks);
    if (vec)
        launch_async(stream, detail::embedding_vec_kernel<WT>, grid, kThreads, table, ids, out, hidden, n);
    else
        launch_async(stream, detail::embedding_scalar_kernel<WT>, grid, kThreads, table, ids, out, hidden, n);
}

} // namespace opworks::ops

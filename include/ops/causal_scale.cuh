#pragma once

// ops::causal_scale — on a [rows, cols] score matrix whose queries sit at
// absolute positions [cols - rows, cols), scales the visible scores (key <=
// query position) and sets the others to -inf, in place. Contract: OpWorks
// include/ops/causal_scale.cuh:24-33 (signature, checks, asynchronous).
//
// One block per row: the row's visible prefix is read, scaled and written
// back in 16-byte vectors when the row allows it; the masked suffix is only
// written (its old values are never needed). The Llama runtime never
// materialises scores (its attention is fused); this is the standalone op.

#include <algorithm>

#include "../core/cuda_utils.cuh"

namespace opworks::detail {

template <int kVec> static __global__ void causal_scale_rows_kernel(float *scores, int rows, int cols, float scale) {
    const int vecs = cols / kVec;
    for (int row = blockIdx.x; row < rows; row += gridDim.x) {
        const int last = cols - rows + row; // last visible key of this query
        float *r = scores + static_cast<int64_t>(row) * cols;
        for (int v = threadIdx.x; v < vecs; v += blockDim.x) {
            const int c0 = v * kVec;
            float val[kVec];
            if (c0 > last) {
#pragma unroll
                for (int k = 0; k < kVec; ++k)
                    val[k] = kNegInf;
            } else {
                if constexpr (kVec == 4) {
                    const float4 f = *reinterpret_cast<const float4 *>(r + c0);
                    val[0] = f.x, val[1] = f.y, val[2] = f.z, val[3] = f.w;
                } else {
                    val[0] = r[c0];
                }
#pragma unroll
                for (int k = 0; k < kVec; ++k)
                    val[k] = c0 + k <= last ? val[k] * scale : kNegInf;
            }
            if constexpr (kVec == 4)
                *reinterpret_cast<float4 *>(r + c0) = make_float4(val[0], val[1], val[2], val[3]);
            else
                r[c0] = val[0];
        }
    }
}

} // namespace opworks::detail

namespace opworks::ops {

inline void causal_scale(float *scores, int rows, int cols, float scale, cudaStream_t stream = nullptr) {
    detail::validate_matrix(rows, cols);
    if (rows == 0)
        return;
    detail::require(cols >= rows, "causal scores need at least as many keys as queries");
    detail::require(scores && scale > 0.f, "causal_scale requires a buffer and a positive scale");
    const bool vec = cols % 4 == 0 && reinterpret_cast<uintptr_t>(scores) % 16 == 0;
    const int grid = std::min(rows, detail::device_facts().max_grid_blocks);
    if (vec)
        launch_async(stream, detail::causal_scale_rows_kernel<4>, dim3(grid), dim3(kThreads), scores, rows, cols, scale);
    else
        launch_async(stream, detail::causal_scale_rows_kernel<1>, dim3(grid), dim3(kThreads), scores, rows, cols, scale);
}

} // namespace opworks::ops

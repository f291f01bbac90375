#pragma once

// ops::causal_scale — scale visible scores, -inf the masked ones, on a
// [rows, cols] score matrix whose queries sit at positions [cols-rows, cols)
// (OpWorks include/ops/causal_scale.cuh:24-33). The Llama runtime never
// materialises scores (flash attention); this is the standalone op.

#include "../core/cuda_utils.cuh"

namespace opworks::detail {

static __global__ void causal_scale_kernel(float *scores, int rows, int cols, float scale) {
    OPWORKS_GRID_LOOP(i, static_cast<int64_t>(rows) * cols) {
        const int row = static_cast<int>(i / cols);
        const int col = static_cast<int>(i % cols);
        scores[i] = col <= cols - rows + row ? scores[i] * scale : kNegInf;
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
    launch_async(stream, detail::causal_scale_kernel, num_blocks_for(rows * cols), kThreads, scores, rows, cols,
                 scale);
}

} // namespace opworks::ops

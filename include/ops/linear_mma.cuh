#pragma once

// ops::linear_mma_bf16 — tensor-core Y = X @ W^T for bf16 weights
// (OpWorks include/ops/linear_mma.cuh:101-115: X fp32 rounded to bf16, W bf16
// [out, in], fp32 accumulation). Here it is the tcgen05 kind::f16 GEMM with
// TMA-fed operands and a TMEM accumulator, for any row count.

#include "linear.cuh"

namespace opworks::ops {

inline void linear_mma_bf16(const float *X, const __nv_bfloat16 *W, float *Y, int rows, int in_features,
                            int out_features, cudaStream_t stream = nullptr) {
    detail::validate_matrix(rows, in_features);
    detail::validate_matrix(out_features, in_features);
    detail::validate_matrix(rows, out_features);
    if (rows == 0 || out_features == 0)
        return;
    detail::require(X && W && Y, "linear_mma_bf16 requires non-null pointers");
    detail::require(in_features > 0, "linear_mma_bf16 requires a positive reduction dim");
    detail::linear_bf16_tc(X, W, Y, rows, in_features, out_features, stream);
}

} // namespace opworks::ops

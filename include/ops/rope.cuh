#pragma once

// ops::rope — in-place rotary embedding, HF rotate_half convention: pair
// (i, i + D/2), a' = a cos - b sin, b' = b cos + a sin, angle
// (pos_start + row) * inv_freq[i] evaluated in fp32 with cosf/sinf
// (OpWorks include/ops/rope.cuh:10-46). The Llama runtime applies RoPE inside
// its QKV finalisation kernel from a precomputed cos/sin table built with the
// same fp32 expression; this is the standalone op.

#include "../core/cuda_utils.cuh"

namespace opworks::detail {

static __global__ void rope_kernel(float *x, const float *inv_freq, int rows, int heads, int head_dim, int pos_start) {
    const int half = head_dim / 2;
    OPWORKS_GRID_LOOP(i, static_cast<int64_t>(rows) * heads * half) {
        const int pair = static_cast<int>(i % half);
        const int64_t rh = i / half; // row * heads + head
        const int row = static_cast<int>(rh / heads);
        const float angle = static_cast<float>(pos_start + row) * inv_freq[pair];
        const float c = cosf(angle), s = sinf(angle);
        float *p = x + rh * head_dim + pair;
        const float a = p[0], b = p[half];
        p[0] = a * c - b * s;
        p[half] = b * c + a * s;
    }
}

} // namespace opworks::detail

namespace opworks::ops {

inline void rope(float *x, const float *inv_freq, int rows, int heads, int head_dim, int pos_start,
                 cudaStream_t stream = nullptr) {
    detail::validate_size(rows);
    if (rows == 0)
        return;
    detail::require(heads > 0 && head_dim > 0 && head_dim % 2 == 0, "rope requires even positive head_dim");
    detail::require(pos_start >= 0, "rope position must be nonnegative");
    detail::require(x && inv_freq, "rope requires non-null pointers");
    const int64_t n = static_cast<int64_t>(rows) * heads * (head_dim / 2);
    detail::require(n <= std::numeric_limits<int>::max(), "rope input exceeds the supported INT_MAX pairs");
    launch_async(stream, detail::rope_kernel, num_blocks_for(static_cast<int>(n)), kThreads, x, inv_freq, rows, heads,
                 head_dim, pos_start);
}

} // namespace opworks::ops

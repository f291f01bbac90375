#pragma once

// ops::split_heads / ops::merge_heads — packed rows [rows, heads * head_dim]
// to per-head slabs [heads, stride, head_dim] (written from row `offset`) and
// back. Contract: OpWorks include/ops/split_heads.cuh:39-66 (signatures,
// checks, asynchronous launch).
//
// Both are one primitive here: a strided copy of head_dim-float segments,
// segment (row t, head h) going from src + t * src_row + h * src_head to
// dst + t * dst_row + h * dst_head. Heads run on the grid's y dimension, so a
// block's segments of one head are contiguous on the slab side; segments move
// in 16-byte vectors when head_dim and both pointers allow it. The Llama
// runtime writes K/V straight into its paged cache from the QKV GEMM epilogue
// and never calls these.

#include <algorithm>

#include "../core/cuda_utils.cuh"

namespace opworks::detail {

struct HeadSlabCopy {
    const float *src;
    float *dst;
    int rows, heads, head_dim;
    int64_t src_row, src_head, dst_row, dst_head;
};

template <int kVec> static __global__ void head_slab_copy_kernel(HeadSlabCopy c) {
    const int vecs = c.head_dim / kVec;
    const int64_t per_head = static_cast<int64_t>(c.rows) * vecs;
    for (int h = blockIdx.y; h < c.heads; h += gridDim.y) {
        const float *src = c.src + h * c.src_head;
        float *dst = c.dst + h * c.dst_head;
        for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < per_head;
             i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
            const int64_t t = i / vecs;
            const int d = static_cast<int>(i - t * vecs) * kVec;
            if constexpr (kVec == 4)
                *reinterpret_cast<float4 *>(dst + t * c.dst_row + d) =
                    *reinterpret_cast<const float4 *>(src + t * c.src_row + d);
            else
                dst[t * c.dst_row + d] = src[t * c.src_row + d];
        }
    }
}

inline void head_slab_copy(const HeadSlabCopy &c, cudaStream_t stream) {
    const bool vec = c.head_dim % 4 == 0 && reinterpret_cast<uintptr_t>(c.src) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(c.dst) % 16 == 0 && c.src_row % 4 == 0 && c.dst_row % 4 == 0 &&
                     c.src_head % 4 == 0 && c.dst_head % 4 == 0;
    const int vec_width = vec ? 4 : 1;
    const int64_t per_head = static_cast<int64_t>(c.rows) * (c.head_dim / vec_width);
    const int heads_y = std::min(c.heads, 65535);
    const int64_t want_x = (per_head + kThreads - 1) / kThreads;
    const int cap_x = std::max(1, device_facts().max_grid_blocks / heads_y);
    const dim3 grid(static_cast<unsigned>(std::min<int64_t>(want_x, cap_x)), static_cast<unsigned>(heads_y));
    if (vec)
        launch_async(stream, head_slab_copy_kernel<4>, grid, dim3(kThreads), c);
    else
        launch_async(stream, head_slab_copy_kernel<1>, grid, dim3(kThreads), c);
}

} // namespace opworks::detail

namespace opworks::ops {

inline void split_heads(const float *in, float *out, int rows, int heads, int head_dim, int out_row_stride,
                        int out_row_offset = 0, cudaStream_t stream = nullptr) {
    detail::validate_size(rows);
    if (rows == 0)
        return;
    detail::require(heads > 0 && head_dim > 0, "split_heads requires positive head shape");
    detail::require(out_row_stride >= out_row_offset + rows, "split_heads exceeds the output row stride");
    detail::require(in && out, "split_heads requires non-null pointers");
    detail::require(static_cast<int64_t>(rows) * heads * head_dim <= std::numeric_limits<int>::max(),
                    "split_heads input exceeds INT_MAX elements");
    const int64_t D = head_dim;
    detail::head_slab_copy({in, out + static_cast<int64_t>(out_row_offset) * D, rows, heads, head_dim, heads * D, D, D,
                            static_cast<int64_t>(out_row_stride) * D},
                           stream);
}

inline void merge_heads(const float *in, float *out, int rows, int heads, int head_dim, int in_row_stride,
                        int in_row_offset = 0, cudaStream_t stream = nullptr) {
    detail::validate_size(rows);
    if (rows == 0)
        return;
    detail::require(heads > 0 && head_dim > 0, "merge_heads requires positive head shape");
    detail::require(in_row_stride >= in_row_offset + rows, "merge_heads exceeds the input row stride");
    detail::require(in && out, "merge_heads requires non-null pointers");
    detail::require(static_cast<int64_t>(rows) * heads * head_dim <= std::numeric_limits<int>::max(),
                    "merge_heads input exceeds INT_MAX elements");
    const int64_t D = head_dim;
    detail::head_slab_copy({in + static_cast<int64_t>(in_row_offset) * D, out, rows, heads, head_dim, D,
                            static_cast<int64_t>(in_row_stride) * D, heads * D, D},
                           stream);
}

} // namespace opworks::ops

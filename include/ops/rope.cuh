#pragma once

// ops::rope — in-place rotary position embedding on x[rows, heads * head_dim]
// at absolute positions [pos_start, pos_start + rows), HF rotate_half pairing
// (i, i + head_dim/2): a' = a cos - b sin, b' = b cos + a sin, with the angle
// (pos_start + row) * inv_freq[i] formed in fp32 and cosf / sinf.
// Contract: OpWorks include/ops/rope.cuh:34-46 (signature, checks, async).
//
// Layout of the work: one block per position. The block evaluates the
// position's head_dim/2 angles once into shared memory (every head of the row
// uses the same cos/sin), then rotates all heads with 16-byte loads and
// stores of four pairs at a time when the row allows it. The Llama runtime
// itself never calls this op: RoPE is applied in its QKV GEMM epilogue from
// a precomputed table.

#include <algorithm>

#include "../core/cuda_utils.cuh"

namespace opworks::detail {

constexpr int kRopeThreads = 128;
constexpr int kRopeMaxTableHalf = 2048; // cos/sin table in shared memory up to head_dim 4096

template <bool kTable, int kVec>
static __global__ void __launch_bounds__(kRopeThreads)
    rope_rows_kernel(float *x, const float *inv_freq, int rows, int heads, int head_dim, int pos_start) {
    extern __shared__ float rope_tab[]; // [half] cos, then [half] sin
    const int half = head_dim / 2;
    const int vecs = half / kVec;
    for (int row = blockIdx.x; row < rows; row += gridDim.x) {
        const float pos = static_cast<float>(pos_start + row);
        if constexpr (kTable) {
            for (int j = threadIdx.x; j < half; j += blockDim.x) {
                const float angle = pos * inv_freq[j];
                rope_tab[j] = cosf(angle);
                rope_tab[half + j] = sinf(angle);
            }
            __syncthreads();
        }
        float *xr = x + static_cast<int64_t>(row) * heads * head_dim;
        for (int u = threadIdx.x; u < heads * vecs; u += blockDim.x) {
            const int j0 = (u % vecs) * kVec;
            float *lo = xr + static_cast<int64_t>(u / vecs) * head_dim + j0;
            float *hi = lo + half;
            float a[kVec], b[kVec];
            if constexpr (kVec == 4) {
                const float4 va = *reinterpret_cast<const float4 *>(lo), vb = *reinterpret_cast<const float4 *>(hi);
                a[0] = va.x, a[1] = va.y, a[2] = va.z, a[3] = va.w;
                b[0] = vb.x, b[1] = vb.y, b[2] = vb.z, b[3] = vb.w;
            } else {
                a[0] = lo[0];
                b[0] = hi[0];
            }
#pragma unroll
            for (int k = 0; k < kVec; ++k) {
                float c, s;
                if constexpr (kTable) {
                    c = rope_tab[j0 + k];
                    s = rope_tab[half + j0 + k];
                } else {
                    const float angle = pos * inv_freq[j0 + k];
                    c = cosf(angle);
                    s = sinf(angle);
                }
                const float ra = a[k] * c - b[k] * s, rb = b[k] * c + a[k] * s;
                a[k] = ra;
                b[k] = rb;
            }
            if constexpr (kVec == 4) {
                *reinterpret_cast<float4 *>(lo) = make_float4(a[0], a[1], a[2], a[3]);
                *reinterpret_cast<float4 *>(hi) = make_float4(b[0], b[1], b[2], b[3]);
            } else {
                lo[0] = a[0];
                hi[0] = b[0];
            }
        }
        if constexpr (kTable)
            __syncthreads(); // the next row rewrites the table
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
    const int half = head_dim / 2;
    const bool vec = half % 4 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0;
    const bool table = half <= detail::kRopeMaxTableHalf;
    const int grid = std::min(rows, detail::device_facts().max_grid_blocks);
    const size_t smem = table ? sizeof(float) * 2 * half : 0;
    using K = void (*)(float *, const float *, int, int, int, int);
    const K kernel = table ? (vec ? detail::rope_rows_kernel<true, 4> : detail::rope_rows_kernel<true, 1>)
                           : (vec ? detail::rope_rows_kernel<false, 4> : detail::rope_rows_kernel<false, 1>);
    kernel<<<grid, detail::kRopeThreads, smem, stream>>>(x, inv_freq, rows, heads, head_dim, pos_start);
    OPWORKS_CUDA_CHECK(cudaGetLastError());
}

} // namespace opworks::ops

#pragma once

// ops::rms_norm — out = x * rsqrt(mean(x^2) + eps) * weight per row
// (OpWorks include/ops/rms_norm.cuh:31-40; same arguments and checks).
//
// B200 kernel: register-resident row (warp per row up to 1024 columns, block
// per row up to 8192), one read and one write of each element.

#include "detail/rows.cuh"

namespace opworks::detail {

template <int kGroup, int kSlots, typename V>
__global__ void __launch_bounds__(kThreads)
    rms_norm_rows_kernel(const float *x, const float *weight, float *out, int rows, int cols, float eps) {
    using T = VecTraits<V>;
    constexpr int W = T::kWidth;
    const int64_t row = row_of_group<kGroup>();
    if (row >= rows)
        return;
    const int nv = cols / W;
    const V *src = reinterpret_cast<const V *>(x + row * cols);
    V *dst = reinterpret_cast<V *>(out + row * cols);
    const V *w = reinterpret_cast<const V *>(weight);
    const int r = RowGroup<kGroup>::rank();
    V v[kSlots];
    float ss = 0.f;
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
        const int idx = r + s * kGroup;
        if (idx < nv) {
            v[s] = src[idx];
#pragma unroll
            for (int i = 0; i < W; ++i)
                ss += T::get(v[s], i) * T::get(v[s], i);
        }
    }
    const float inv = rsqrtf(RowGroup<kGroup>::sum(ss) / cols + eps);
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
        const int idx = r + s * kGroup;
        if (idx < nv) {
            const V wv = w[idx];
            V y;
#pragma unroll
            for (int i = 0; i < W; ++i)
                T::set(y, i, T::get(v[s], i) * inv * T::get(wv, i));
            dst[idx] = y;
        }
    }
}

static __global__ void __launch_bounds__(kThreads)
    rms_norm_rows_stream_kernel(const float *x, const float *weight, float *out, int cols, float eps) {
    const float *src = x + static_cast<int64_t>(blockIdx.x) * cols;
    float *dst = out + static_cast<int64_t>(blockIdx.x) * cols;
    float ss = 0.f;
    for (int j = threadIdx.x; j < cols; j += blockDim.x)
        ss += src[j] * src[j];
    const float inv = rsqrtf(block_reduce_all<ReduceSum>(ss) / cols + eps);
    for (int j = threadIdx.x; j < cols; j += blockDim.x)
        dst[j] = src[j] * inv * weight[j];
}

template <int kGroup, int kSlots>
inline void rms_norm_launch(bool vec, const float *x, const float *w, float *out, int rows, int cols, float eps,
                            cudaStream_t stream) {
    const int grid = row_grid(rows, kGroup);
    if (vec)
        launch_async(stream, rms_norm_rows_kernel<kGroup, kSlots, float4>, grid, kThreads, x, w, out, rows, cols,
                     eps);
    else
        launch_async(stream, rms_norm_rows_kernel<kGroup, kSlots, float>, grid, kThreads, x, w, out, rows, cols,
                     eps);
}

template <int kGroup>
inline void rms_norm_dispatch(const RowPlan &p, const float *x, const float *w, float *out, int rows, int cols,
                              float eps, cudaStream_t stream) {
    switch (p.slots) {
    case 1: rms_norm_launch<kGroup, 1>(p.vec, x, w, out, rows, cols, eps, stream); break;
    case 2: rms_norm_launch<kGroup, 2>(p.vec, x, w, out, rows, cols, eps, stream); break;
    case 4: rms_norm_launch<kGroup, 4>(p.vec, x, w, out, rows, cols, eps, stream); break;
    default: rms_norm_launch<kGroup, 8>(p.vec, x, w, out, rows, cols, eps, stream); break;
    }
}

} // namespace opworks::detail

namespace opworks::ops {

inline void rms_norm(const float *x, const float *weight, float *out, int rows, int cols, float eps,
                     cudaStream_t stream = nullptr) {
    detail::validate_matrix(rows, cols);
    if (rows == 0)
        return;
    detail::require(cols > 0, "rms_norm requires positive columns for nonempty rows");
    detail::require(x && weight && out, "rms_norm requires non-null pointers");
    detail::require(eps > 0.f, "rms_norm epsilon must be positive");
    const bool aligned = detail::aligned16(x) && detail::aligned16(weight) && detail::aligned16(out);
    const detail::RowPlan p = detail::plan_rows(cols, aligned);
    if (p.slots == 0)
        launch_async(stream, detail::rms_norm_rows_stream_kernel, rows, kThreads, x, weight, out, cols, eps);
    else if (p.group == 32)
        detail::rms_norm_dispatch<32>(p, x, weight, out, rows, cols, eps, stream);
    else
        detail::rms_norm_dispatch<kThreads>(p, x, weight, out, rows, cols, eps, stream);
}

} // namespace opworks::ops

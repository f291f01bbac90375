#pragma once

// ops::layer_norm — (x - mean) * rsqrt(var + eps) * gamma + beta per row,
// two-pass variance. Contract of OpWorks include/ops/layer_norm.cuh:38-47.
//
// B200 kernel: the row stays in registers between the mean pass, the
// variance pass and the write, so HBM sees one read and one write per
// element (the original read each row three times).

#include "detail/rows.cuh"

namespace opworks::detail {

template <int kGroup, int kSlots, typename V>
__global__ void __launch_bounds__(kThreads)
    layer_norm_rows_kernel(const float *in, float *out, const float *gamma, const float *beta, int rows, int cols,
                           float eps) {
    using T = VecTraits<V>;
    constexpr int W = T::kWidth;
    const int64_t row = row_of_group<kGroup>();
    if (row >= rows)
        return;
    const int nv = cols / W;
    const V *src = reinterpret_cast<const V *>(in + row * cols);
    V *dst = reinterpret_cast<V *>(out + row * cols);
    const V *g = reinterpret_cast<const V *>(gamma);
    const V *b = reinterpret_cast<const V *>(beta);
    const int r = RowGroup<kGroup>::rank();

    V x[kSlots];
    float sum = 0.f;
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
        const int idx = r + s * kGroup;
        if (idx < nv) {
            x[s] = src[idx];
#pragma unroll
            for (int i = 0; i < W; ++i)
                sum += T::get(x[s], i);
        }
    }
    const float mean = RowGroup<kGroup>::sum(sum) / cols;
    float var = 0.f;
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
        const int idx = r + s * kGroup;
        if (idx < nv) {
#pragma unroll
            for (int i = 0; i < W; ++i) {
                const float d = T::get(x[s], i) - mean;
                var += d * d;
            }
        }
    }
    const float rstd = rsqrtf(RowGroup<kGroup>::sum(var) / cols + eps);
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
        const int idx = r + s * kGroup;
        if (idx < nv) {
            const V gv = g[idx], bv = b[idx];
            V y;
#pragma unroll
            for (int i = 0; i < W; ++i)
                T::set(y, i, (T::get(x[s], i) - mean) * rstd * T::get(gv, i) + T::get(bv, i));
            dst[idx] = y;
        }
    }
}

static __global__ void __launch_bounds__(kThreads) layer_norm_rows_stream_kernel(const float *in, float *out,
                                                                                 const float *gamma,
                                                                                 const float *beta, int cols,
                                                                                 float eps) {
    const float *src = in + static_cast<int64_t>(blockIdx.x) * cols;
    float *dst = out + static_cast<int64_t>(blockIdx.x) * cols;
    float sum = 0.f;
    for (int j = threadIdx.x; j < cols; j += blockDim.x)
        sum += src[j];
    const float mean = block_reduce_all<ReduceSum>(sum) / cols;
    float var = 0.f;
    for (int j = threadIdx.x; j < cols; j += blockDim.x) {
        const float d = src[j] - mean;
        var += d * d;
    }
    const float rstd = rsqrtf(block_reduce_all<ReduceSum>(var) / cols + eps);
    for (int j = threadIdx.x; j < cols; j += blockDim.x)
        dst[j] = (src[j] - mean) * rstd * gamma[j] + beta[j];
}

template <int kGroup, int kSlots>
inline void layer_norm_launch(bool vec, const float *in, float *out, const float *gamma, const float *beta, int rows,
                              int cols, float eps, cudaStream_t stream) {
    const int grid = row_grid(rows, kGroup);
    if (vec)
        launch_async(stream, layer_norm_rows_kernel<kGroup, kSlots, float4>, grid, kThreads, in, out, gamma, beta,
                     rows, cols, eps);
    else
        launch_async(stream, layer_norm_rows_kernel<kGroup, kSlots, float>, grid, kThreads, in, out, gamma, beta,
                     rows, cols, eps);
}

template <int kGroup>
inline void layer_norm_dispatch(const RowPlan &p, const float *in, float *out, const float *gamma, const float *beta,
                                int rows, int cols, float eps, cudaStream_t stream) {
    switch (p.slots) {
    case 1: layer_norm_launch<kGroup, 1>(p.vec, in, out, gamma, beta, rows, cols, eps, stream); break;
    case 2: layer_norm_launch<kGroup, 2>(p.vec, in, out, gamma, beta, rows, cols, eps, stream); break;
    case 4: layer_norm_launch<kGroup, 4>(p.vec, in, out, gamma, beta, rows, cols, eps, stream); break;
    default: layer_norm_launch<kGroup, 8>(p.vec, in, out, gamma, beta, rows, cols, eps, stream); break;
    }
}

} // namespace opworks::detail

namespace opworks::ops {

inline void layer_norm(const float *in, float *out, const float *gamma, const float *beta, int rows, int cols,
                       float eps = kLayerNormEps, cudaStream_t stream = nullptr) {
    detail::validate_matrix(rows, cols);
    detail::require(std::isfinite(eps) && eps > 0, "layer norm epsilon must be finite and positive");
    if (rows == 0)
        return;
    detail::require(cols > 0, "layer norm requires positive columns for nonempty rows");
    detail::require(in && out && gamma && beta, "layer norm requires non-null pointers");
    const bool aligned = detail::aligned16(in) && detail::aligned16(out) && detail::aligned16(gamma) &&
                         detail::aligned16(beta);
    const detail::RowPlan p = detail::plan_rows(cols, aligned);
    if (p.slots == 0)
        launch_async(stream, detail::layer_norm_rows_stream_kernel, rows, kThreads, in, out, gamma, beta, cols, eps);
    else if (p.group == 32)
        detail::layer_norm_dispatch<32>(p, in, out, gamma, beta, rows, cols, eps, stream);
    else
        detail::layer_norm_dispatch<kThreads>(p, in, out, gamma, beta, rows, cols, eps, stream);
}

} // namespace opworks::ops

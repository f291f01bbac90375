#pragma once

// ops::softmax — row-wise softmax over the last dim of a rows x cols matrix.
// Contract of OpWorks include/ops/softmax.cuh:36-43 (max-subtracted,
// expf, rows == 0 is a no-op, cols must be positive otherwise).
//
// B200 kernel: the row is read once into registers, max and sum(exp) are
// reduced in registers (warp per row up to 1024 columns, block per row up to
// 8192), and the result is written once: 8 bytes of HBM traffic per element.

#include "detail/rows.cuh"

namespace opworks::detail {

template <int kGroup, int kSlots, typename V>
__global__ void __launch_bounds__(kThreads) softmax_rows_kernel(const float *in, float *out, int rows, int cols) {
    using T = VecTraits<V>;
    constexpr int W = T::kWidth;
    const int64_t row = row_of_group<kGroup>();
    if (row >= rows)
        return; // whole warp leaves together (warp-per-row mode only)
    const int nv = cols / W;
    const V *src = reinterpret_cast<const V *>(in + row * cols);
    V *dst = reinterpret_cast<V *>(out + row * cols);
    const int r = RowGroup<kGroup>::rank();

    V x[kSlots];
    float m = kNegInf;
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
        const int idx = r + s * kGroup;
        if (idx < nv) {
            x[s] = src[idx];
#pragma unroll
            for (int i = 0; i < W; ++i)
                m = fmaxf(m, T::get(x[s], i));
        }
    }
    m = RowGroup<kGroup>::max(m);
    float sum = 0.f;
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
        const int idx = r + s * kGroup;
        if (idx < nv) {
#pragma unroll
            for (int i = 0; i < W; ++i) {
                const float e = expf(T::get(x[s], i) - m);
                T::set(x[s], i, e);
                sum += e;
            }
        }
    }
    sum = RowGroup<kGroup>::sum(sum);
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
        const int idx = r + s * kGroup;
        if (idx < nv) {
#pragma unroll
            for (int i = 0; i < W; ++i)
                T::set(x[s], i, T::get(x[s], i) / sum);
            dst[idx] = x[s];
        }
    }
}

// Rows longer than the register tile: one online (max, sum) pass, one write pass.
static __global__ void __launch_bounds__(kThreads) softmax_rows_stream_kernel(const float *in, float *out, int cols) {
    const float *src = in + static_cast<int64_t>(blockIdx.x) * cols;
    float *dst = out + static_cast<int64_t>(blockIdx.x) * cols;
    float m = kNegInf, s = 0.f;
    for (int j = threadIdx.x; j < cols; j += blockDim.x) {
        const float x = src[j];
        if (x > m) {
            s = s * expf(m - x) + 1.f;
            m = x;
        } else {
            s += expf(x - m);
        }
    }
    const float gm = block_reduce_all<ReduceMax>(m);
    const float gs = block_reduce_all<ReduceSum>(m == kNegInf ? 0.f : s * expf(m - gm));
    for (int j = threadIdx.x; j < cols; j += blockDim.x)
        dst[j] = expf(src[j] - gm) / gs;
}

template <int kGroup, int kSlots>
inline void softmax_dispatch_slots(bool vec, const float *in, float *out, int rows, int cols, cudaStream_t stream) {
    const int grid = row_grid(rows, kGroup);
    if (vec)
        launch_async(stream, softmax_rows_kernel<kGroup, kSlots, float4>, grid, kThreads, in, out, rows, cols);
    else
        launch_async(stream, softmax_rows_kernel<kGroup, kSlots, float>, grid, kThreads, in, out, rows, cols);
}

template <int kGroup>
inline void softmax_dispatch(const RowPlan &p, const float *in, float *out, int rows, int cols, cudaStream_t stream) {
    switch (p.slots) {
    case 1: softmax_dispatch_slots<kGroup, 1>(p.vec, in, out, rows, cols, stream); break;
    case 2: softmax_dispatch_slots<kGroup, 2>(p.vec, in, out, rows, cols, stream); break;
    case 4: softmax_dispatch_slots<kGroup, 4>(p.vec, in, out, rows, cols, stream); break;
    default: softmax_dispatch_slots<kGroup, 8>(p.vec, in, out, rows, cols, stream); break;
    }
}

} // namespace opworks::detail

namespace opworks::ops {

inline void softmax(const float *in, float *out, int rows, int cols, cudaStream_t stream = nullptr) {
    detail::validate_matrix(rows, cols);
    if (rows == 0)
        return;
    detail::require(cols > 0, "softmax requires positive columns for nonempty rows");
    detail::require(in && out, "softmax requires non-null pointers");
    const detail::RowPlan p = detail::plan_rows(cols, detail::aligned16(in) && detail::aligned16(out));
    if (p.slots == 0)
        launch_async(stream, detail::softmax_rows_stream_kernel, rows, kThreads, in, out, cols);
    else if (p.group == 32)
        detail::softmax_dispatch<32>(p, in, out, rows, cols, stream);
    else
        detail::softmax_dispatch<kThreads>(p, in, out, rows, cols, stream);
}

} // namespace opworks::ops

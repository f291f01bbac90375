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

// Warp per row, float4 columns (<= 1024 per row), on a grid of a few warps
// per SM slot that walk the rows with a stride: each warp loads its next row
// into a second register tile before it finishes the current one, so the
// stores of one row overlap the loads of the next (a one-row-per-warp grid
// runs as a single wave in which every warp loads, then computes, then
// stores at the same time, and HBM reads and writes do not overlap). The
// arithmetic is one exponential (SFU) per element and one reciprocal per row.
template <int kSlots>
__global__ void __launch_bounds__(kThreads) softmax_rows_pipe_kernel(const float *in, float *out, int64_t rows,
                                                                     int cols) {
    const int lane = threadIdx.x % kWarpSize;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (kThreads / kWarpSize);
    int64_t row = static_cast<int64_t>(blockIdx.x) * (kThreads / kWarpSize) + threadIdx.x / kWarpSize;
    const int nv = cols / 4;
    float4 x[kSlots], y[kSlots];
    auto load = [&](int64_t r, float4(&v)[kSlots]) {
        const float4 *src = reinterpret_cast<const float4 *>(in + r * cols);
#pragma unroll
        for (int s = 0; s < kSlots; ++s) {
            const int idx = lane + s * kWarpSize;
            v[s] = idx < nv ? src[idx] : make_float4(kNegInf, kNegInf, kNegInf, kNegInf);
        }
    };
    if (row < rows)
        load(row, x);
    for (; row < rows; row += warps) {
        if (row + warps < rows)
            load(row + warps, y);
        float m = kNegInf;
#pragma unroll
        for (int s = 0; s < kSlots; ++s)
            m = fmaxf(m, fmaxf(fmaxf(x[s].x, x[s].y), fmaxf(x[s].z, x[s].w)));
        m = warp_reduce<ReduceMax>(m);
        float sum = 0.f;
#pragma unroll
        for (int s = 0; s < kSlots; ++s) {
            x[s].x = __expf(x[s].x - m);
            x[s].y = __expf(x[s].y - m);
            x[s].z = __expf(x[s].z - m);
            x[s].w = __expf(x[s].w - m);
            sum += (x[s].x + x[s].y) + (x[s].z + x[s].w);
        }
        const float inv = 1.f / warp_reduce<ReduceSum>(sum);
        float4 *dst = reinterpret_cast<float4 *>(out + row * cols);
#pragma unroll
        for (int s = 0; s < kSlots; ++s) {
            const int idx = lane + s * kWarpSize;
            if (idx < nv)
                dst[idx] = make_float4(x[s].x * inv, x[s].y * inv, x[s].z * inv, x[s].w * inv);
        }
#pragma unroll
        for (int s = 0; s < kSlots; ++s)
            x[s] = y[s];
    }
}

template <int kSlots> inline void softmax_pipe_launch(const float *in, float *out, int rows, int cols, cudaStream_t stream) {
    constexpr auto kernel = softmax_rows_pipe_kernel<kSlots>;
    launch_async(stream, kernel, row_walk_grid<kernel>(rows), kThreads, in, out, int64_t(rows), cols);
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
    else if (p.group == 32 && p.vec) {
        switch (p.slots) {
        case 1: detail::softmax_pipe_launch<1>(in, out, rows, cols, stream); break;
        case 2: detail::softmax_pipe_launch<2>(in, out, rows, cols, stream); break;
        case 4: detail::softmax_pipe_launch<4>(in, out, rows, cols, stream); break;
        default: detail::softmax_pipe_launch<8>(in, out, rows, cols, stream); break;
        }
    } else if (p.group == 32)
        detail::softmax_dispatch<32>(p, in, out, rows, cols, stream);
    else
        detail::softmax_dispatch<kThreads>(p, in, out, rows, cols, stream);
}

} // namespace opworks::ops

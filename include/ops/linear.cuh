#pragma once

// ops::linear — Y[rows, out] = X[rows, in] @ W[out, in]^T with W in the HF
// [out, in] layout, fp32 activations, WT = float or __nv_bfloat16
// (OpWorks include/ops/linear.cuh:130-153; same checks and semantics).
//
// B200 paths:
//   rows == 1  HBM-streaming GEMV: x staged once per block in shared memory,
//              one warp per output row, 16-byte weight loads eight deep per
//              lane, warp-shuffle reduction. This is the decode path of the
//              fp32 (accurate) model.
//   rows > 1   tcgen05 GEMM. fp32 weights: split-precision TF32 (x3) so the
//              result stays fp32-accurate. bf16 weights: X is rounded to bf16
//              (as the reference's tensor-core path does) and one
//              kind::f16 MMA per K step.

#include <cuda_bf16.h>

#include "../core/cuda_utils.cuh"
#include "detail/operand_prep.cuh"
#include "embedding.cuh" // detail::to_f32
#include "gemm_sm100.cuh"

namespace opworks::detail {

template <typename WT> struct GemvVec;
template <> struct GemvVec<float> {
    static constexpr int kPer = 4; // weights per 16-byte load
    __device__ __forceinline__ static float dot(const uint4 &w, const float *xs) {
        const float4 v = *reinterpret_cast<const float4 *>(&w);
        const float4 a = *reinterpret_cast<const float4 *>(xs);
        return v.x * a.x + v.y * a.y + v.z * a.z + v.w * a.w;
    }
};
template <> struct GemvVec<__nv_bfloat16> {
    static constexpr int kPer = 8;
    __device__ __forceinline__ static float dot(const uint4 &w, const float *xs) {
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&w);
        const float4 a = *reinterpret_cast<const float4 *>(xs);
        const float4 b = *reinterpret_cast<const float4 *>(xs + 4);
        const float2 w0 = __bfloat1622float2(h[0]), w1 = __bfloat1622float2(h[1]);
        const float2 w2 = __bfloat1622float2(h[2]), w3 = __bfloat1622float2(h[3]);
        return w0.x * a.x + w0.y * a.y + w1.x * a.z + w1.y * a.w + w2.x * b.x + w2.y * b.y + w3.x * b.z + w3.y * b.w;
    }
};

// y[r][o] = sum_i x[r][i] W[o][i] for R <= 4 rows sharing every weight read.
// x rows are staged once per block in shared memory; one warp per output
// row, 16-byte weight loads eight deep per lane, warp-shuffle reduction.
// Requires in % kPer == 0 and 16-byte aligned W and x rows.
template <typename WT, int R>
__global__ void __launch_bounds__(kThreads)
    gemv_rows_kernel(const float *__restrict__ x, int64_t ldx, const WT *__restrict__ W, float *__restrict__ y,
                     int64_t ldy, int in, int out) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ float4 xs4[];
    float *xs = reinterpret_cast<float *>(xs4);
    for (int r = 0; r < R; ++r)
        for (int j = threadIdx.x; j < in / 4; j += blockDim.x)
            xs4[r * (in / 4) + j] = reinterpret_cast<const float4 *>(x + r * ldx)[j];
    __syncthreads();
    constexpr int kPer = GemvVec<WT>::kPer;
    const int nvec = in / kPer;
    const int lane = threadIdx.x % kWarpSize;
    const int warps_total = gridDim.x * (blockDim.x / kWarpSize);
    for (int row = blockIdx.x * (blockDim.x / kWarpSize) + threadIdx.x / kWarpSize; row < out; row += warps_total) {
        const uint4 *w = reinterpret_cast<const uint4 *>(W + static_cast<int64_t>(row) * in);
        // kDepth 16-byte loads per lane in flight per round trip (a row of
        // 2048 fp32 weights is two round trips); partial sums alternate
        // between two accumulators per row
        constexpr int kDepth = 8;
        float acc[R][2];
#pragma unroll
        for (int r = 0; r < R; ++r)
            acc[r][0] = acc[r][1] = 0.f;
        int v = lane;
        for (; v + (kDepth - 1) * kWarpSize < nvec; v += kDepth * kWarpSize) {
            uint4 a[kDepth];
#pragma unroll
            for (int d = 0; d < kDepth; ++d)
                a[d] = __ldg(w + v + d * kWarpSize);
#pragma unroll
            for (int d = 0; d < kDepth; ++d)
#pragma unroll
                for (int r = 0; r < R; ++r)
                    acc[r][d & 1] += GemvVec<WT>::dot(a[d], xs + r * in + (v + d * kWarpSize) * kPer);
        }
        for (; v < nvec; v += kWarpSize) {
            const uint4 a = __ldg(w + v);
#pragma unroll
            for (int r = 0; r < R; ++r)
                acc[r][0] += GemvVec<WT>::dot(a, xs + r * in + v * kPer);
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float t = warp_reduce<ReduceSum>(acc[r][0] + acc[r][1]);
            if (lane == 0)
                y[r * ldy + row] = t;
        }
    }
}

template <typename WT, int R>
inline void gemv_rows_launch_r(const float *x, int64_t ldx, const WT *W, float *y, int64_t ldy, int in, int out,
                               cudaStream_t stream) {
    const int rows_per_block = kThreads / kWarpSize;
    const int need = (out + rows_per_block - 1) / rows_per_block;
    const int cap = device_facts().sm_count * 8;
    const int grid = need < cap ? need : cap;
    const size_t smem = sizeof(float) * static_cast<size_t>(in) * R;
    static thread_local int attr_dev = -1;
    static thread_local size_t attr_bytes = 0;
    int dev = 0;
    OPWORKS_CUDA_CHECK(cudaGetDevice(&dev));
    if (smem > 48 * 1024 && (attr_dev != dev || attr_bytes < smem)) {
        OPWORKS_CUDA_CHECK(cudaFuncSetAttribute(gemv_rows_kernel<WT, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(smem)));
        attr_dev = dev;
        attr_bytes = smem;
    }
    launch_ex(gemv_rows_kernel<WT, R>, dim3(grid), dim3(kThreads), smem, stream, x, ldx, W, y, ldy, in, out);
}

inline bool gemv_rows_supported(int in, int rows, size_t kper) {
    return in % static_cast<int>(kper) == 0 && sizeof(float) * static_cast<size_t>(in) * rows <= 200 * 1024;
}

// rows in [1, 4]; vector path requirements as gemv_rows_kernel.
template <typename WT>
inline void gemv_rows_launch(const float *x, int64_t ldx, const WT *W, float *y, int64_t ldy, int rows, int in,
                             int out, cudaStream_t stream) {
    switch (rows) {
    case 1: gemv_rows_launch_r<WT, 1>(x, ldx, W, y, ldy, in, out, stream); break;
    case 2: gemv_rows_launch_r<WT, 2>(x, ldx, W, y, ldy, in, out, stream); break;
    case 3: gemv_rows_launch_r<WT, 3>(x, ldx, W, y, ldy, in, out, stream); break;
    default: gemv_rows_launch_r<WT, 4>(x, ldx, W, y, ldy, in, out, stream); break;
    }
}

// Any alignment / width: one warp per output row, scalar loads.
template <typename WT>
__global__ void __launch_bounds__(kThreads)
    gemv_scalar_kernel(const float *__restrict__ x, const WT *__restrict__ W, float *__restrict__ y, int in, int out) {
    const int lane = threadIdx.x % kWarpSize;
    const int warps_total = gridDim.x * (blockDim.x / kWarpSize);
    for (int row = blockIdx.x * (blockDim.x / kWarpSize) + threadIdx.x / kWarpSize; row < out; row += warps_total) {
        const WT *w = W + static_cast<int64_t>(row) * in;
        float acc = 0.f;
        for (int j = lane; j < in; j += kWarpSize)
            acc += x[j] * to_f32(w[j]);
        acc = warp_reduce<ReduceSum>(acc);
        if (lane == 0)
            y[row] = acc;
    }
}

template <typename WT>
inline void gemv_launch(const float *x, const WT *W, float *y, int in, int out, cudaStream_t stream) {
    constexpr int kPer = GemvVec<WT>::kPer;
    const bool vec = reinterpret_cast<uintptr_t>(W) % 16 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                     gemv_rows_supported(in, 1, kPer);
    if (!vec) {
        const int rows_per_block = kThreads / kWarpSize;
        const int need = (out + rows_per_block - 1) / rows_per_block;
        const int cap = device_facts().sm_count * 16;
        launch_async(stream, gemv_scalar_kernel<WT>, need < cap ? need : cap, kThreads, x, W, y, in, out);
        return;
    }
    gemv_rows_launch<WT>(x, in, W, y, out, 1, in, out, stream);
}

static __global__ void copy_bf16_rows_kernel(const __nv_bfloat16 *__restrict__ src, int rows, int cols,
                                             __nv_bfloat16 *__restrict__ dst, int64_t ld) {
    OPWORKS_GRID_LOOP(i, static_cast<int64_t>(rows) * ld) {
        const int64_t r = i / ld, c = i % ld;
        dst[i] = c < cols ? src[r * cols + c] : __float2bfloat16_rn(0.f);
    }
}

// Tensor-core Y = X @ W^T for bf16 weights and any row count.
inline void linear_bf16_tc(const float *X, const __nv_bfloat16 *W, float *Y, int rows, int in, int out,
                           cudaStream_t stream) {
    const int64_t ld = round_up(in, 8);
    const bool w_direct = ld == in && reinterpret_cast<uintptr_t>(W) % 16 == 0;
    const size_t x_bytes = sizeof(__nv_bfloat16) * static_cast<size_t>(rows) * ld;
    const size_t w_bytes = w_direct ? 0 : sizeof(__nv_bfloat16) * static_cast<size_t>(out) * ld;
    StreamScratch scratch(round_up(static_cast<int64_t>(x_bytes), 256) + w_bytes, stream);
    __nv_bfloat16 *xb = scratch.as<__nv_bfloat16>(0);
    const __nv_bfloat16 *wb = W;
    launch_async(stream, rows_to_bf16_kernel, grid_for(static_cast<int64_t>(rows) * ld), kThreads, X, rows, in,
                 static_cast<int64_t>(in), xb, ld);
    if (!w_direct) {
        __nv_bfloat16 *wp = scratch.as<__nv_bfloat16>(round_up(static_cast<int64_t>(x_bytes), 256));
        launch_async(stream, copy_bf16_rows_kernel, grid_for(static_cast<int64_t>(out) * ld), kThreads, W, out, in,
                     wp, ld);
        wb = wp;
    }
    sm100::GemmOperand feat{wb, nullptr, out, ld};
    sm100::GemmOperand tok{xb, nullptr, rows, ld};
    sm100::gemm_tn<sm100::GemmKind::kBF16>(feat, tok, in, Y, out, 1, 0, stream);
}

// Tensor-core Y = X @ W^T for fp32 weights in split-precision TF32.
inline void linear_f32_tc(const float *X, const float *W, float *Y, int rows, int in, int out, cudaStream_t stream) {
    const int64_t ld = round_up(in, 4);
    const size_t x_bytes = sizeof(float) * static_cast<size_t>(rows) * ld;
    const size_t w_bytes = sizeof(float) * static_cast<size_t>(out) * ld;
    StreamScratch scratch(2 * x_bytes + 2 * w_bytes, stream);
    float *x_hi = scratch.as<float>(0), *x_lo = scratch.as<float>(x_bytes);
    float *w_hi = scratch.as<float>(2 * x_bytes), *w_lo = scratch.as<float>(2 * x_bytes + w_bytes);
    split_rows_launch(stream, X, rows, in, static_cast<int64_t>(in), x_hi, x_lo, ld);
    split_rows_launch(stream, W, out, in, static_cast<int64_t>(in), w_hi, w_lo, ld);
    sm100::GemmOperand feat{w_hi, w_lo, out, ld};
    sm100::GemmOperand tok{x_hi, x_lo, rows, ld};
    sm100::gemm_tf32x3(feat, tok, in, Y, out, stream);
}

} // namespace opworks::detail

namespace opworks::ops {

template <typename WT>
inline void linear(const float *X, const WT *W, float *Y, int rows, int in_features, int out_features,
                   cudaStream_t stream = nullptr) {
    detail::validate_matrix(rows, in_features);
    detail::validate_matrix(out_features, in_features);
    detail::validate_matrix(rows, out_features);
    if (rows == 0 || out_features == 0)
        return;
    detail::require(X && W && Y, "linear requires non-null pointers");
    detail::require(in_features > 0, "linear requires a positive reduction dim");
    if (rows == 1) {
        detail::gemv_launch<WT>(X, W, Y, in_features, out_features, stream);
        return;
    }
    if constexpr (std::is_same_v<WT, __nv_bfloat16>)
        detail::linear_bf16_tc(X, W, Y, rows, in_features, out_features, stream);
    else
        detail::linear_f32_tc(X, W, Y, rows, in_features, out_features, stream);
}

} // namespace opworks::ops

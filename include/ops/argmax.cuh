#pragma once

// ops::argmax — index of the maximum of x[0..n), ties resolve to the lowest
// index, result stays on the device (OpWorks include/ops/argmax.cuh:59-63).
// The Llama runtime fuses greedy argmax into its sampler kernel; this is the
// standalone op (one 1024-thread block, 16-byte loads).

#include "../core/cuda_utils.cuh"

namespace opworks::detail {

__device__ __forceinline__ void argmax_merge(float &v, int &i, float ov, int oi) {
    if (ov > v || (ov == v && oi < i)) {
        v = ov;
        i = oi;
    }
}

// NaN is never selected over a number (comparisons with NaN are false).
__device__ __forceinline__ void warp_argmax(float &v, int &i) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(kFullWarpMask, v, off);
        const int oi = __shfl_xor_sync(kFullWarpMask, i, off);
        argmax_merge(v, i, ov, oi);
    }
}

static __global__ void __launch_bounds__(1024) argmax_kernel(const float *x, int n, int *out) {
    float best = kNegInf;
    int best_i = 0x7fffffff;
    const bool vec = reinterpret_cast<uintptr_t>(x) % 16 == 0;
    const int nv = vec ? n / 4 : 0;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    for (int v = threadIdx.x; v < nv; v += blockDim.x) {
        const float4 q = x4[v];
        argmax_merge(best, best_i, q.x, 4 * v);
        argmax_merge(best, best_i, q.y, 4 * v + 1);
        argmax_merge(best, best_i, q.z, 4 * v + 2);
        argmax_merge(best, best_i, q.w, 4 * v + 3);
    }
    for (int j = 4 * nv + threadIdx.x; j < n; j += blockDim.x)
        argmax_merge(best, best_i, x[j], j);
    warp_argmax(best, best_i);
    __shared__ float sv[32];
    __shared__ int si[32];
    const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
    if (lane == 0) {
        sv[warp] = best;
        si[warp] = best_i;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = (blockDim.x + 31) / 32;
        best = lane < nw ? sv[lane] : kNegInf;
        best_i = lane < nw ? si[lane] : 0x7fffffff;
        warp_argmax(best, best_i);
        if (lane == 0)
            out[0] = best_i;
    }
}

} // namespace opworks::detail

namespace opworks::ops {

inline void argmax(const float *x, int n, int *out, cudaStream_t stream = nullptr) {
    detail::require(n > 0, "argmax requires a nonempty input");
    detail::require(x && out, "argmax requires non-null pointers");
    launch_async(stream, detail::argmax_kernel, 1, kMaxThreadsPerBlock, x, n, out);
}

} // namespace opworks::ops

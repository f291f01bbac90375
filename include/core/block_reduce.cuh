#pragma once

// Warp- and block-wide reductions.
//
// block_reduce<Op>(v): result valid on thread 0. block_reduce_all<Op>(v):
// result valid on every thread. Same contract as OpWorks
// include/core/block_reduce.cuh:11-41 (1D block, a positive multiple of 32
// threads, whole-block participation). Unlike the original, back-to-back
// calls are safe without an extra barrier: each call fences the shared
// scratch before reusing it.

#include <cuda_runtime.h>

#include "config.cuh"

namespace opworks {

// Butterfly reduction: every lane ends with the warp-wide result.
template <typename Op> __device__ __forceinline__ float warp_reduce(float val) {
#pragma unroll
    for (int offset = kWarpSize / 2; offset > 0; offset >>= 1)
        val = Op::combine(val, __shfl_xor_sync(kFullWarpMask, val, offset));
    return val;
}

template <typename Op> __device__ float block_reduce(float val) {
    __shared__ float partial[kMaxThreadsPerBlock / kWarpSize];
    const int lane = threadIdx.x % kWarpSize;
    const int warp = threadIdx.x / kWarpSize;
    val = warp_reduce<Op>(val);
    __syncthreads(); // a previous call's readers are done with `partial`
    if (lane == 0)
        partial[warp] = val;
    __syncthreads();
    if (warp == 0) {
        const int nwarps = (blockDim.x + kWarpSize - 1) / kWarpSize;
        val = warp_reduce<Op>(lane < nwarps ? partial[lane] : Op::identity());
    }
    return val;
}

template <typename Op> __device__ float block_reduce_all(float val) {
    __shared__ float broadcast;
    const float r = block_reduce<Op>(val);
    if (threadIdx.x == 0)
        broadcast = r;
    __syncthreads();
    return broadcast;
}

} // namespace opworks

namespace opworks::detail {

struct ReduceSum {
    static __device__ __forceinline__ float identity() { return 0.f; }
    static __device__ __forceinline__ float combine(float a, float b) { return a + b; }
};
struct ReduceMax {
    static __device__ __forceinline__ float identity() { return kNegInf; }
    static __device__ __forceinline__ float combine(float a, float b) { return fmaxf(a, b); }
};

} // namespace opworks::detail

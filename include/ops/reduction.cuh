#pragma once

// ops::reduce<Op> — fold of n floats with a user (identity, combine) functor.
//
// API of OpWorks include/ops/reduction.cuh:34-67: reduction_workspace_size(n),
// an allocation-free overload taking an explicit workspace (graph-capture
// safe) and a convenience overload using stream-ordered allocation. n == 0
// writes Op::identity().
//
// B200 kernel: one pass. Up to 1024 blocks stream the input with 16-byte
// loads (eight in flight per thread) into four independent accumulators per
// thread; each block publishes
// its partial, and the last block to arrive (arrival counter in the
// workspace) folds the partials in block order, so the result is
// deterministic. The counter is cleared with a 4-byte memset node before the
// kernel, which keeps the sequence capturable in a CUDA graph.

#include "../core/block_reduce.cuh"
#include "../core/cuda_utils.cuh"
#include "../core/device_span.cuh"

namespace opworks::detail {

constexpr int kReduceMaxBlocks = 1024;
constexpr int kReduceElemsPerBlock = kThreads * 16; // 4 float4 per thread per pass

template <typename Op> __device__ __forceinline__ float reduce_range(const float *in, int64_t n) {
    // peel to 16-byte alignment so the bulk uses float4 loads
    const uintptr_t mis = reinterpret_cast<uintptr_t>(in) % 16;
    int64_t head = mis == 0 ? 0 : static_cast<int64_t>((16 - mis) / 4);
    head = head < n ? head : n;
    const int64_t n_vec = (n - head) / 4;
    const int64_t tail_begin = head + 4 * n_vec;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;

    float acc0 = Op::identity(), acc1 = Op::identity(), acc2 = Op::identity(), acc3 = Op::identity();
    for (int64_t i = tid; i < head; i += stride)
        acc0 = Op::combine(acc0, in[i]);
    for (int64_t i = tail_begin + tid; i < n; i += stride)
        acc1 = Op::combine(acc1, in[i]);
    const float4 *v4 = reinterpret_cast<const float4 *>(in + head);
    int64_t v = tid;
    // eight 16-byte loads in flight per thread per iteration (128 bytes):
    // the grid is one wave, so each thread's iterations are round trips
    constexpr int kUnroll = 8;
    for (; v + (kUnroll - 1) * stride < n_vec; v += kUnroll * stride) {
        float4 a[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
            a[u] = v4[v + u * stride];
#pragma unroll
        for (int u = 0; u < kUnroll; u += 2) {
            acc0 = Op::combine(acc0, Op::combine(a[u].x, a[u].y));
            acc1 = Op::combine(acc1, Op::combine(a[u].z, a[u].w));
            acc2 = Op::combine(acc2, Op::combine(a[u + 1].x, a[u + 1].y));
            acc3 = Op::combine(acc3, Op::combine(a[u + 1].z, a[u + 1].w));
        }
    }
    for (; v < n_vec; v += stride) {
        const float4 a = v4[v];
        acc0 = Op::combine(acc0, Op::combine(a.x, a.y));
        acc1 = Op::combine(acc1, Op::combine(a.z, a.w));
    }
    return Op::combine(Op::combine(acc0, acc1), Op::combine(acc2, acc3));
}

// partial == nullptr: single block writes out directly.
template <typename Op>
__global__ void __launch_bounds__(kThreads)
    reduce_onepass_kernel(const float *in, int64_t n, float *out, float *partial, unsigned int *arrivals) {
    float acc = n > 0 ? reduce_range<Op>(in, n) : Op::identity();
    acc = block_reduce<Op>(acc);
    if (partial == nullptr) {
        if (threadIdx.x == 0)
            out[0] = acc;
        return;
    }
    __shared__ bool is_last;
    if (threadIdx.x == 0) {
        partial[blockIdx.x] = acc;
        __threadfence();
        const unsigned int arrived = atomicAdd(arrivals, 1u);
        is_last = arrived == gridDim.x - 1;
    }
    __syncthreads();
    if (!is_last)
        return;
    __threadfence();
    float fold = Op::identity();
    const volatile float *vp = partial;
    for (int i = threadIdx.x; i < static_cast<int>(gridDim.x); i += blockDim.x)
        fold = Op::combine(fold, vp[i]);
    fold = block_reduce<Op>(fold);
    if (threadIdx.x == 0)
        out[0] = fold;
}

inline int reduce_block_count(int n) {
    int b = n / kReduceElemsPerBlock + (n % kReduceElemsPerBlock != 0 ? 1 : 0);
    return b < kReduceMaxBlocks ? b : kReduceMaxBlocks;
}

} // namespace opworks::detail

namespace opworks::ops {

// Workspace size in floats for reduce<Op>(in, out, n, workspace): partial
// slots plus one arrival counter. Inputs reduced by one block need none.
inline int reduction_workspace_size(int n) {
    const int blocks = detail::blocks_for(n);
    if (blocks <= 1)
        return 0;
    return (blocks < detail::kReduceMaxBlocks ? blocks : detail::kReduceMaxBlocks) + 1;
}

// Allocation-free asynchronous reduction. The workspace must stay alive until
// the stream reaches this work and must not be shared by concurrent
// reductions or overlap the input/output.
template <typename Op>
inline void reduce(const float *in, float *out, int n, DeviceSpan<float> workspace, cudaStream_t stream = nullptr) {
    const int needed = reduction_workspace_size(n);
    detail::require(out && (n == 0 || in), "reduction requires valid input/output pointers");
    detail::require(workspace.size() >= needed, "reduction workspace is too small");
    const int blocks = detail::reduce_block_count(n);
    if (blocks <= 1) {
        launch_async(stream, detail::reduce_onepass_kernel<Op>, 1, kThreads, in, static_cast<int64_t>(n), out,
                     static_cast<float *>(nullptr), static_cast<unsigned int *>(nullptr));
        return;
    }
    float *partial = workspace.data();
    unsigned int *arrivals = reinterpret_cast<unsigned int *>(workspace.data() + blocks);
    OPWORKS_CUDA_CHECK(cudaMemsetAsync(arrivals, 0, sizeof(unsigned int), stream));
    launch_async(stream, detail::reduce_onepass_kernel<Op>, blocks, kThreads, in, static_cast<int64_t>(n), out,
                 partial, arrivals);
}

// Convenience overload: scratch comes from the stream-ordered allocator and
// is released after the kernel (requires memory-pool support).
template <typename Op> inline void reduce(const float *in, float *out, int n, cudaStream_t stream = nullptr) {
    const int count = reduction_workspace_size(n);
    detail::require(out && (n == 0 || in), "reduction requires valid input/output pointers");
    float *scratch = nullptr;
    if (count != 0)
        OPWORKS_CUDA_CHECK(cudaMallocAsync(reinterpret_cast<void **>(&scratch), sizeof(float) * count, stream));
    reduce<Op>(in, out, n, DeviceSpan<float>(scratch, count), stream);
    if (scratch)
        OPWORKS_CUDA_CHECK(cudaFreeAsync(scratch, stream));
}

} // namespace opworks::ops

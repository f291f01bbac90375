#pragma once

// ops::map — unary and binary elementwise maps with a user functor.
//
// API and contracts of OpWorks include/ops/elementwise.cuh:63-77: asynchronous,
// n == 0 submits nothing, null pointers with n > 0 throw, exact in-place use
// is allowed, partial overlap is not. The functor is copied to the kernel by
// value, so stateful functors work.
//
// B200 kernel: each thread moves 32 bytes per input per iteration (two
// independent 16-byte loads) so an SM keeps enough bytes in flight to stream
// HBM3e. Pointers that share the same misalignment are peeled to a 16-byte
// boundary instead of dropping to the scalar path; only inputs whose
// alignments differ fall back to scalar accesses.

#include <cstdint>

#include "../core/cuda_utils.cuh"

namespace opworks::detail {

template <int kArity> struct MapArgs {
    const float *in[2];
    float *out;
    int64_t n;      // total elements
    int64_t head;   // scalar elements before the first aligned vector
    int64_t n_vec;  // float4 vectors after the head
};

template <int kArity, typename Op>
__device__ __forceinline__ float map_apply(const Op &op, const MapArgs<kArity> &a, int64_t i) {
    if constexpr (kArity == 1)
        return op(a.in[0][i]);
    else
        return op(a.in[0][i], a.in[1][i]);
}

template <int kArity, typename Op> __device__ __forceinline__ float4 map_apply4(const Op &op, float4 x, float4 y) {
    float4 r;
    if constexpr (kArity == 1) {
        r.x = op(x.x);
        r.y = op(x.y);
        r.z = op(x.z);
        r.w = op(x.w);
    } else {
        r.x = op(x.x, y.x);
        r.y = op(x.y, y.y);
        r.z = op(x.z, y.z);
        r.w = op(x.w, y.w);
    }
    return r;
}

template <int kArity, typename Op> __global__ void __launch_bounds__(kThreads) map_kernel(Op op, MapArgs<kArity> a) {
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;

    // scalar head / tail (also the whole range when alignments differ)
    const int64_t tail_begin = a.head + 4 * a.n_vec;
    for (int64_t i = tid; i < a.head; i += stride)
        a.out[i] = map_apply(op, a, i);
    for (int64_t i = tail_begin + tid; i < a.n; i += stride)
        a.out[i] = map_apply(op, a, i);

    const float4 *x4 = reinterpret_cast<const float4 *>(a.in[0] + a.head);
    const float4 *y4 = reinterpret_cast<const float4 *>(a.in[kArity - 1] + a.head);
    float4 *o4 = reinterpret_cast<float4 *>(a.out + a.head);
    int64_t v = tid;
    for (; v + stride < a.n_vec; v += 2 * stride) {
        const float4 x0 = x4[v], x1 = x4[v + stride];
        float4 y0 = x0, y1 = x1;
        if constexpr (kArity == 2) {
            y0 = y4[v];
            y1 = y4[v + stride];
        }
        o4[v] = map_apply4<kArity>(op, x0, y0);
        o4[v + stride] = map_apply4<kArity>(op, x1, y1);
    }
    if (v < a.n_vec) {
        const float4 x0 = x4[v];
        const float4 y0 = kArity == 2 ? y4[v] : x0;
        o4[v] = map_apply4<kArity>(op, x0, y0);
    }
}

template <int kArity, typename Op>
void map_launch(const Op &op, int n, float *out, cudaStream_t stream, const float *in0, const float *in1) {
    validate_size(n);
    if (n == 0)
        return;
    require(out != nullptr && in0 != nullptr && (kArity == 1 || in1 != nullptr), "map requires non-null pointers");
    MapArgs<kArity> a;
    a.in[0] = in0;
    a.in[1] = kArity == 2 ? in1 : in0;
    a.out = out;
    a.n = n;
    const uintptr_t mis = reinterpret_cast<uintptr_t>(out) % 16;
    const bool same = reinterpret_cast<uintptr_t>(in0) % 16 == mis &&
                      (kArity == 1 || reinterpret_cast<uintptr_t>(in1) % 16 == mis) && mis % 4 == 0;
    if (same && kPackSize == 4) {
        const int64_t head = mis == 0 ? 0 : static_cast<int64_t>((16 - mis) / 4);
        a.head = head < n ? head : n;
        a.n_vec = (n - a.head) / 4;
    } else {
        a.head = n; // scalar everywhere
        a.n_vec = 0;
    }
    const int64_t work = a.n_vec > 0 ? (a.n_vec + 1) / 2 : n;
    const int blocks = num_blocks_for(static_cast<int>(work < std::numeric_limits<int>::max() ? work : n));
    launch_async(stream, map_kernel<kArity, Op>, blocks, kThreads, op, a);
}

} // namespace opworks::detail

namespace opworks::ops {

// binary map: out[i] = op(a[i], b[i])
template <typename Op>
inline void map(const float *a, const float *b, float *out, int n, const Op &op = {}, cudaStream_t stream = nullptr) {
    detail::map_launch<2>(op, n, out, stream, a, b);
}

// unary map: out[i] = op(in[i])
template <typename Op>
inline void map(const float *in, float *out, int n, const Op &op = {}, cudaStream_t stream = nullptr) {
    detail::map_launch<1>(op, n, out, stream, in, nullptr);
}

} // namespace opworks::ops

#pragma once

// ops::add — out = a + b (out may alias a or b), OpWorks include/ops/add.cuh:18-25.
// 16-byte vectorised via ops::map's kernel.

#include "elementwise.cuh"

namespace opworks::detail {
struct AddOp {
    __device__ __forceinline__ float operator()(float a, float b) const { return a + b; }
};
} // namespace opworks::detail

namespace opworks::ops {

inline void add(const float *a, const float *b, float *out, int64_t n, cudaStream_t stream = nullptr) {
    detail::require(n >= 0, "add size must be nonnegative");
    if (n == 0)
        return;
    detail::require(a && b && out, "add requires non-null pointers");
    detail::require(n <= std::numeric_limits<int>::max(), "add input exceeds the supported INT_MAX elements");
    detail::map_launch<2>(detail::AddOp{}, static_cast<int>(n), out, stream, a, b);
}

} // namespace opworks::ops

#pragma once

// ops::swiglu — out = silu(gate) * up = gate / (1 + exp(-gate)) * up
// (OpWorks include/ops/swiglu.cuh:18-26). In the Llama runtime the SiLU-mul
// is fused into the consumer of the gate/up GEMM; this is the standalone op.

#include "elementwise.cuh"

namespace opworks::detail {
struct SwigluOp {
    __device__ __forceinline__ float operator()(float g, float u) const { return g / (1.f + expf(-g)) * u; }
};
} // namespace opworks::detail

namespace opworks::ops {

inline void swiglu(const float *gate, const float *up, float *out, int64_t n, cudaStream_t stream = nullptr) {
    detail::require(n >= 0, "swiglu size must be nonnegative");
    if (n == 0)
        return;
    detail::require(gate && up && out, "swiglu requires non-null pointers");
    detail::require(n <= std::numeric_limits<int>::max(), "swiglu input exceeds the supported INT_MAX elements");
    detail::map_launch<2>(detail::SwigluOp{}, static_cast<int>(n), out, stream, gate, up);
}

} // namespace opworks::ops

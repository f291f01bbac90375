#pragma once

// MatmulBuilder: validated GEMM configuration (transpose_a/b, bias,
// activation none/relu/gelu) handed to a callback
// (OpWorks include/builders/matmul.cuh:9-57).
//
// The original defines no kernel behind apply(fn); ops::matmul_launcher is a
// ready-made callback that runs it on the tcgen05 tensor cores in
// split-precision TF32 with bias and activation fused into the epilogue:
//   MatmulBuilder(a, b, c, M, N, K).transpose_b().bias(bias)
//       .activation(MatmulActivation::relu).apply(ops::matmul_launcher{});
// Shapes follow ops::mat_mul: C is M x K, the contraction dim is N; with
// transpose_a A is stored N x M, with transpose_b B is stored K x N.

#include "../ops/matmul.cuh"
#include "builder_common.cuh"

namespace opworks {

enum class MatmulActivation { none, relu, gelu };

class MatmulBuilder {
  public:
    MatmulBuilder(DeviceSpan<const float> a, DeviceSpan<const float> b, DeviceSpan<float> output, int m, int n, int k,
                  cudaStream_t stream = nullptr)
        : a_(a), b_(b), output_(output), m_(m), n_(n), k_(k), stream_(stream) {
        detail::validate_matrix(m, n);
        detail::validate_matrix(n, k);
        detail::validate_matrix(m, k);
        detail::require(a.size() >= m * n && b.size() >= n * k && output.size() >= m * k, "matmul buffer is too small");
    }
    MatmulBuilder &transpose_a(bool value = true) {
        transpose_a_ = value;
        return *this;
    }
    MatmulBuilder &transpose_b(bool value = true) {
        transpose_b_ = value;
        return *this;
    }
    MatmulBuilder &bias(DeviceSpan<const float> value) {
        bias_ = value;
        return *this;
    }
    MatmulBuilder &activation(MatmulActivation value) {
        activation_ = value;
        return *this;
    }
    bool transposed_a() const { return transpose_a_; }
    bool transposed_b() const { return transpose_b_; }
    DeviceSpan<const float> a() const { return a_; }
    DeviceSpan<const float> b() const { return b_; }
    DeviceSpan<float> output() const { return output_; }
    DeviceSpan<const float> bias() const { return bias_; }
    MatmulActivation activation() const { return activation_; }
    int m() const { return m_; }
    int n() const { return n_; }
    int k() const { return k_; }
    cudaStream_t stream() const { return stream_; }

    template <typename Fn> decltype(auto) apply(Fn &&fn) const { return apply_builder(*this, static_cast<Fn &&>(fn)); }

  private:
    DeviceSpan<const float> a_, b_;
    DeviceSpan<float> output_;
    DeviceSpan<const float> bias_;
    int m_, n_, k_;
    bool transpose_a_ = false, transpose_b_ = false;
    MatmulActivation activation_ = MatmulActivation::none;
    cudaStream_t stream_;
};

namespace detail {

// bias[col] + activation, applied per output element (col = feature index).
struct BiasActivation {
    const float *bias;
    int act; // 0 none, 1 relu, 2 gelu (erf form)
    __device__ __forceinline__ float operator()(float v, int, int col) const {
        if (bias)
            v += bias[col];
        if (act == 1)
            return fmaxf(v, 0.f);
        if (act == 2)
            return 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
        return v;
    }
};

template <typename Epi> __global__ void fill_positional_kernel(float *out, int rows, int cols, Epi epi) {
    OPWORKS_GRID_LOOP(i, static_cast<int64_t>(rows) * cols) {
        out[i] = epi(0.f, static_cast<int>(i / cols), static_cast<int>(i % cols));
    }
}

} // namespace detail

namespace ops {

struct matmul_launcher {
    void operator()(const MatmulBuilder &g) const {
        const int M = g.m(), N = g.n(), K = g.k();
        if (M == 0 || K == 0)
            return;
        detail::require(g.bias().size() == 0 || g.bias().size() >= K, "matmul bias must cover the output columns");
        const detail::BiasActivation epi{g.bias().size() ? g.bias().data() : nullptr,
                                         static_cast<int>(g.activation())};
        cudaStream_t stream = g.stream();
        const int64_t out_elems = static_cast<int64_t>(M) * K;
        float *C = g.output().data();
        if (N == 0) {
            // empty contraction: every element is epilogue(0 + bias)
            launch_async(stream, detail::fill_positional_kernel<detail::BiasActivation>, detail::grid_for(out_elems),
                         kThreads, C, M, K, epi);
            return;
        }
        const int64_t ld = detail::round_up(N, 4);
        const size_t a_bytes = sizeof(float) * static_cast<size_t>(M) * ld;
        const size_t b_bytes = sizeof(float) * static_cast<size_t>(K) * ld;
        detail::StreamScratch scratch(2 * a_bytes + 2 * b_bytes, stream);
        float *a_hi = scratch.as<float>(0), *a_lo = scratch.as<float>(a_bytes);
        float *bt_hi = scratch.as<float>(2 * a_bytes), *bt_lo = scratch.as<float>(2 * a_bytes + b_bytes);
        // token operand: A as [M][N] K-major
        if (!g.transposed_a())
            detail::split_rows_launch(stream, g.a().data(), M, N, static_cast<int64_t>(N), a_hi, a_lo, ld);
        else
            launch_async(stream, detail::split_cols_t_kernel,
                         dim3(detail::blocks_for(M, 32), detail::blocks_for(static_cast<int>(ld), 32)), dim3(32, 8),
                         g.a().data(), N, M, a_hi, a_lo, ld);
        // feature operand: B^T as [K][N] K-major
        if (!g.transposed_b())
            launch_async(stream, detail::split_cols_t_kernel,
                         dim3(detail::blocks_for(K, 32), detail::blocks_for(static_cast<int>(ld), 32)), dim3(32, 8),
                         g.b().data(), N, K, bt_hi, bt_lo, ld);
        else
            detail::split_rows_launch(stream, g.b().data(), K, N, static_cast<int64_t>(N), bt_hi, bt_lo, ld);
        sm100::GemmOperand feat{bt_hi, bt_lo, K, ld};
        sm100::GemmOperand tok{a_hi, a_lo, M, ld};
        sm100::gemm_tf32x3(feat, tok, N, C, K, stream, epi);
    }
};

} // namespace ops

} // namespace opworks

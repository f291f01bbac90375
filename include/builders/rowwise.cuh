#pragma once

// RowwiseBuilder: a validated row-operation configuration (softmax,
// layer_norm or rms_norm over a rows x cols row-major matrix) handed to a
// launcher callback. Contract: OpWorks include/builders/rowwise.cuh:11-63
// (factory names and defaults, accessor names, std::invalid_argument on bad
// sizes, a non-finite or non-positive eps, or a missing parameter).
//
// ops::rowwise_launcher is the ready-made callback that runs this library's
// sm_100a row kernels:
//   RowwiseBuilder::rms_norm(in, out, w, rows, cols).apply(ops::rowwise_launcher{});

#include <cmath>

#include "../ops/layer_norm.cuh"
#include "../ops/rms_norm.cuh"
#include "../ops/softmax.cuh"
#include "builder_common.cuh"

namespace opworks {

enum class RowwiseOp { softmax, layer_norm, rms_norm };

class RowwiseBuilder {
  public:
    static RowwiseBuilder softmax(DeviceSpan<const float> input, DeviceSpan<float> output, int rows, int cols,
                                  cudaStream_t stream = nullptr) {
        Spec s{RowwiseOp::softmax, input, output};
        s.rows = rows;
        s.cols = cols;
        s.stream = stream;
        return RowwiseBuilder(s);
    }
    static RowwiseBuilder layer_norm(DeviceSpan<const float> input, DeviceSpan<float> output,
                                     DeviceSpan<const float> gamma, DeviceSpan<const float> beta, int rows, int cols,
                                     float eps = kLayerNormEps, cudaStream_t stream = nullptr) {
        Spec s{RowwiseOp::layer_norm, input, output};
        s.scale = gamma.data();
        s.shift = beta.data();
        s.rows = rows;
        s.cols = cols;
        s.eps = eps;
        s.stream = stream;
        return RowwiseBuilder(s);
    }
    static RowwiseBuilder rms_norm(DeviceSpan<const float> input, DeviceSpan<float> output,
                                   DeviceSpan<const float> weight, int rows, int cols, float eps = kLayerNormEps,
                                   cudaStream_t stream = nullptr) {
        Spec s{RowwiseOp::rms_norm, input, output};
        s.scale = weight.data();
        s.rows = rows;
        s.cols = cols;
        s.eps = eps;
        s.stream = stream;
        return RowwiseBuilder(s);
    }

    RowwiseOp op() const { return spec_.op; }
    DeviceSpan<const float> input() const { return spec_.input; }
    DeviceSpan<float> output() const { return spec_.output; }
    const float *parameter() const { return spec_.scale; } // gamma (layer_norm) or weight (rms_norm)
    const float *beta() const { return spec_.shift; }
    int rows() const { return spec_.rows; }
    int cols() const { return spec_.cols; }
    float epsilon() const { return spec_.eps; }
    cudaStream_t stream() const { return spec_.stream; }

    template <typename Fn> decltype(auto) apply(Fn &&fn) const { return apply_builder(*this, std::forward<Fn>(fn)); }

  private:
    struct Spec {
        RowwiseOp op;
        DeviceSpan<const float> input;
        DeviceSpan<float> output;
        const float *scale = nullptr;
        const float *shift = nullptr;
        int rows = 0, cols = 0;
        float eps = kLayerNormEps;
        cudaStream_t stream = nullptr;
    };

    explicit RowwiseBuilder(const Spec &s) : spec_(s) {
        detail::validate_matrix(s.rows, s.cols);
        const int64_t elems = static_cast<int64_t>(s.rows) * s.cols;
        detail::require(s.input.size() >= elems && s.output.size() >= elems, "rowwise buffer is too small");
        detail::require(s.rows == 0 || s.cols > 0, "rowwise columns must be positive");
        detail::require(std::isfinite(s.eps) && s.eps > 0, "rowwise epsilon must be finite and positive");
        const bool empty_rows = s.cols == 0;
        if (s.op != RowwiseOp::softmax)
            detail::require(s.scale != nullptr || empty_rows, "rowwise parameter is required");
        if (s.op == RowwiseOp::layer_norm)
            detail::require(s.shift != nullptr || empty_rows, "layer norm beta is required");
    }

    Spec spec_;
};

namespace ops {

// Callback for RowwiseBuilder::apply that launches the matching kernel.
struct rowwise_launcher {
    void operator()(const RowwiseBuilder &b) const {
        const float *in = b.input().data();
        float *out = b.output().data();
        if (b.op() == RowwiseOp::softmax)
            softmax(in, out, b.rows(), b.cols(), b.stream());
        else if (b.op() == RowwiseOp::layer_norm)
            layer_norm(in, out, b.parameter(), b.beta(), b.rows(), b.cols(), b.epsilon(), b.stream());
        else
            rms_norm(in, b.parameter(), out, b.rows(), b.cols(), b.epsilon(), b.stream());
    }
};

} // namespace ops

} // namespace opworks

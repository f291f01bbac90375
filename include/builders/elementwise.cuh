#pragma once

// ElementwiseBuilder: out = op(in) or op(lhs, rhs) into a fresh DeviceBuffer,
// through ops::map (16-byte vector path when every pointer allows it).
//
// Contract (OpWorks include/builders/elementwise.cuh:8-43, README.md:80-112):
// the builder borrows its inputs, so constructing it from a DeviceBuffer that
// dies at the end of the full expression is refused at compile time; the
// functor's kArity must match the number of inputs (std::invalid_argument
// otherwise); a stateful functor is passed by value to the kernel.

#include <array>

#include "../core/device_buffer.cuh"
#include "../ops/elementwise.cuh"

namespace opworks {

class ElementwiseBuilder {
  public:
    explicit ElementwiseBuilder(DeviceSpan<const float> in) : inputs_{in, {}}, arity_(1) {}
    ElementwiseBuilder(DeviceSpan<const float> lhs, DeviceSpan<const float> rhs) : inputs_{lhs, rhs}, arity_(2) {
        detail::require(lhs.size() == rhs.size(), "elementwise inputs must have equal lengths");
    }
    explicit ElementwiseBuilder(const DeviceBuffer &in) : ElementwiseBuilder(in.view()) {}
    ElementwiseBuilder(const DeviceBuffer &lhs, const DeviceBuffer &rhs) : ElementwiseBuilder(lhs.view(), rhs.view()) {}

    // temporaries would leave the builder pointing at freed memory
    ElementwiseBuilder(const DeviceBuffer &&) = delete;
    ElementwiseBuilder(const DeviceBuffer &&, const DeviceBuffer &) = delete;
    ElementwiseBuilder(const DeviceBuffer &, const DeviceBuffer &&) = delete;
    ElementwiseBuilder(const DeviceBuffer &&, const DeviceBuffer &&) = delete;

    int arity() const { return arity_; }
    int size() const { return inputs_[0].size(); }

    // Allocates the result and launches asynchronously on `stream`.
    template <typename Op> DeviceBuffer apply(const Op &op = Op{}, cudaStream_t stream = nullptr) const {
        static_assert(Op::kArity == 1 || Op::kArity == 2, "elementwise arity must be 1 or 2");
        detail::require(Op::kArity == arity_, "functor arity does not match builder inputs");
        DeviceBuffer result(size());
        launch(op, result.data(), stream);
        return result;
    }

  private:
    template <typename Op> void launch(const Op &op, float *out, cudaStream_t stream) const {
        const float *first = inputs_[0].data();
        if constexpr (Op::kArity == 1)
            ops::map(first, out, size(), op, stream);
        else
            ops::map(first, inputs_[1].data(), out, size(), op, stream);
    }

    std::array<DeviceSpan<const float>, 2> inputs_;
    int arity_;
};

} // namespace opworks

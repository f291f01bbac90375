#pragma once

// ReductionBuilder: folds a borrowed input with a reduction functor into a
// one-element DeviceBuffer, through ops::reduce (identity for an empty input).
// Contract: OpWorks include/builders/reduction.cuh:8-28 (rvalue owners are
// refused; an optional caller workspace of reduction_workspace_size(n)
// floats avoids the per-call scratch allocation).

#include "../core/device_buffer.cuh"
#include "../ops/reduction.cuh"

namespace opworks {

class ReductionBuilder {
  public:
    explicit ReductionBuilder(DeviceSpan<const float> in) : in_(in) {}
    explicit ReductionBuilder(const DeviceBuffer &in) : in_(in.view()) {}
    ReductionBuilder(const DeviceBuffer &&) = delete;

    template <typename Op> DeviceBuffer apply(cudaStream_t stream = nullptr) const {
        return fold<Op>(nullptr, stream);
    }
    template <typename Op> DeviceBuffer apply(DeviceSpan<float> workspace, cudaStream_t stream = nullptr) const {
        return fold<Op>(&workspace, stream);
    }

  private:
    template <typename Op> DeviceBuffer fold(const DeviceSpan<float> *workspace, cudaStream_t stream) const {
        DeviceBuffer result(1);
        if (workspace)
            ops::reduce<Op>(in_.data(), result.data(), in_.size(), *workspace, stream);
        else
            ops::reduce<Op>(in_.data(), result.data(), in_.size(), stream);
        return result;
    }

    DeviceSpan<const float> in_;
};

} // namespace opworks

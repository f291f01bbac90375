#pragma once

// The callback boundary of the configuration builders (RowwiseBuilder,
// MatmulBuilder). A configuration builder only validates and records one
// operation; apply(fn) passes the finished, immutable configuration to a
// launcher and returns whatever the launcher returns, so callers choose the
// kernel (ops::rowwise_launcher, ops::matmul_launcher, or their own).
// Contract: OpWorks include/builders/builder_common.cuh:7-9.

#include <functional>
#include <utility>

#include "../core/device_span.cuh"

namespace opworks {

template <typename Builder, typename Fn> decltype(auto) apply_builder(const Builder &builder, Fn &&fn) {
    return std::invoke(std::forward<Fn>(fn), builder);
}

} // namespace opworks

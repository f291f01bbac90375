#pragma once

// Shared callback boundary of the configuration builders: apply(fn) returns
// fn(builder) (OpWorks include/builders/builder_common.cuh:7-9).

#include "../core/device_span.cuh"

namespace opworks {

template <typename Builder, typename Fn> decltype(auto) apply_builder(const Builder &builder, Fn &&fn) {
    return static_cast<Fn &&>(fn)(builder);
}

} // namespace opworks

#pragma once

// Non-owning, const-correct view of device memory (float32 or int32).
// Contract as in OpWorks include/core/device_span.cuh:10-30: a nonempty span
// needs a pointer; DeviceSpan<T> converts to DeviceSpan<const T>, not back.

#include <type_traits>

#include "cuda_utils.cuh"

namespace opworks {

template <typename T> class DeviceSpan {
    using Element = std::remove_const_t<T>;
    static_assert(std::is_same_v<Element, float> || std::is_same_v<Element, int>,
                  "device spans support float32 and int32");

  public:
    DeviceSpan() = default;
    DeviceSpan(T *data, int size) : data_(data), size_(size) {
        detail::validate_size(size);
        detail::require(size == 0 || data != nullptr, "nonempty span requires a pointer");
    }

    template <typename U, std::enable_if_t<std::is_convertible_v<U *, T *>, int> = 0>
    DeviceSpan(DeviceSpan<U> other) : data_(other.data()), size_(other.size()) {}

    T *data() const { return data_; }
    int size() const { return size_; }

  private:
    T *data_ = nullptr;
    int size_ = 0;
};

} // namespace opworks

#pragma once

// RAII device allocation for the runtime's element types (float, int32_t,
// __nv_bfloat16, uint16_t for 16-bit tensor-core operands whose format is
// kept beside them, uint8_t for raw byte pools), 64-bit sizes. API of
// OpWorks include/core/typed_device_buffer.cuh:15-92.

#include <cstdint>
#include <cuda_bf16.h>
#include <type_traits>
#include <utility>
#include <vector>

#include "device_span.cuh"

namespace opworks {

template <typename T> class TypedDeviceBuffer {
    static_assert(std::is_same_v<T, float> || std::is_same_v<T, int32_t> || std::is_same_v<T, __nv_bfloat16> ||
                      std::is_same_v<T, uint16_t> || std::is_same_v<T, uint8_t>,
                  "TypedDeviceBuffer supports float, int32_t, __nv_bfloat16, uint16_t and uint8_t");

  public:
    TypedDeviceBuffer() = default;
    explicit TypedDeviceBuffer(int64_t n) : n_(n) {
        detail::require(n >= 0, "size must be nonnegative");
        if (n_ > 0)
            OPWORKS_CUDA_CHECK(cudaMalloc(reinterpret_cast<void **>(&ptr_), sizeof(T) * static_cast<size_t>(n_)));
    }
    ~TypedDeviceBuffer() { release(); }

    TypedDeviceBuffer(const TypedDeviceBuffer &) = delete;
    TypedDeviceBuffer &operator=(const TypedDeviceBuffer &) = delete;
    TypedDeviceBuffer(TypedDeviceBuffer &&other) noexcept
        : ptr_(std::exchange(other.ptr_, nullptr)), n_(std::exchange(other.n_, 0)) {}
    TypedDeviceBuffer &operator=(TypedDeviceBuffer &&other) noexcept {
        if (this != &other) {
            release();
            ptr_ = std::exchange(other.ptr_, nullptr);
            n_ = std::exchange(other.n_, 0);
        }
        return *this;
    }

    static TypedDeviceBuffer from_host(const std::vector<T> &h, cudaStream_t stream = nullptr) {
        return from_host(h.data(), static_cast<int64_t>(h.size()), stream);
    }

    static TypedDeviceBuffer from_host(const T *data, int64_t n, cudaStream_t stream = nullptr) {
        TypedDeviceBuffer buf(n);
        if (n > 0) {
            OPWORKS_CUDA_CHECK(cudaMemcpyAsync(buf.ptr_, data, sizeof(T) * static_cast<size_t>(n),
                                               cudaMemcpyHostToDevice, stream));
            synchronize(stream);
        }
        return buf;
    }

    std::vector<T> to_host(cudaStream_t stream = nullptr) const {
        std::vector<T> h(static_cast<size_t>(n_));
        if (n_ > 0) {
            OPWORKS_CUDA_CHECK(cudaMemcpyAsync(h.data(), ptr_, sizeof(T) * h.size(), cudaMemcpyDeviceToHost, stream));
            synchronize(stream);
        }
        return h;
    }

    T to_host_scalar(cudaStream_t stream = nullptr) const {
        detail::require(n_ == 1, "scalar copy requires exactly one element");
        return to_host(stream)[0];
    }

    T *data() { return ptr_; }
    const T *data() const { return ptr_; }
    int64_t size() const { return n_; }

  private:
    void release() {
        if (ptr_)
            cudaFree(ptr_);
        ptr_ = nullptr;
        n_ = 0;
    }
    T *ptr_ = nullptr;
    int64_t n_ = 0;
};

} // namespace opworks

#pragma once

// RAII fp32 device allocation (OpWorks include/core/device_buffer.cuh:9-81):
// move-only, empty buffers own no memory, host copies block until done,
// view() hands out a span whose constness follows the owner and is refused
// on temporaries.

#include <utility>
#include <vector>

#include "device_span.cuh"

namespace opworks {

class DeviceBuffer {
  public:
    DeviceBuffer() = default;
    explicit DeviceBuffer(int n) : n_(n) {
        detail::validate_size(n);
        if (n_ > 0)
            OPWORKS_CUDA_CHECK(cudaMalloc(reinterpret_cast<void **>(&ptr_), sizeof(float) * static_cast<size_t>(n_)));
    }
    ~DeviceBuffer() { release(); }

    DeviceBuffer(const DeviceBuffer &) = delete;
    DeviceBuffer &operator=(const DeviceBuffer &) = delete;
    DeviceBuffer(DeviceBuffer &&other) noexcept
        : ptr_(std::exchange(other.ptr_, nullptr)), n_(std::exchange(other.n_, 0)) {}
    DeviceBuffer &operator=(DeviceBuffer &&other) noexcept {
        if (this != &other) {
            release();
            ptr_ = std::exchange(other.ptr_, nullptr);
            n_ = std::exchange(other.n_, 0);
        }
        return *this;
    }

    static DeviceBuffer from_host(const std::vector<float> &h, cudaStream_t stream = nullptr) {
        detail::require(h.size() <= static_cast<size_t>(std::numeric_limits<int>::max()),
                        "buffer exceeds the supported INT_MAX elements");
        DeviceBuffer buf(static_cast<int>(h.size()));
        if (!h.empty()) {
            OPWORKS_CUDA_CHECK(
                cudaMemcpyAsync(buf.ptr_, h.data(), sizeof(float) * h.size(), cudaMemcpyHostToDevice, stream));
            synchronize(stream);
        }
        return buf;
    }

    std::vector<float> to_host(cudaStream_t stream = nullptr) const {
        std::vector<float> h(static_cast<size_t>(n_));
        if (n_ > 0) {
            OPWORKS_CUDA_CHECK(cudaMemcpyAsync(h.data(), ptr_, sizeof(float) * h.size(), cudaMemcpyDeviceToHost, stream));
            synchronize(stream);
        }
        return h;
    }

    float to_host_scalar(cudaStream_t stream = nullptr) const {
        detail::require(n_ == 1, "scalar copy requires exactly one element");
        return to_host(stream)[0];
    }

    DeviceSpan<float> view() & { return {ptr_, n_}; }
    DeviceSpan<const float> view() const & { return {ptr_, n_}; }
    DeviceSpan<float> view() && = delete;
    DeviceSpan<const float> view() const && = delete;

    float *data() { return ptr_; }
    const float *data() const { return ptr_; }
    int size() const { return n_; }

  private:
    void release() {
        if (ptr_)
            cudaFree(ptr_);
        ptr_ = nullptr;
        n_ = 0;
    }
    float *ptr_ = nullptr;
    int n_ = 0;
};

} // namespace opworks

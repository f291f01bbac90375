#pragma once

// Error handling, argument contracts, grid sizing and launch helpers.
//
// Public names and contracts follow OpWorks include/core/cuda_utils.cuh:
//   OPWORKS_CUDA_CHECK aborts on a CUDA error (:13-21), detail::require throws
//   std::invalid_argument (:29-32), num_blocks_for caps the grid at
//   SMs x (max threads per SM / kThreads) x kNumWaves, cached per device and
//   host thread (:56-74), launch_async / launch / launch_sync / synchronize
//   (:93-118) and the stride-loop macros (:76-90).

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <limits>
#include <stdexcept>
#include <cuda_runtime.h>

#include "config.cuh"

#define OPWORKS_CUDA_CHECK(expr)                                                                                       \
    do {                                                                                                               \
        const cudaError_t opw_status_ = (expr);                                                                        \
        if (opw_status_ != cudaSuccess) {                                                                              \
            std::fprintf(stderr, "[OpWorks] CUDA error %s at %s:%d: %s\n", #expr, __FILE__, __LINE__,                  \
                         cudaGetErrorString(opw_status_));                                                             \
            std::abort();                                                                                              \
        }                                                                                                              \
    } while (0)

namespace opworks {

namespace detail {

inline void require(bool condition, const char *message) {
    if (!condition)
        throw std::invalid_argument(message);
}

inline void validate_size(int n) { require(n >= 0, "size must be nonnegative"); }

inline void validate_matrix(int rows, int cols) {
    validate_size(rows);
    validate_size(cols);
    require(static_cast<int64_t>(rows) * static_cast<int64_t>(cols) <= std::numeric_limits<int>::max(),
            "matrix exceeds the supported INT_MAX elements");
}

// Overflow-free ceil(n / threads).
inline int blocks_for(int n, int threads = kThreads) {
    validate_size(n);
    require(threads > 0, "block size must be positive");
    return n / threads + (n % threads != 0 ? 1 : 0);
}

struct DeviceFacts {
    int device = -1;
    int sm_count = 0;
    int max_threads_per_sm = 0;
    int max_grid_blocks = 0;
};

// Per host thread, per device: queried once, then served from a small table
// (a process uses at most a handful of devices).
inline const DeviceFacts &device_facts() {
    int dev = 0;
    OPWORKS_CUDA_CHECK(cudaGetDevice(&dev));
    constexpr int kSlots = 16;
    static thread_local DeviceFacts table[kSlots];
    DeviceFacts &slot = table[dev % kSlots];
    if (slot.device != dev) {
        DeviceFacts f;
        f.device = dev;
        OPWORKS_CUDA_CHECK(cudaDeviceGetAttribute(&f.sm_count, cudaDevAttrMultiProcessorCount, dev));
        OPWORKS_CUDA_CHECK(cudaDeviceGetAttribute(&f.max_threads_per_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev));
        f.max_grid_blocks = f.sm_count * (f.max_threads_per_sm / kThreads) * kNumWaves;
        slot = f;
    }
    return slot;
}

} // namespace detail

// Enough blocks of kThreads to cover n, capped at kNumWaves waves of resident
// blocks on the current device.
inline int num_blocks_for(int n) {
    detail::validate_size(n);
    if (n == 0)
        return 0;
    const int cap = detail::device_facts().max_grid_blocks;
    const int need = detail::blocks_for(n);
    return need < cap ? need : cap;
}

// Grid-stride loop over [0, n) for a 1D launch.
#define OPWORKS_GRID_LOOP(i, n)                                                                                        \
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < (n);                             \
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)

// Block-stride loop over [0, n) for a 1D block.
#define OPWORKS_BLOCK_LOOP(i, n) for (int64_t i = threadIdx.x; i < (n); i += blockDim.x)

// Block-stride loop over [0, n) using the flattened id of a 1D/2D/3D block.
#define OPWORKS_BLOCK_LOOP_FLAT(i, n)                                                                                  \
    for (int i = static_cast<int>(threadIdx.x + blockDim.x * (threadIdx.y + blockDim.y * threadIdx.z)); i < (n);       \
         i += static_cast<int>(blockDim.x * blockDim.y * blockDim.z))

// Enqueue `kernel` on `stream`; only launch errors are checked here. Execution
// errors surface at the next synchronize / blocking copy.
template <typename... Params, typename... Args>
inline void launch_async(cudaStream_t stream, void (*kernel)(Params...), dim3 grid, dim3 block, Args... args) {
    detail::require(grid.x != 0 && grid.y != 0 && grid.z != 0 && block.x != 0 && block.y != 0 && block.z != 0,
                    "launch dimensions must be positive");
    kernel<<<grid, block, 0, stream>>>(args...);
    OPWORKS_CUDA_CHECK(cudaGetLastError());
}

inline void synchronize(cudaStream_t stream = nullptr) { OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream)); }

// ------------------------------------------------ programmatic dependent launch
//
// Launches made on a host thread while a PdlScope is active carry the
// programmatic-stream-serialization attribute: the next kernel in the stream
// may be scheduled as soon as every CTA of the current one has called
// pdl_trigger(), so its prologue (barrier setup, TMEM allocation, weight
// prefetch) overlaps the current kernel's tail. Every kernel launched that
// way calls pdl_wait() before it touches memory that an earlier kernel of the
// stream writes or reads; pdl_wait() returns once those kernels completed and
// their writes are visible. Both are no-ops for an ordinary launch.
namespace detail {
inline bool &pdl_flag() {
    static thread_local bool on = false;
    return on;
}
} // namespace detail

class PdlScope {
  public:
    explicit PdlScope(bool on) : prev_(detail::pdl_flag()) { detail::pdl_flag() = on; }
    ~PdlScope() { detail::pdl_flag() = prev_; }
    PdlScope(const PdlScope &) = delete;
    PdlScope &operator=(const PdlScope &) = delete;

  private:
    bool prev_;
};

__device__ __forceinline__ void pdl_wait() {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
    asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}
__device__ __forceinline__ void pdl_trigger() {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
}

// cudaLaunchKernelEx with the calling thread's PDL policy.
template <typename... Params, typename... Args>
inline void launch_ex(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      Args &&...args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    if (detail::pdl_flag()) {
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    OPWORKS_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...));
}

// Same with a runtime thread-block cluster shape (1 x 1 x 1 = no cluster).
template <typename... Params, typename... Args>
inline void launch_ex_cluster(void (*kernel)(Params...), dim3 grid, dim3 cluster, dim3 block, size_t smem,
                              cudaStream_t stream, Args &&...args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int n = 0;
    if (cluster.x * cluster.y * cluster.z > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = cluster.x;
        attr[n].val.clusterDim.y = cluster.y;
        attr[n].val.clusterDim.z = cluster.z;
        ++n;
    }
    if (detail::pdl_flag()) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cfg.attrs = n ? attr : nullptr;
    cfg.numAttrs = static_cast<unsigned>(n);
    OPWORKS_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...));
}

template <typename... Params, typename... Args>
inline void launch(void (*kernel)(Params...), dim3 grid, dim3 block, Args... args) {
    launch_async(nullptr, kernel, grid, block, args...);
}

template <typename... Params, typename... Args>
inline void launch_sync(cudaStream_t stream, void (*kernel)(Params...), dim3 grid, dim3 block, Args... args) {
    launch_async(stream, kernel, grid, block, args...);
    synchronize(stream);
}

template <typename... Params, typename... Args>
inline void launch_sync(void (*kernel)(Params...), dim3 grid, dim3 block, Args... args) {
    launch_sync(nullptr, kernel, grid, block, args...);
}

} // namespace opworks

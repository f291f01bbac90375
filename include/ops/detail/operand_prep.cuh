#pragma once

// Operand preparation for the tcgen05 GEMM's fp32 API paths.
//
//   split_rows   : fp32 [rows][cols] -> tf32 hi/lo pair [rows][ld]
//   split_cols_t : fp32 [rows][cols] -> transposed tf32 hi/lo [cols][ld]
//   rows_to_bf16 : fp32 [rows][cols] -> bf16 [rows][ld]
//
// hi = x rounded to tf32 (10 explicit mantissa bits, round-to-nearest-even),
// lo = x - hi (exact in fp32). hi*hi + hi*lo + lo*hi reproduces an fp32
// product to ~2^-21 relative error, which is what ops::mat_mul and the fp32
// ops::linear promise. Columns in [cols, ld) are written as zeros.

#include <cuda_bf16.h>

#include "../../core/cuda_utils.cuh"

namespace opworks::detail {

__device__ __forceinline__ float tf32_round(float x) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7f800000u) == 0x7f800000u)
        return x; // inf / nan pass through
    u += 0xfffu + ((u >> 13) & 1u);
    return __uint_as_float(u & 0xffffe000u);
}

// One block per row (grid-stride over rows): 16-byte stores of the hi / lo
// rows (ld is a multiple of 4), 16-byte loads when the source row allows.
static __global__ void split_rows_kernel(const float *__restrict__ src, int rows, int cols, int64_t ld_src,
                                         float *__restrict__ hi, float *__restrict__ lo, int64_t ld) {
    const bool vec_src = (ld_src % 4 == 0) && (reinterpret_cast<uintptr_t>(src) % 16 == 0);
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const float *s = src + r * ld_src;
        float4 *h4 = reinterpret_cast<float4 *>(hi + r * ld);
        float4 *l4 = reinterpret_cast<float4 *>(lo + r * ld);
        for (int64_t c = 4 * static_cast<int64_t>(threadIdx.x); c < ld; c += 4 * static_cast<int64_t>(blockDim.x)) {
            float4 x;
            if (vec_src && c + 3 < cols) {
                x = *reinterpret_cast<const float4 *>(s + c);
            } else {
                x.x = c < cols ? s[c] : 0.f;
                x.y = c + 1 < cols ? s[c + 1] : 0.f;
                x.z = c + 2 < cols ? s[c + 2] : 0.f;
                x.w = c + 3 < cols ? s[c + 3] : 0.f;
            }
            const float4 h = make_float4(tf32_round(x.x), tf32_round(x.y), tf32_round(x.z), tf32_round(x.w));
            h4[c / 4] = h;
            l4[c / 4] = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
        }
    }
}

// Launch of split_rows_kernel: ld must be a multiple of 4 (16-byte rows).
inline void split_rows_launch(cudaStream_t stream, const float *src, int rows, int cols, int64_t ld_src, float *hi,
                              float *lo, int64_t ld) {
    require(ld % 4 == 0, "split_rows: the padded row stride must be a multiple of 4");
    const int grid = rows < 65535 ? rows : 65535;
    if (grid > 0)
        launch_async(stream, split_rows_kernel, grid, kThreads, src, rows, cols, ld_src, hi, lo, ld);
}

// 32x32 tiles through shared memory so both the read of src rows and the
// write of dst rows are coalesced.
static __global__ void split_cols_t_kernel(const float *__restrict__ src, int rows, int cols,
                                           float *__restrict__ hi, float *__restrict__ lo, int64_t ld) {
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32;
    const int r0 = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int r = r0 + j, c = c0 + threadIdx.x;
        tile[j][threadIdx.x] = (r < rows && c < cols) ? src[static_cast<int64_t>(r) * cols + c] : 0.f;
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int c = c0 + j;          // output row
        const int r = r0 + threadIdx.x; // output column
        if (c < cols && r < ld) {
            const float x = tile[threadIdx.x][j];
            const float h = tf32_round(x);
            hi[static_cast<int64_t>(c) * ld + r] = h;
            lo[static_cast<int64_t>(c) * ld + r] = x - h;
        }
    }
}

static __global__ void rows_to_bf16_kernel(const float *__restrict__ src, int rows, int cols, int64_t ld_src,
                                           __nv_bfloat16 *__restrict__ dst, int64_t ld) {
    const int64_t total = static_cast<int64_t>(rows) * ld;
    OPWORKS_GRID_LOOP(i, total) {
        const int64_t r = i / ld;
        const int64_t c = i % ld;
        dst[i] = __float2bfloat16_rn(c < cols ? src[r * ld_src + c] : 0.f);
    }
}

static __global__ void fill_kernel(float *__restrict__ out, int64_t n, float value) {
    OPWORKS_GRID_LOOP(i, n) { out[i] = value; }
}

template <typename Epi> __global__ void fill_epilogue_kernel(float *__restrict__ out, int64_t n, Epi epi) {
    OPWORKS_GRID_LOOP(i, n) { out[i] = epi(0.f); }
}

inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

inline int grid_for(int64_t n) {
    const int64_t b = (n + kThreads - 1) / kThreads;
    const int cap = device_facts().max_grid_blocks;
    return static_cast<int>(b < cap ? (b > 0 ? b : 1) : cap);
}

// Stream-ordered scratch that is released after the work queued on `stream`.
// Operand scratch from the stream-ordered allocator. The first use on a
// device raises its default memory pool's release threshold to
// kScratchKeepBytes, so scratch freed here stays mapped across stream
// synchronisations (with the default threshold of 0 every synchronisation
// returns it and the next call maps it again, which costs more than the GEMM
// at C1 sizes). The setting is process-local and only affects the default pool.
constexpr uint64_t kScratchKeepBytes = 1ull << 30;
inline void keep_pool_scratch() {
    static thread_local int done_mask = 0; // bit per device id < 32
    int dev = 0;
    OPWORKS_CUDA_CHECK(cudaGetDevice(&dev));
    if (dev < 32 && (done_mask >> dev & 1))
        return;
    cudaMemPool_t pool;
    uint64_t cur = 0, keep = kScratchKeepBytes;
    cudaError_t rc = cudaDeviceGetDefaultMemPool(&pool, dev);
    if (rc == cudaSuccess)
        rc = cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &cur);
    if (rc == cudaSuccess && cur < keep)
        rc = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    if (rc != cudaSuccess)
        cudaGetLastError(); // pools unsupported: keep the default behaviour
    if (dev < 32)
        done_mask |= 1 << dev;
}

class StreamScratch {
  public:
    StreamScratch(size_t bytes, cudaStream_t stream) : stream_(stream) {
        if (bytes) {
            keep_pool_scratch();
            OPWORKS_CUDA_CHECK(cudaMallocAsync(&ptr_, bytes, stream));
        }
    }
    ~StreamScratch() {
        if (ptr_)
            cudaFreeAsync(ptr_, stream_);
    }
    StreamScratch(const StreamScratch &) = delete;
    StreamScratch &operator=(const StreamScratch &) = delete;
    template <typename T> T *as(size_t byte_offset = 0) const {
        return reinterpret_cast<T *>(static_cast<char *>(ptr_) + byte_offset);
    }

  private:
    void *ptr_ = nullptr;
    cudaStream_t stream_;
};

} // namespace opworks::detail

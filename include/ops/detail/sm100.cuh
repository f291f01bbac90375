#pragma once

// Blackwell (sm_100a) building blocks written directly in PTX:
//   - mbarrier init / arrive / expect_tx / bounded parity wait
//   - TMA tiled 2D loads (cp.async.bulk.tensor) and 1D bulk copies
//   - tcgen05: TMEM alloc/dealloc, MMA (kind::f16 and kind::tf32), commit,
//     32x32b loads, thread-sync fences
//   - shared-memory matrix descriptors (K-major, 128-byte swizzle) and
//     instruction descriptors
//   - host-side tensor-map encoding through the driver entry point
//
// No cluster multicast is used anywhere: every CTA issues its own loads,
// so the same kernels are safe in multi-GPU runs.
//
// Every wait is bounded (kWaitTimeoutNs of %globaltimer); a wait that runs out
// returns false, the caller records an error code in global memory and the
// kernel winds down instead of hanging.

#include <cstdint>
#include <cstring>
#include <mutex>
#include <vector>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include "../../core/cuda_utils.cuh"

namespace opworks::sm100 {

// ---------------------------------------------------------------- device ---

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(done)
                 : "r"(smem_u32(bar)), "r"(parity)
                 : "memory");
    return done != 0;
}

// Wait for completion of the phase with the given parity; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity))
        return true;
    const uint64_t start = global_timer_ns();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity))
                return true;
        if (global_timer_ns() - start > kWaitTimeoutNs)
            return false;
    }
}

// mbar_wait by every lane of a warp, with a warp-uniform result: code that
// follows a failed wait (and skips tcgen05 warp-collective instructions)
// stays convergent even if the lanes' deadlines fell on both sides.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *tm) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

// Bulk prefetch of [src, src + bytes) into L2 (no shared-memory destination,
// no completion to wait for). src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)), "r"(bytes)
                 : "memory");
}

// 2D tiled TMA load of box (c0 = innermost coordinate, c1 = row) into smem,
// completing `bytes` on `bar`. c0 * elem_size must be a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *tm, uint64_t *bar, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
                 "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
                 : "memory");
}

// 1D bulk copy global -> shared (both 16-byte aligned, size multiple of 16).
__device__ __forceinline__ void bulk_load(void *smem_dst, const void *gsrc, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(smem_dst)),
                 "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// ---- tcgen05 ----

__device__ __forceinline__ void tmem_alloc(uint32_t *slot_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
                 "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
                 : "memory");
}

// Same with tf32 inputs (32-bit words in smem).
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
                 "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
                 : "memory");
}

// Arrive on `bar` once every previously issued tcgen05.mma of this thread
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns; lane i of the warp receives TMEM
// lane (taddr.lane + i).
__device__ __forceinline__ void tmem_ld_32x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                 "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15])
                 : "r"(taddr)
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Registers loaded by tcgen05.ld are valid only after tcgen05.wait::ld. When
// several loads are issued before one wait, this empty statement (placed
// after the wait) redefines the registers so the compiler cannot move their
// uses above the wait.
__device__ __forceinline__ void tmem_reg_fence(uint32_t (&r)[16]) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}

// Shared-memory matrix descriptor for a K-major tile whose rows are 128 bytes
// (one 128B swizzle atom per row, 8-row groups 1024 bytes apart), as written
// by a TMA load with CU_TENSOR_MAP_SWIZZLE_128B. Fields: start address >> 4
// [0,14), leading byte offset >> 4 [16,30) (unused for swizzled K-major, 1),
// stride byte offset >> 4 [32,46) (1024 B), descriptor version 1 [46,48),
// base offset 0 [49,52), layout 2 = SWIZZLE_128B [61,64).
__device__ __forceinline__ uint64_t sdesc_k128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// Instruction descriptor: D fp32, A/B format (kind::f16: 0 = fp16, 1 = bf16;
// kind::tf32: 2), both K-major, N >> 3 at [17,23), M >> 4 at [24,29).
// Shared-memory descriptor of an MN-major tf32 operand: MN-major 32-bit
// operands take the 128-byte swizzle with 32-byte atomicity (layout type 1,
// SWIZZLE_128B_BASE32B; atoms of 4 K-rows x 128 bytes along MN, as a TMA load
// with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B writes them): `lbo` = bytes between
// atoms adjacent along MN, `sbo` = bytes between 4-row groups along K.
__device__ __forceinline__ uint64_t sdesc_mn128_32b(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(1u) << 61;
    return d;
}

__host__ __device__ constexpr uint32_t idesc_make(uint32_t ab_format, int m, int n) {
    return (1u << 4) | (ab_format << 7) | (ab_format << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}
constexpr uint32_t kFmtF16 = 0;
constexpr uint32_t kFmtBF16 = 1;
constexpr uint32_t kFmtTF32 = 2;

// ------------------------------------------------------------------ host ---

inline PFN_cuTensorMapEncodeTiled_v12000 load_tensor_map_encoder() {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    OPWORKS_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    detail::require(q == cudaDriverEntryPointSuccess && p != nullptr, "cuTensorMapEncodeTiled is unavailable");
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
}

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static const PFN_cuTensorMapEncodeTiled_v12000 fn = load_tensor_map_encoder(); // thread-safe static init
    return fn;
}

// 2D row-major tensor [rows][cols] with row stride `ld` elements, loaded as
// boxes of box_cols x box_rows with 128B swizzle (box_cols * elem == 128).
// 2-D tiled map of 16-bit (word16) or 32-bit elements. Tiled copies move
// bytes without conversion, so 16-bit words of either format (bf16 or fp16)
// use the one 16-bit map type.
// swz: CU_TENSOR_MAP_SWIZZLE_128B for K-major operands; MN-major 32-bit
// operands take CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B (sdesc_mn128_32b)
inline CUtensorMap make_tmap_2d(const void *base, bool word16, uint64_t cols, uint64_t rows, uint64_t ld,
                                uint32_t box_cols, uint32_t box_rows,
                                CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
    const size_t elem = word16 ? 2 : 4;
    detail::require(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
    detail::require((ld * elem) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
    detail::require(box_cols * elem == 128, "TMA box must be one 128-byte swizzle atom wide");
    CUtensorMap tm;
    std::memset(&tm, 0, sizeof(tm));
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {ld * elem};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = tensor_map_encoder()(
        &tm, word16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base),
        dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    detail::require(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed");
    return tm;
}

// Per-device error word written by kernels whose bounded waits ran out.
inline int *device_error_word() {
    static std::vector<int *> words; // one word per device index
    static std::mutex mu;
    int dev = 0, count = 0;
    OPWORKS_CUDA_CHECK(cudaGetDevice(&dev));
    OPWORKS_CUDA_CHECK(cudaGetDeviceCount(&count));
    std::lock_guard<std::mutex> lock(mu);
    if (words.size() < static_cast<size_t>(count))
        words.resize(static_cast<size_t>(count), nullptr);
    detail::require(dev >= 0 && dev < count, "device index outside the visible devices");
    int *&w = words[static_cast<size_t>(dev)];
    if (w == nullptr) {
        OPWORKS_CUDA_CHECK(cudaMalloc(reinterpret_cast<void **>(&w), sizeof(int)));
        OPWORKS_CUDA_CHECK(cudaMemset(w, 0, sizeof(int)));
    }
    return w;
}

} // namespace opworks::sm100

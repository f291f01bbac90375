#pragma once

// ops::mat_mul — C(M x K) = epilogue(A(M x N) @ B(N x K)), N is the
// contraction dimension; the epilogue is a unary per-element functor.
// Contract of OpWorks include/ops/matmul.cuh:71-91: asynchronous, zero output
// rows/columns is a no-op, N == 0 writes epilogue(0), C must not overlap A/B.
//
// B200 path: split-precision TF32 on the tcgen05 tensor cores (three
// kind::tf32 MMAs per K step on hi/lo operand halves), so the fp32 API keeps
// fp32-class accuracy (~1e-6 relative) instead of plain TF32's ~1e-3. When
// the rows of A and B are 16-byte aligned (N and K multiples of 4) the GEMM
// (sm100::gemm_tf32x3s) loads both matrices as they are — B's rows as an
// MN-major operand — and four converter warps split each staged tile into
// hi/lo in shared memory: asynchronous, allocation-free, one launch.
// Otherwise a pre-pass writes aligned hi/lo halves of A and of B^T into
// stream-ordered scratch for the K-major kernel. Either way the GEMM streams
// through TMA into a 128 x BN TMEM accumulator and applies the epilogue
// functor on the way out. Grids of few 128 x 128 tiles (e.g. 1024 x
// 1024 outputs) split K across a thread-block cluster and reduce the partial
// tiles on chip before the epilogue (sm100::gemm_tf32x3).

#include "../core/cuda_utils.cuh"
#include "detail/operand_prep.cuh"
#include "gemm_sm100.cuh"

namespace opworks::ops {

struct PassThrough {
    __device__ float operator()(float x) const { return x; }
};

template <typename Epilogue = PassThrough>
inline void mat_mul(const float *A, const float *B, float *C, int M, int N, int K, Epilogue epilogue = {},
                    cudaStream_t stream = nullptr) {
    detail::validate_matrix(M, N);
    detail::validate_matrix(N, K);
    detail::validate_matrix(M, K);
    if (M == 0 || K == 0)
        return;
    detail::require(C && (N == 0 || (A && B)), "matmul requires non-null pointers for nonempty tensors");
    const int64_t out_elems = static_cast<int64_t>(M) * K;
    if (N == 0) {
        launch_async(stream, detail::fill_epilogue_kernel<Epilogue>, detail::grid_for(out_elems), kThreads, C,
                     out_elems, epilogue);
        return;
    }
    if (N % 4 == 0 && K % 4 == 0 && reinterpret_cast<uintptr_t>(A) % 16 == 0 &&
        reinterpret_cast<uintptr_t>(B) % 16 == 0) {
        // rows of A and B are 16-byte aligned: the GEMM reads both as they
        // are and splits them into tf32 hi / lo in shared memory (no
        // pre-pass, no scratch, nothing allocated)
        sm100::gemm_tf32x3s<Epilogue>(A, N, B, K, M, N, K, C, K, stream, epilogue);
        return;
    }
    // unaligned rows: a pre-pass writes 16-byte-aligned hi / lo copies
    const int64_t ld = detail::round_up(N, 4); // 16-byte row stride for TMA
    const size_t a_bytes = sizeof(float) * static_cast<size_t>(M) * ld;
    const size_t b_bytes = sizeof(float) * static_cast<size_t>(K) * ld;
    detail::StreamScratch scratch(2 * a_bytes + 2 * b_bytes, stream);
    float *a_hi = scratch.as<float>(0);
    float *a_lo = scratch.as<float>(a_bytes);
    float *bt_hi = scratch.as<float>(2 * a_bytes);
    float *bt_lo = scratch.as<float>(2 * a_bytes + b_bytes);

    detail::split_rows_launch(stream, A, M, N, static_cast<int64_t>(N), a_hi, a_lo, ld);
    const dim3 tgrid(detail::blocks_for(K, 32), detail::blocks_for(static_cast<int>(ld), 32));
    launch_async(stream, detail::split_cols_t_kernel, tgrid, dim3(32, 8), B, N, K, bt_hi, bt_lo, ld);

    sm100::GemmOperand feat{bt_hi, bt_lo, K, ld};
    sm100::GemmOperand tok{a_hi, a_lo, M, ld};
    sm100::gemm_tf32x3<Epilogue>(feat, tok, N, C, K, stream, epilogue);
}

} // namespace opworks::ops

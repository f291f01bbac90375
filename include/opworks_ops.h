/* C ABI over the OpWorks-B200 operator layer (libopworks_ops.so).
 *
 * OpWorks exposes its operators to foreign callers through one-function
 * `extern "C" void solve(...)` adapters (tests/integration/*.cu: vector_add,
 * relu, reduction, softmax, layer_normalization, matrix_multiplication) that
 * run one op on device pointers and synchronise. This library exports the
 * same capability for every operator on the Llama hot path, one named symbol
 * per op, so a ctypes / cgo / JNI caller can bind them all from one .so.
 *
 * Conventions: every pointer is a DEVICE pointer unless stated otherwise;
 * `stream` is a cudaStream_t (NULL = legacy default stream); calls are
 * asynchronous unless they say otherwise. Functions return 0 on success and
 * -1 when the C++ API rejected the arguments (std::invalid_argument); the
 * message is then available from opw_ops_last_error() (thread-local). CUDA
 * runtime failures abort the process, as in OpWorks (OPWORKS_CUDA_CHECK).
 */
#ifndef OPWORKS_OPS_H
#define OPWORKS_OPS_H

#include <stddef.h>
#include <stdint.h>

/* Only the C ABI is exported; the libraries are built with hidden default
 * visibility so two of them (or the reference's library) can share a process. */
#ifndef OPW_API
#define OPW_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Thread-local message of the last failed call. */
OPW_API const char *opw_ops_last_error(void);
/* Waits for `stream`; returns 0, or -1 if the device error word is set (a
 * bounded device-side wait ran out), clearing it. */
OPW_API int opw_ops_sync(void *stream);

/* ops::map with fixed functors (include/ops/elementwise.cuh:63-77;
 * tests/integration/vector_add.cu, relu.cu). */
OPW_API int opw_map_add(const float *a, const float *b, float *out, int n, void *stream);
OPW_API int opw_map_relu(const float *in, float *out, int n, void *stream);
OPW_API int opw_map_scale(const float *in, float *out, int n, float factor, void *stream);

/* ops::reduce<Sum|Max> (include/ops/reduction.cuh:34-67;
 * tests/integration/reduction.cu). kind: 0 = sum, 1 = max, 2 = product.
 * workspace may be NULL with workspace_size 0 to use stream-ordered scratch. */
OPW_API int opw_reduction_workspace_size(int n);
OPW_API int opw_reduce(int kind, const float *in, float *out, int n, float *workspace, int workspace_size, void *stream);

/* Allocation-free reduction: no reference counterpart (an extension of this
 * library). Same kinds and result as opw_reduce, with the workspace taken
 * from a static device buffer of 1025 floats (4100 bytes, the largest
 * workspace any n needs) instead of a caller buffer or a stream-ordered
 * allocation; a request that would need more is rejected with an error.
 * Each call clears the buffer's arrival counter before its kernel.
 * - The buffer is shared by every call on a device: calls that may overlap
 *   (different streams, host threads or graph branches without an ordering
 *   between them) race on it and must be serialised by the caller.
 * - The first call on each device looks the buffer's address up and must not
 *   run inside a stream capture; later calls may be captured. */
OPW_API int opw_reduce_static(int kind, const float *in, float *out, int n, void *stream);

/* ops::softmax / ops::layer_norm (softmax.cuh:36-43, layer_norm.cuh:38-47). */
OPW_API int opw_softmax(const float *in, float *out, int rows, int cols, void *stream);
OPW_API int opw_layer_norm(const float *in, float *out, const float *gamma, const float *beta, int rows, int cols, float eps,
                   void *stream);

/* ops::mat_mul (matmul.cuh:78-91): C(MxK) = epi(A(MxN) @ B(NxK)).
 * epilogue: 0 = pass-through, 1 = relu, 2 = scale by `param`. */
OPW_API int opw_mat_mul(const float *A, const float *B, float *C, int M, int N, int K, int epilogue, float param,
                void *stream);

/* MatmulBuilder + ops::matmul_launcher (builders/matmul.cuh:9-57): bias may
 * be NULL; activation 0 none, 1 relu, 2 gelu. */
OPW_API int opw_matmul_builder(const float *A, const float *B, float *C, int M, int N, int K, int transpose_a,
                       int transpose_b, const float *bias, int activation, void *stream);

/* RowwiseBuilder + ops::rowwise_launcher (builders/rowwise.cuh:11-63):
 * op 0 softmax, 1 layer_norm (param, beta), 2 rms_norm (param). */
OPW_API int opw_rowwise_builder(int op, const float *in, float *out, const float *param, const float *beta, int rows,
                        int cols, float eps, void *stream);

/* Model operators (include/ops/*.cuh of OpWorks, same argument order). */
OPW_API int opw_rms_norm(const float *x, const float *weight, float *out, int rows, int cols, float eps, void *stream);
OPW_API int opw_linear_f32(const float *X, const float *W, float *Y, int rows, int in_features, int out_features,
                   void *stream);
OPW_API int opw_linear_bf16(const float *X, const uint16_t *W_bf16, float *Y, int rows, int in_features, int out_features,
                    void *stream);
OPW_API int opw_linear_mma_bf16(const float *X, const uint16_t *W_bf16, float *Y, int rows, int in_features,
                        int out_features, void *stream);
OPW_API int opw_embedding_f32(const float *table, const int32_t *ids, float *out, int n, int hidden, void *stream);
OPW_API int opw_embedding_bf16(const uint16_t *table, const int32_t *ids, float *out, int n, int hidden, void *stream);
OPW_API int opw_rope(float *x, const float *inv_freq, int rows, int heads, int head_dim, int pos_start, void *stream);
OPW_API int opw_split_heads(const float *in, float *out, int rows, int heads, int head_dim, int out_row_stride,
                    int out_row_offset, void *stream);
OPW_API int opw_merge_heads(const float *in, float *out, int rows, int heads, int head_dim, int in_row_stride,
                    int in_row_offset, void *stream);
OPW_API int opw_causal_scale(float *scores, int rows, int cols, float scale, void *stream);
OPW_API int opw_swiglu(const float *gate, const float *up, float *out, int64_t n, void *stream);
OPW_API int opw_add(const float *a, const float *b, float *out, int64_t n, void *stream);
OPW_API int opw_argmax(const float *x, int n, int32_t *out, void *stream);
OPW_API int opw_attention_decode(const float *q, const float *kcache, const float *vcache, float *out, int num_q_heads,
                         int kv_rep, int head_dim, int len, int max_seq, void *stream);
OPW_API int opw_attention_prefill_chunked(const float *q_heads, const float *kcache, const float *vcache, float *out, int T,
                                  int S, int q_offset, int num_q_heads, int kv_rep, int head_dim, int cap,
                                  void *stream);

/* Fused greedy / top-p sampler of the Llama runtime (ops/llama_kernels.cuh),
 * the device form of OpWorks' host sampler examples/llama/generate.py:83-109:
 * one token per row of logits [rows, vocab]; temperature[r] <= 0 selects the
 * first argmax, otherwise top-p with uniform[r] (device arrays). */
OPW_API int opw_sample(const float *logits, int rows, int vocab, const float *temperature, const float *top_p,
               const double *uniform, int32_t *out, void *stream);

/* Batched decode attention over a paged fp32 KV cache (the Llama runtime's
 * kernel): q [B][qh*64], pools [blocks][kvh][16][64], block_table
 * [B][table_stride], lens[B] (device int32); out [B][qh*64] fp32. Scratch for
 * the split-KV partials comes from stream-ordered allocation. */
OPW_API int opw_paged_attention_decode(const float *q, const float *kpool, const float *vpool,
                                       const int32_t *block_table, int table_stride, const int32_t *lens, int B,
                                       int max_len, int num_q_heads, int num_kv_heads, float *out, void *stream);
/* Causal GQA prefill attention of query rows [0, T) of sequence b (absolute
 * positions q_offset + t) over a paged fp32 KV pool [num_blocks][kvh][16][64]
 * with block_table[b * table_stride + page]; q and out are [T][num_q_heads *
 * 64] fp32; head_dim 64, scale 1/8. tensor_cores = 1: TF32 tcgen05 flash
 * attention (include/ops/attention_prefill_tc.cuh); 0: the fp32 SIMT kernel.
 * Extension of this library (no reference counterpart; the reference's
 * prefill attention is ops::attention_prefill_chunked over contiguous K/V). */
OPW_API int opw_paged_attention_prefill(const float *q, const float *kpool, const float *vpool, const int32_t *block_table,
                                        int table_stride, int num_blocks, int b, int T, int q_offset, int num_q_heads,
                                        int num_kv_heads, float *out, int tensor_cores, void *stream);
/* out[split][M][N] (fp32 partials) = W[N][K] (bf16) . (Xhi + Xlo)[M][K]^T with
 * the runtime's two-term bf16 activation GEMM; splits = 0 picks the runtime's
 * split-K plan. Returns the split count used, or -1. */
OPW_API int opw_gemm_bf16x2(const uint16_t *W, const uint16_t *x_hi, const uint16_t *x_lo, float *out, int N, int K,
                            int M, int splits, void *stream);
/* out[M][N] (fp32) = W[N][K] (bf16) . (Xhi + Xlo)[M][K]^T by the two-SM
 * (tcgen05 cta_group::2) GEMM of the runtime's prefill projections: pairs of
 * CTAs compute 256 x 256 tiles (include/ops/gemm_sm100_pair.cuh). K must be a
 * multiple of 8. Extension of this library (no reference counterpart). */
OPW_API int opw_gemm_bf16x2_pair(const uint16_t *W, const uint16_t *x_hi, const uint16_t *x_lo, float *out, int N,
                                 int K, int M, void *stream);
/* The same two GEMMs with every 16-bit word read as fp16 instead of bf16 (the
 * format the runtime's fast path uses for float32 packs: 11 significant bits
 * at 2 bytes). The pair entry points accept x_lo == NULL: one activation term,
 * one MMA per K step. Extensions of this library (no reference counterpart). */
OPW_API int opw_gemm_f16x2(const uint16_t *W, const uint16_t *x_hi, const uint16_t *x_lo, float *out, int N, int K,
                           int M, int splits, void *stream);
OPW_API int opw_gemm_f16x2_pair(const uint16_t *W, const uint16_t *x_hi, const uint16_t *x_lo, float *out, int N,
                                int K, int M, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* OPWORKS_OPS_H */

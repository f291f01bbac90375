// libopworks_ops.so: C ABI over the header-only operator layer, declared in
// include/opworks_ops.h. Each entry point forwards to the C++ API and turns
// std::exception into -1 plus a thread-local message.

#include <opworks>

#include <cstring>
#include <mutex>
#include <string>

#include "opworks_ops.h"
#include "ops/add.cuh"
#include "ops/argmax.cuh"
#include "ops/attention_decode.cuh"
#include "ops/attention_prefill.cuh"
#include "ops/attention_prefill_tc.cuh"
#include "ops/gemm_sm100_pair.cuh"
#include "ops/causal_scale.cuh"
#include "ops/embedding.cuh"
#include "ops/linear.cuh"
#include "ops/linear_mma.cuh"
#include "ops/llama_kernels.cuh"
#include "ops/rms_norm.cuh"
#include "ops/rope.cuh"
#include "ops/split_heads.cuh"
#include "ops/swiglu.cuh"

namespace {

thread_local std::string g_error;

template <typename F> int guarded(F &&f) {
    try {
        f();
        return 0;
    } catch (const std::exception &e) {
        g_error = e.what();
    } catch (...) {
        g_error = "unknown C++ exception";
    }
    return -1;
}

cudaStream_t as_stream(void *s) { return static_cast<cudaStream_t>(s); }

struct AddF {
    __device__ float operator()(float a, float b) const { return a + b; }
};
struct ReluF {
    __device__ float operator()(float x) const { return fmaxf(x, 0.f); }
};
struct ScaleF {
    float factor;
    __device__ float operator()(float x) const { return factor * x; }
};
struct SumF {
    static __device__ float identity() { return 0.f; }
    static __device__ float combine(float a, float b) { return a + b; }
};
struct MaxF {
    static __device__ float identity() { return -INFINITY; }
    static __device__ float combine(float a, float b) { return fmaxf(a, b); }
};
struct ProdF {
    static __device__ float identity() { return 1.f; }
    static __device__ float combine(float a, float b) { return a * b; }
};

template <typename Op>
void reduce_with(const float *in, float *out, int n, float *ws, int ws_size, cudaStream_t s) {
    if (ws == nullptr && ws_size == 0)
        opworks::ops::reduce<Op>(in, out, n, s);
    else
        opworks::ops::reduce<Op>(in, out, n, opworks::DeviceSpan<float>(ws, ws_size), s);
}

const __nv_bfloat16 *as_bf16(const uint16_t *p) { return reinterpret_cast<const __nv_bfloat16 *>(p); }

// Scratch of opw_reduce_static: the largest reduction workspace there is
// (kReduceMaxBlocks partial slots + the arrival counter = 1025 floats,
// 4100 bytes), one copy per device context.
constexpr int kStaticReduceFloats = opworks::detail::kReduceMaxBlocks + 1;
static __device__ __align__(256) float g_reduce_scratch[kStaticReduceFloats];

// Device address of g_reduce_scratch on the current device, looked up once per
// device (cudaGetSymbolAddress may load the module, which a stream capture
// does not allow: the first call on a device must not be captured).
float *static_reduce_scratch() {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static float *addr[kMaxDevices] = {};
    int dev = 0;
    OPWORKS_CUDA_CHECK(cudaGetDevice(&dev));
    opworks::detail::require(dev >= 0 && dev < kMaxDevices, "opw_reduce_static: device index out of range");
    const std::lock_guard<std::mutex> lock(mu);
    if (addr[dev] == nullptr)
        OPWORKS_CUDA_CHECK(cudaGetSymbolAddress(reinterpret_cast<void **>(&addr[dev]), g_reduce_scratch));
    return addr[dev];
}

template <typename Op> void reduce_static_with(const float *in, float *out, int n, cudaStream_t s) {
    const int needed = opworks::ops::reduction_workspace_size(n);
    opworks::detail::require(needed <= kStaticReduceFloats,
                             "opw_reduce_static: the reduction needs more scratch than the static buffer holds");
    float *ws = needed > 0 ? static_reduce_scratch() : nullptr;
    // the workspace overload clears the arrival counter (a memset node) before
    // the kernel, so every call starts from a clean state
    opworks::ops::reduce<Op>(in, out, n, opworks::DeviceSpan<float>(ws, needed), s);
}

} // namespace

extern "C" {

const char *opw_ops_last_error(void) { return g_error.c_str(); }

int opw_ops_sync(void *stream) {
    OPWORKS_CUDA_CHECK(cudaStreamSynchronize(as_stream(stream)));
    int *word = opworks::sm100::device_error_word();
    int value = 0;
    OPWORKS_CUDA_CHECK(cudaMemcpy(&value, word, sizeof(int), cudaMemcpyDeviceToHost));
    if (value != 0) {
        OPWORKS_CUDA_CHECK(cudaMemset(word, 0, sizeof(int)));
        g_error = "a device-side wait timed out (error code " + std::to_string(value) + ")";
        return -1;
    }
    return 0;
}

int opw_map_add(const float *a, const float *b, float *out, int n, void *stream) {
    return guarded([&] { opworks::ops::map(a, b, out, n, AddF{}, as_stream(stream)); });
}
int opw_map_relu(const float *in, float *out, int n, void *stream) {
    return guarded([&] { opworks::ops::map(in, out, n, ReluF{}, as_stream(stream)); });
}
int opw_map_scale(const float *in, float *out, int n, float factor, void *stream) {
    return guarded([&] { opworks::ops::map(in, out, n, ScaleF{factor}, as_stream(stream)); });
}

int opw_reduction_workspace_size(int n) {
    int r = -1;
    guarded([&] { r = opworks::ops::reduction_workspace_size(n); });
    return r;
}

int opw_reduce(int kind, const float *in, float *out, int n, float *workspace, int workspace_size, void *stream) {
    return guarded([&] {
        switch (kind) {
        case 0: reduce_with<SumF>(in, out, n, workspace, workspace_size, as_stream(stream)); break;
        case 1: reduce_with<MaxF>(in, out, n, workspace, workspace_size, as_stream(stream)); break;
        case 2: reduce_with<ProdF>(in, out, n, workspace, workspace_size, as_stream(stream)); break;
        default: throw std::invalid_argument("unknown reduction kind");
        }
    });
}

int opw_reduce_static(int kind, const float *in, float *out, int n, void *stream) {
    return guarded([&] {
        switch (kind) {
        case 0: reduce_static_with<SumF>(in, out, n, as_stream(stream)); break;
        case 1: reduce_static_with<MaxF>(in, out, n, as_stream(stream)); break;
        case 2: reduce_static_with<ProdF>(in, out, n, as_stream(stream)); break;
        default: throw std::invalid_argument("unknown reduction kind");
        }
    });
}

int opw_softmax(const float *in, float *out, int rows, int cols, void *stream) {
    return guarded([&] { opworks::ops::softmax(in, out, rows, cols, as_stream(stream)); });
}

int opw_layer_norm(const float *in, float *out, const float *gamma, const float *beta, int rows, int cols, float eps,
                   void *stream) {
    return guarded([&] { opworks::ops::layer_norm(in, out, gamma, beta, rows, cols, eps, as_stream(stream)); });
}

int opw_mat_mul(const float *A, const float *B, float *C, int M, int N, int K, int epilogue, float param,
                void *stream) {
    return guarded([&] {
        switch (epilogue) {
        case 0: opworks::ops::mat_mul(A, B, C, M, N, K, opworks::ops::PassThrough{}, as_stream(stream)); break;
        case 1: opworks::ops::mat_mul(A, B, C, M, N, K, ReluF{}, as_stream(stream)); break;
        case 2: opworks::ops::mat_mul(A, B, C, M, N, K, ScaleF{param}, as_stream(stream)); break;
        default: throw std::invalid_argument("unknown epilogue");
        }
    });
}

int opw_matmul_builder(const float *A, const float *B, float *C, int M, int N, int K, int transpose_a,
                       int transpose_b, const float *bias, int activation, void *stream) {
    return guarded([&] {
        using namespace opworks;
        MatmulBuilder g(DeviceSpan<const float>(A, M * N), DeviceSpan<const float>(B, N * K),
                        DeviceSpan<float>(C, M * K), M, N, K, as_stream(stream));
        g.transpose_a(transpose_a != 0).transpose_b(transpose_b != 0);
        if (bias)
            g.bias(DeviceSpan<const float>(bias, K));
        g.activation(static_cast<MatmulActivation>(activation));
        g.apply(ops::matmul_launcher{});
    });
}

int opw_rowwise_builder(int op, const float *in, float *out, const float *param, const float *beta, int rows,
                        int cols, float eps, void *stream) {
    return guarded([&] {
        using namespace opworks;
        const DeviceSpan<const float> i(in, rows * cols);
        const DeviceSpan<float> o(out, rows * cols);
        if (op == 0)
            RowwiseBuilder::softmax(i, o, rows, cols, as_stream(stream)).apply(ops::rowwise_launcher{});
        else if (op == 1)
            RowwiseBuilder::layer_norm(i, o, DeviceSpan<const float>(param, cols), DeviceSpan<const float>(beta, cols),
                                       rows, cols, eps, as_stream(stream))
                .apply(ops::rowwise_launcher{});
        else if (op == 2)
            RowwiseBuilder::rms_norm(i, o, DeviceSpan<const float>(param, cols), rows, cols, eps, as_stream(stream))
                .apply(ops::rowwise_launcher{});
        else
            throw std::invalid_argument("unknown rowwise op");
    });
}

int opw_rms_norm(const float *x, const float *weight, float *out, int rows, int cols, float eps, void *stream) {
    return guarded([&] { opworks::ops::rms_norm(x, weight, out, rows, cols, eps, as_stream(stream)); });
}

int opw_linear_f32(const float *X, const float *W, float *Y, int rows, int in_features, int out_features,
                   void *stream) {
    return guarded([&] { opworks::ops::linear(X, W, Y, rows, in_features, out_features, as_stream(stream)); });
}

int opw_linear_bf16(const float *X, const uint16_t *W, float *Y, int rows, int in_features, int out_features,
                    void *stream) {
    return guarded(
        [&] { opworks::ops::linear(X, as_bf16(W), Y, rows, in_features, out_features, as_stream(stream)); });
}

int opw_linear_mma_bf16(const float *X, const uint16_t *W, float *Y, int rows, int in_features, int out_features,
                        void *stream) {
    return guarded([&] {
        opworks::ops::linear_mma_bf16(X, as_bf16(W), Y, rows, in_features, out_features, as_stream(stream));
    });
}

int opw_embedding_f32(const float *table, const int32_t *ids, float *out, int n, int hidden, void *stream) {
    return guarded([&] { opworks::ops::embedding(table, ids, out, n, hidden, as_stream(stream)); });
}

int opw_embedding_bf16(const uint16_t *table, const int32_t *ids, float *out, int n, int hidden, void *stream) {
    return guarded([&] { opworks::ops::embedding(as_bf16(table), ids, out, n, hidden, as_stream(stream)); });
}

int opw_rope(float *x, const float *inv_freq, int rows, int heads, int head_dim, int pos_start, void *stream) {
    return guarded([&] { opworks::ops::rope(x, inv_freq, rows, heads, head_dim, pos_start, as_stream(stream)); });
}

int opw_split_heads(const float *in, float *out, int rows, int heads, int head_dim, int out_row_stride,
                    int out_row_offset, void *stream) {
    return guarded([&] {
        opworks::ops::split_heads(in, out, rows, heads, head_dim, out_row_stride, out_row_offset, as_stream(stream));
    });
}

int opw_merge_heads(const float *in, float *out, int rows, int heads, int head_dim, int in_row_stride,
                    int in_row_offset, void *stream) {
    return guarded([&] {
        opworks::ops::merge_heads(in, out, rows, heads, head_dim, in_row_stride, in_row_offset, as_stream(stream));
    });
}

int opw_causal_scale(float *scores, int rows, int cols, float scale, void *stream) {
    return guarded([&] { opworks::ops::causal_scale(scores, rows, cols, scale, as_stream(stream)); });
}

int opw_swiglu(const float *gate, const float *up, float *out, int64_t n, void *stream) {
    return guarded([&] { opworks::ops::swiglu(gate, up, out, n, as_stream(stream)); });
}

int opw_add(const float *a, const float *b, float *out, int64_t n, void *stream) {
    return guarded([&] { opworks::ops::add(a, b, out, n, as_stream(stream)); });
}

int opw_argmax(const float *x, int n, int32_t *out, void *stream) {
    return guarded([&] { opworks::ops::argmax(x, n, out, as_stream(stream)); });
}

int opw_attention_decode(const float *q, const float *kcache, const float *vcache, float *out, int num_q_heads,
                         int kv_rep, int head_dim, int len, int max_seq, void *stream) {
    return guarded([&] {
        opworks::ops::attention_decode(q, kcache, vcache, out, num_q_heads, kv_rep, head_dim, len, max_seq,
                                       as_stream(stream));
    });
}

int opw_attention_prefill_chunked(const float *q_heads, const float *kcache, const float *vcache, float *out, int T,
                                  int S, int q_offset, int num_q_heads, int kv_rep, int head_dim, int cap,
                                  void *stream) {
    return guarded([&] {
        opworks::ops::attention_prefill_chunked(q_heads, kcache, vcache, out, T, S, q_offset, num_q_heads, kv_rep,
                                                head_dim, cap, as_stream(stream));
    });
}

int opw_paged_attention_decode(const float *q, const float *kpool, const float *vpool, const int32_t *block_table,
                               int table_stride, const int32_t *lens, int B, int max_len, int num_q_heads,
                               int num_kv_heads, float *out, void *stream) {
    return guarded([&] {
        using namespace opworks::detail;
        require(B > 0 && max_len > 0 && num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
                "paged attention: bad shape");
        require(q && kpool && vpool && block_table && lens && out, "paged attention: null pointer");
        const int rep = num_q_heads / num_kv_heads;
        const int tps = decode_tokens_per_split(B * num_kv_heads, max_len, device_facts().sm_count);
        const int splits = (max_len + tps - 1) / tps;
        const size_t po = sizeof(float) * static_cast<size_t>(B) * num_q_heads * splits * kAttnD;
        const size_t pml = sizeof(float) * static_cast<size_t>(B) * num_q_heads * splits * 2;
        StreamScratch scratch(po + pml, as_stream(stream));
        const PagedKV kv{kpool, vpool, block_table, table_stride, num_kv_heads};
        const StridedOut<float> o{out, static_cast<int64_t>(num_q_heads) * kAttnD, kAttnD};
        float *part_o = scratch.as<float>(0), *part_ml = scratch.as<float>(po);
        const float scale = 0.125f;
        switch (rep) {
        case 1: attn_decode_launch<PagedKV, 1>(q, num_q_heads * kAttnD, kv, lens, B, num_kv_heads, tps, splits, scale, part_o, part_ml, o, as_stream(stream)); break;
        case 2: attn_decode_launch<PagedKV, 2>(q, num_q_heads * kAttnD, kv, lens, B, num_kv_heads, tps, splits, scale, part_o, part_ml, o, as_stream(stream)); break;
        case 4: attn_decode_launch<PagedKV, 4>(q, num_q_heads * kAttnD, kv, lens, B, num_kv_heads, tps, splits, scale, part_o, part_ml, o, as_stream(stream)); break;
        case 8: attn_decode_launch<PagedKV, 8>(q, num_q_heads * kAttnD, kv, lens, B, num_kv_heads, tps, splits, scale, part_o, part_ml, o, as_stream(stream)); break;
        default: throw std::invalid_argument("paged attention: GQA ratio must be 1, 2, 4 or 8");
        }
    });
}

int opw_paged_attention_prefill(const float *q, const float *kpool, const float *vpool, const int32_t *block_table,
                                int table_stride, int num_blocks, int b, int T, int q_offset, int num_q_heads,
                                int num_kv_heads, float *out, int tensor_cores, void *stream) {
    return guarded([&] {
        using namespace opworks::detail;
        require(T > 0 && q_offset >= 0 && num_kv_heads > 0 && num_q_heads % num_kv_heads == 0 && num_blocks > 0,
                "paged prefill attention: bad shape");
        require(q && kpool && vpool && block_table && out, "paged prefill attention: null pointer");
        const int rep = num_q_heads / num_kv_heads;
        const float scale = 0.125f;
        const int64_t qw = static_cast<int64_t>(num_q_heads) * kAttnD;
        const StridedOut<float> o{out, qw, kAttnD};
        if (tensor_cores) {
            const KvPoolMaps maps = make_kv_pool_maps(kpool, vpool, num_blocks, num_kv_heads);
            switch (rep) {
            case 1: attn_prefill_tc_launch<1>(q, qw, num_q_heads, maps, block_table, table_stride, num_kv_heads, b, T, q_offset, scale, o, as_stream(stream)); break;
            case 2: attn_prefill_tc_launch<2>(q, qw, num_q_heads, maps, block_table, table_stride, num_kv_heads, b, T, q_offset, scale, o, as_stream(stream)); break;
            case 4: attn_prefill_tc_launch<4>(q, qw, num_q_heads, maps, block_table, table_stride, num_kv_heads, b, T, q_offset, scale, o, as_stream(stream)); break;
            case 8: attn_prefill_tc_launch<8>(q, qw, num_q_heads, maps, block_table, table_stride, num_kv_heads, b, T, q_offset, scale, o, as_stream(stream)); break;
            default: throw std::invalid_argument("paged prefill attention: GQA ratio must be 1, 2, 4 or 8");
            }
        } else {
            const PagedKV kv{kpool, vpool, block_table, table_stride, num_kv_heads};
            switch (rep) {
            case 1: attn_prefill_launch<PagedKV, 1>(q, qw, kAttnD, o, kv, b, T, q_offset, num_kv_heads, scale, as_stream(stream)); break;
            case 2: attn_prefill_launch<PagedKV, 2>(q, qw, kAttnD, o, kv, b, T, q_offset, num_kv_heads, scale, as_stream(stream)); break;
            case 4: attn_prefill_launch<PagedKV, 4>(q, qw, kAttnD, o, kv, b, T, q_offset, num_kv_heads, scale, as_stream(stream)); break;
            case 8: attn_prefill_launch<PagedKV, 8>(q, qw, kAttnD, o, kv, b, T, q_offset, num_kv_heads, scale, as_stream(stream)); break;
            default: throw std::invalid_argument("paged prefill attention: GQA ratio must be 1, 2, 4 or 8");
            }
        }
    });
}

namespace {
// Two-term 16-bit GEMM out[M][N] = W[N][K] . (x_hi + x_lo)[M][K]^T with the
// 16-bit words read as fp16 (f16) or bf16.
int gemm_16x2(const uint16_t *W, const uint16_t *x_hi, const uint16_t *x_lo, float *out, int N, int K, int M,
              int splits, bool f16, void *stream) {
    int used = -1;
    const int rc = guarded([&] {
        using namespace opworks;
        detail::require(W && x_hi && x_lo && out && N > 0 && K > 0 && M > 0, "gemm_16x2: bad arguments");
        const int bn = sm100::gemm_pick_bn(sm100::GemmKind::kBF16x2, M);
        if (splits <= 0) {
            const int tiles = ((N + kUmmaM - 1) / kUmmaM) * ((M + bn - 1) / bn);
            splits = sm100::gemm_pick_splits(tiles, (K + 63) / 64,
                                             detail::device_facts().sm_count * sm100::gemm_ctas_per_sm(bn));
        }
        sm100::gemm_tn<sm100::GemmKind::kBF16x2>({W, nullptr, N, K, f16}, {x_hi, x_lo, M, K, f16}, K, out, N, splits,
                                                 static_cast<int64_t>(M) * N, as_stream(stream), sm100::Identity{},
                                                 bn);
        used = splits;
    });
    return rc == 0 ? used : -1;
}

int gemm_16x2_pair(const uint16_t *W, const uint16_t *x_hi, const uint16_t *x_lo, float *out, int N, int K, int M,
                   bool f16, void *stream) {
    return guarded([&] {
        using namespace opworks;
        detail::require(W && x_hi && out && N > 0 && K > 0 && M > 0, "gemm_16x2_pair: bad arguments");
        detail::require(K % 8 == 0, "gemm_16x2_pair: K must be a multiple of 8 (16-byte rows)");
        sm100::gemm_pair_bf16x2({W, nullptr, N, K, f16}, {x_hi, x_lo, M, K, f16}, K, as_stream(stream),
                                sm100::StoreTileEpi<sm100::Identity>{out, N, {}});
    });
}
} // namespace

int opw_gemm_bf16x2(const uint16_t *W, const uint16_t *x_hi, const uint16_t *x_lo, float *out, int N, int K, int M,
                    int splits, void *stream) {
    return gemm_16x2(W, x_hi, x_lo, out, N, K, M, splits, false, stream);
}

int opw_gemm_f16x2(const uint16_t *W, const uint16_t *x_hi, const uint16_t *x_lo, float *out, int N, int K, int M,
                   int splits, void *stream) {
    return gemm_16x2(W, x_hi, x_lo, out, N, K, M, splits, true, stream);
}

int opw_gemm_bf16x2_pair(const uint16_t *W, const uint16_t *x_hi, const uint16_t *x_lo, float *out, int N, int K,
                         int M, void *stream) {
    return gemm_16x2_pair(W, x_hi, x_lo, out, N, K, M, false, stream);
}

int opw_gemm_f16x2_pair(const uint16_t *W, const uint16_t *x_hi, const uint16_t *x_lo, float *out, int N, int K, int M,
                        void *stream) {
    return gemm_16x2_pair(W, x_hi, x_lo, out, N, K, M, true, stream);
}

int opw_sample(const float *logits, int rows, int vocab, const float *temperature, const float *top_p,
               const double *uniform, int32_t *out, void *stream) {
    return guarded([&] {
        opworks::detail::require(rows >= 0 && vocab > 0, "sample requires rows >= 0 and vocab > 0");
        opworks::detail::require(logits && temperature && top_p && uniform && out, "sample requires non-null pointers");
        if (rows == 0)
            return;
        opworks::detail::SampleParams sp{temperature, top_p, uniform, nullptr, nullptr};
        opworks::detail::sample_launch(logits, vocab, rows, vocab, sp, out, as_stream(stream));
    });
}

} // extern "C"

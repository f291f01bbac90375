// ORACLE — test infrastructure only. Compiled against the REFERENCE's own
// headers (include path = the reference tree, see oracle/build_ref.py) so
// the GPU tests can run the reference kernels on the same inputs as ours.
// Every symbol is prefixed ref_ and mirrors one OpWorks operator call.

#include <opworks>

#include "ops/argmax.cuh"
#include "ops/attention_decode.cuh"
#include "ops/attention_prefill.cuh"
#include "ops/embedding.cuh"
#include "ops/linear.cuh"
#include "ops/rms_norm.cuh"
#include "ops/rope.cuh"
#include "ops/swiglu.cuh"

namespace {
struct RefSum {
    static __device__ float identity() { return 0.f; }
    static __device__ float combine(float a, float b) { return a + b; }
};
struct RefRelu {
    __device__ float operator()(float x) const { return fmaxf(x, 0.f); }
};
struct RefAdd {
    __device__ float operator()(float a, float b) const { return a + b; }
};
} // namespace

extern "C" {
void ref_map_add(const float *a, const float *b, float *out, int n) { opworks::ops::map(a, b, out, n, RefAdd{}); }
void ref_reduce_sum(const float *in, float *out, int n) { opworks::ops::reduce<RefSum>(in, out, n); }
// the allocation-free overload (caller's workspace of reduction_workspace_size(n) floats)
int ref_reduction_workspace_size(int n) { return opworks::ops::reduction_workspace_size(n); }
void ref_reduce_sum_ws(const float *in, float *out, int n, float *ws, int ws_floats) {
    opworks::ops::reduce<RefSum>(in, out, n, opworks::DeviceSpan<float>(ws, ws_floats));
}
void ref_softmax(const float *in, float *out, int rows, int cols) { opworks::ops::softmax(in, out, rows, cols); }
void ref_layer_norm(const float *in, float *out, const float *g, const float *b, int rows, int cols, float eps) {
    opworks::ops::layer_norm(in, out, g, b, rows, cols, eps);
}
void ref_mat_mul_relu(const float *A, const float *B, float *C, int M, int N, int K) {
    opworks::ops::mat_mul(A, B, C, M, N, K, RefRelu{});
}
void ref_rms_norm(const float *x, const float *w, float *out, int rows, int cols, float eps) {
    opworks::ops::rms_norm(x, w, out, rows, cols, eps);
}
void ref_linear_f32(const float *X, const float *W, float *Y, int rows, int in, int out) {
    opworks::ops::linear(X, W, Y, rows, in, out);
}
void ref_rope(float *x, const float *inv_freq, int rows, int heads, int head_dim, int pos_start) {
    opworks::ops::rope(x, inv_freq, rows, heads, head_dim, pos_start);
}
void ref_attention_decode(const float *q, const float *k, const float *v, float *out, int qh, int rep, int D, int len,
                          int max_seq) {
    opworks::ops::attention_decode(q, k, v, out, qh, rep, D, len, max_seq);
}
void ref_attention_prefill_chunked(const float *q, const float *k, const float *v, float *out, int T, int S,
                                   int q_offset, int qh, int rep, int D, int cap) {
    opworks::ops::attention_prefill_chunked(q, k, v, out, T, S, q_offset, qh, rep, D, cap);
}
void ref_argmax(const float *x, int n, int *out) { opworks::ops::argmax(x, n, out); }
void ref_embedding_f32(const float *table, const int *ids, float *out, int n, int hidden) {
    opworks::ops::embedding(table, ids, out, n, hidden);
}
void ref_swiglu(const float *g, const float *u, float *out, long long n) { opworks::ops::swiglu(g, u, out, n); }
void ref_sync() { opworks::synchronize(); }
}

// ORACLE — test infrastructure only. CPU restatement of the OpWorks (reference)
// algorithms on the Llama hot path, used by tests/ as the parity checker and by
// bench.py's cpu_baseline / --impl reference arm as the timed CPU baseline. The
// product never links, loads or calls this code.
//
// Pinned against: the closed-form expectations of the reference's
// tests/unit/framework.cu:182-223, golden vectors produced by the reference's
// own Python math (scripts/llama/export_reference.py:32-88, imported by
// tests/golden/make_golden.py), a transformers LlamaForCausalLM forward with
// the same weights, and the reference's host sampler
// (examples/llama/generate.py:83-109) driven with the same uniforms.
//
// Numerics: fp32 storage, double accumulation (the "truth" the fp32 GPU
// kernels are compared against within the stated tolerances).

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0)
        omp_set_num_threads(n);
#else
    (void)n;
#endif
}

// ops::softmax (include/ops/softmax.cuh:10-29): max-subtracted exp / sum.
void orc_softmax(const float *in, float *out, int rows, int cols) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const float *x = in + static_cast<int64_t>(r) * cols;
        float *y = out + static_cast<int64_t>(r) * cols;
        double m = -INFINITY;
        for (int j = 0; j < cols; ++j)
            m = std::max(m, static_cast<double>(x[j]));
        double s = 0.0;
        for (int j = 0; j < cols; ++j)
            s += std::exp(static_cast<double>(x[j]) - m);
        for (int j = 0; j < cols; ++j)
            y[j] = static_cast<float>(std::exp(static_cast<double>(x[j]) - m) / s);
    }
}

// ops::layer_norm (include/ops/layer_norm.cuh:10-31): two-pass variance.
void orc_layer_norm(const float *in, float *out, const float *gamma, const float *beta, int rows, int cols,
                    float eps) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const float *x = in + static_cast<int64_t>(r) * cols;
        float *y = out + static_cast<int64_t>(r) * cols;
        double mean = 0.0;
        for (int j = 0; j < cols; ++j)
            mean += x[j];
        mean /= cols;
        double var = 0.0;
        for (int j = 0; j < cols; ++j)
            var += (x[j] - mean) * (x[j] - mean);
        var /= cols;
        const double rstd = 1.0 / std::sqrt(var + eps);
        for (int j = 0; j < cols; ++j)
            y[j] = static_cast<float>((x[j] - mean) * rstd * gamma[j] + beta[j]);
    }
}

// ops::mat_mul (include/ops/matmul.cuh:11-91): C(MxK) = epi(A(MxN) B(NxK)).
// epilogue 0 identity, 1 relu, 2 scale(param).
void orc_mat_mul(const float *A, const float *B, float *C, int M, int N, int K, int epilogue, float param) {
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m) {
        std::vector<double> acc(K, 0.0);
        for (int n = 0; n < N; ++n) {
            const double a = A[static_cast<int64_t>(m) * N + n];
            const float *b = B + static_cast<int64_t>(n) * K;
            for (int k = 0; k < K; ++k)
                acc[k] += a * b[k];
        }
        for (int k = 0; k < K; ++k) {
            double v = acc[k];
            if (epilogue == 1)
                v = v > 0.0 ? v : 0.0;
            else if (epilogue == 2)
                v = v * param;
            C[static_cast<int64_t>(m) * K + k] = static_cast<float>(v);
        }
    }
}

double orc_reduce_sum(const float *in, int64_t n) {
    double s = 0.0;
#pragma omp parallel for reduction(+ : s) schedule(static)
    for (int64_t i = 0; i < n; ++i)
        s += in[i];
    return s;
}

// rms_norm: export_reference.py:32-34 / include/ops/rms_norm.cuh:9-24.
void orc_rms_norm(const float *x, const float *w, float *out, int rows, int cols, float eps) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const float *xr = x + static_cast<int64_t>(r) * cols;
        float *o = out + static_cast<int64_t>(r) * cols;
        double ss = 0.0;
        for (int j = 0; j < cols; ++j)
            ss += static_cast<double>(xr[j]) * xr[j];
        const double inv = 1.0 / std::sqrt(ss / cols + eps);
        for (int j = 0; j < cols; ++j)
            o[j] = static_cast<float>(xr[j] * inv * w[j]);
    }
}

// Double-accumulated dot product with eight independent partial sums (fixed
// order, so results are deterministic; the independent chains let the CPU
// pipeline the FMAs instead of waiting on one accumulator).
static inline double dot_f64(const float *x, const float *w, int n) {
    double a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= n; i += 8)
        for (int j = 0; j < 8; ++j)
            a[j] += static_cast<double>(x[i + j]) * w[i + j];
    for (; i < n; ++i)
        a[0] += static_cast<double>(x[i]) * w[i];
    return ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
}

// Y[rows, out] = X[rows, in] @ W[out, in]^T (include/ops/linear.cuh:18-121).
// Each weight row is streamed once for all rows of X.
// Four dot products of one x row against four weight rows, each summed in
// exactly dot_f64's order (same lanes, same tree), so the blocked linear
// below is bit-identical to the unblocked one; one x load feeds four FMAs.
// (A float x float product is exact in double, so a fused multiply-add of
// the widened operands rounds exactly like the scalar multiply and add.) The
// weight rows come pre-widened to double (wd, 4 x n), converted once per
// block of outputs.
typedef double v4d __attribute__((vector_size(32)));
typedef float v4f __attribute__((vector_size(16)));
static inline v4d load4d(const float *p) {
    v4f f;
    std::memcpy(&f, p, sizeof(f));
    return __builtin_convertvector(f, v4d);
}
static inline v4d load4dd(const double *p) {
    v4d d;
    std::memcpy(&d, p, sizeof(d));
    return d;
}
static inline v4d fma4(v4d a, v4d b, v4d c) {
#if defined(__FMA__)
    return __builtin_ia32_vfmaddpd256(a, b, c);
#else
    return a * b + c;
#endif
}
static inline void dot4_f64(const float *x, const double *wd, int n, double out[4]) {
    v4d lo[4] = {}, hi[4] = {}; // lanes 0-3 and 4-7 of dot_f64's eight partial sums
    int i = 0;
    for (; i + 8 <= n; i += 8) {
        const v4d x0 = load4d(x + i), x1 = load4d(x + i + 4);
        for (int k = 0; k < 4; ++k) {
            lo[k] = fma4(x0, load4dd(wd + static_cast<int64_t>(k) * n + i), lo[k]);
            hi[k] = fma4(x1, load4dd(wd + static_cast<int64_t>(k) * n + i + 4), hi[k]);
        }
    }
    for (int k = 0; k < 4; ++k) {
        double a[8];
        for (int j = 0; j < 4; ++j) {
            a[j] = lo[k][j];
            a[j + 4] = hi[k][j];
        }
        for (int t = i; t < n; ++t)
            a[0] += static_cast<double>(x[t]) * wd[static_cast<int64_t>(k) * n + t];
        out[k] = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
    }
}

void orc_linear(const float *X, const float *W, float *Y, int rows, int in, int out) {
    const int blocks = (out + 3) / 4;
#pragma omp parallel for schedule(dynamic, 4)
    for (int b = 0; b < blocks; ++b) {
        const int o0 = b * 4;
        if (o0 + 4 <= out) {
            thread_local std::vector<double> wd;
            wd.resize(static_cast<size_t>(4) * in);
            for (int64_t i = 0; i < static_cast<int64_t>(4) * in; ++i)
                wd[i] = W[static_cast<int64_t>(o0) * in + i];
            for (int r = 0; r < rows; ++r) {
                double d[4];
                dot4_f64(X + static_cast<int64_t>(r) * in, wd.data(), in, d);
                for (int k = 0; k < 4; ++k)
                    Y[static_cast<int64_t>(r) * out + o0 + k] = static_cast<float>(d[k]);
            }
        } else {
            for (int o = o0; o < out; ++o) {
                const float *w = W + static_cast<int64_t>(o) * in;
                for (int r = 0; r < rows; ++r)
                    Y[static_cast<int64_t>(r) * out + o] =
                        static_cast<float>(dot_f64(X + static_cast<int64_t>(r) * in, w, in));
            }
        }
    }
}

// Same with bf16 weights (raw uint16 bits).
void orc_linear_bf16(const float *X, const uint16_t *W, float *Y, int rows, int in, int out) {
#pragma omp parallel for schedule(static) collapse(2)
    for (int r = 0; r < rows; ++r)
        for (int o = 0; o < out; ++o) {
            const float *x = X + static_cast<int64_t>(r) * in;
            const uint16_t *w = W + static_cast<int64_t>(o) * in;
            double acc = 0.0;
            for (int i = 0; i < in; ++i) {
                const uint32_t bits = static_cast<uint32_t>(w[i]) << 16;
                float wf;
                std::memcpy(&wf, &bits, 4);
                acc += static_cast<double>(x[i]) * wf;
            }
            Y[static_cast<int64_t>(r) * out + o] = static_cast<float>(acc);
        }
}

// llama3 inv_freq in double (runtime/model_config.cuh:68-89,
// export_reference.py:37-52).
void orc_rope_inv_freq(int head_dim, double theta, int llama3, double factor, double low_freq, double high_freq,
                       double orig_max_pos, float *out) {
    const double pi = 3.14159265358979323846;
    for (int i = 0; i < head_dim / 2; ++i) {
        double f = 1.0 / std::pow(theta, (2.0 * i) / head_dim);
        if (llama3) {
            const double wavelen = 2.0 * pi / f;
            const double low_wl = orig_max_pos / low_freq;
            const double high_wl = orig_max_pos / high_freq;
            if (wavelen > low_wl) {
                f /= factor;
            } else if (wavelen >= high_wl) {
                const double smooth = (orig_max_pos / wavelen - low_freq) / (high_freq - low_freq);
                f = (1.0 - smooth) * f / factor + smooth * f;
            }
        }
        out[i] = static_cast<float>(f);
    }
}

// rotate_half RoPE, angle = fp32(pos) * inv_freq in fp32 (as the reference's
// kernel and HF compute it), cos/sin evaluated in double
// (export_reference.py:55-68, include/ops/rope.cuh:10-25).
void orc_rope(float *x, const float *inv_freq, int rows, int heads, int head_dim, int pos_start) {
    const int half = head_dim / 2;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r)
        for (int h = 0; h < heads; ++h)
            for (int i = 0; i < half; ++i) {
                const float angle = static_cast<float>(pos_start + r) * inv_freq[i];
                const double c = std::cos(static_cast<double>(angle)), s = std::sin(static_cast<double>(angle));
                float *p = x + (static_cast<int64_t>(r) * heads + h) * head_dim + i;
                const double a = p[0], b = p[half];
                p[0] = static_cast<float>(a * c - b * s);
                p[half] = static_cast<float>(b * c + a * s);
            }
}

// causal GQA attention (export_reference.py:71-84): q [T, qh, D], k/v
// [S, kvh, D], query t sits at position S - T + t.
void orc_attention(const float *q, const float *k, const float *v, float *out, int T, int S, int qh, int kvh, int D) {
    const int rep = qh / kvh;
    const double scale = 1.0 / std::sqrt(static_cast<double>(D));
#pragma omp parallel for schedule(dynamic) collapse(2)
    for (int t = 0; t < T; ++t)
        for (int h = 0; h < qh; ++h) {
            const int g = h / rep;
            const int last = S - T + t;
            const float *qv = q + (static_cast<int64_t>(t) * qh + h) * D;
            std::vector<double> sc(last + 1);
            double m = -INFINITY;
            for (int s = 0; s <= last; ++s) {
                const float *kv = k + (static_cast<int64_t>(s) * kvh + g) * D;
                double d = 0.0;
                for (int i = 0; i < D; ++i)
                    d += static_cast<double>(qv[i]) * kv[i];
                sc[s] = d * scale;
                m = std::max(m, sc[s]);
            }
            double z = 0.0;
            for (int s = 0; s <= last; ++s) {
                sc[s] = std::exp(sc[s] - m);
                z += sc[s];
            }
            // every output dim sums its terms in key order s = 0..last
            float *o = out + (static_cast<int64_t>(t) * qh + h) * D;
            std::vector<double> acc(D, 0.0);
            for (int s = 0; s <= last; ++s) {
                const float *vr = v + (static_cast<int64_t>(s) * kvh + g) * D;
                for (int i = 0; i < D; ++i)
                    acc[i] += sc[s] * vr[i];
            }
            for (int i = 0; i < D; ++i)
                o[i] = static_cast<float>(acc[i] / z);
        }
}

// silu(g) * u (export_reference.py:87-88, include/ops/swiglu.cuh:7-12).
void orc_swiglu(const float *g, const float *u, float *out, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const double x = g[i];
        out[i] = static_cast<float>(x / (1.0 + std::exp(-x)) * u[i]);
    }
}

// first index of the maximum (include/ops/argmax.cuh:9-51).
int orc_argmax(const float *x, int n) {
    int best = 0;
    for (int i = 1; i < n; ++i)
        if (x[i] > x[best])
            best = i;
    return best;
}

// ----------------------------------------------------------- Llama forward

// Host weights of one Llama model (fp32), pointers into caller memory.
struct OrcLlama {
    int layers, hidden, inter, qh, kvh, head_dim, vocab;
    float eps;
    const float *embed;      // [V, H] (tied LM head)
    const float *final_norm; // [H]
    const float *const *input_norm, *const *q_proj, *const *k_proj, *const *v_proj, *const *o_proj;
    const float *const *post_norm, *const *gate_proj, *const *up_proj, *const *down_proj;
    const float *inv_freq; // [D/2]
};

// Forward of `n` tokens at positions [pos, pos + n) of one sequence (the op
// order of include/models/llama.cuh:216-285). kcache/vcache: [L][kvh][cap][D]
// (positions < pos already filled). hidden_trace (optional): (L + 1) x n x H
// residual stream after embedding and after each layer. logits: [V] of the
// last position. Returns 0.
int orc_llama_forward(const OrcLlama *m, const int32_t *ids, int n, int pos, float *kcache, float *vcache, int cap,
                      float *hidden_trace, float *logits) {
    const int H = m->hidden, I = m->inter, D = m->head_dim, qh = m->qh, kvh = m->kvh;
    const int S = pos + n;
    std::vector<float> x(static_cast<size_t>(n) * H), h(static_cast<size_t>(n) * H);
    std::vector<float> q(static_cast<size_t>(n) * qh * D), kk(static_cast<size_t>(n) * kvh * D),
        vv(static_cast<size_t>(n) * kvh * D);
    std::vector<float> att(static_cast<size_t>(n) * qh * D), o(static_cast<size_t>(n) * H);
    std::vector<float> g(static_cast<size_t>(n) * I), u(static_cast<size_t>(n) * I);
    for (int t = 0; t < n; ++t)
        std::memcpy(&x[static_cast<size_t>(t) * H], m->embed + static_cast<int64_t>(ids[t]) * H, sizeof(float) * H);
    if (hidden_trace)
        std::memcpy(hidden_trace, x.data(), sizeof(float) * x.size());
    std::vector<float> kfull(static_cast<size_t>(S) * kvh * D), vfull(static_cast<size_t>(S) * kvh * D);
    for (int l = 0; l < m->layers; ++l) {
        float *kc = kcache + static_cast<int64_t>(l) * kvh * cap * D;
        float *vc = vcache + static_cast<int64_t>(l) * kvh * cap * D;
        orc_rms_norm(x.data(), m->input_norm[l], h.data(), n, H, m->eps);
        orc_linear(h.data(), m->q_proj[l], q.data(), n, H, qh * D);
        orc_linear(h.data(), m->k_proj[l], kk.data(), n, H, kvh * D);
        orc_linear(h.data(), m->v_proj[l], vv.data(), n, H, kvh * D);
        orc_rope(q.data(), m->inv_freq, n, qh, D, pos);
        orc_rope(kk.data(), m->inv_freq, n, kvh, D, pos);
        for (int t = 0; t < n; ++t)
            for (int g2 = 0; g2 < kvh; ++g2)
                for (int i = 0; i < D; ++i) {
                    kc[(static_cast<int64_t>(g2) * cap + pos + t) * D + i] = kk[(static_cast<size_t>(t) * kvh + g2) * D + i];
                    vc[(static_cast<int64_t>(g2) * cap + pos + t) * D + i] = vv[(static_cast<size_t>(t) * kvh + g2) * D + i];
                }
        for (int s = 0; s < S; ++s)
            for (int g2 = 0; g2 < kvh; ++g2)
                for (int i = 0; i < D; ++i) {
                    kfull[(static_cast<size_t>(s) * kvh + g2) * D + i] = kc[(static_cast<int64_t>(g2) * cap + s) * D + i];
                    vfull[(static_cast<size_t>(s) * kvh + g2) * D + i] = vc[(static_cast<int64_t>(g2) * cap + s) * D + i];
                }
        orc_attention(q.data(), kfull.data(), vfull.data(), att.data(), n, S, qh, kvh, D);
        orc_linear(att.data(), m->o_proj[l], o.data(), n, qh * D, H);
        for (size_t i = 0; i < x.size(); ++i)
            x[i] += o[i];
        orc_rms_norm(x.data(), m->post_norm[l], h.data(), n, H, m->eps);
        orc_linear(h.data(), m->gate_proj[l], g.data(), n, H, I);
        orc_linear(h.data(), m->up_proj[l], u.data(), n, H, I);
        orc_swiglu(g.data(), u.data(), g.data(), static_cast<int64_t>(n) * I);
        orc_linear(g.data(), m->down_proj[l], o.data(), n, I, H);
        for (size_t i = 0; i < x.size(); ++i)
            x[i] += o[i];
        if (hidden_trace)
            std::memcpy(hidden_trace + static_cast<size_t>(l + 1) * n * H, x.data(), sizeof(float) * x.size());
    }
    orc_rms_norm(x.data() + static_cast<size_t>(n - 1) * H, m->final_norm, h.data(), 1, H, m->eps);
    orc_linear(h.data(), m->embed, logits, 1, H, m->vocab);
    return 0;
}

// Batched decode step of B sequences (the CPU baseline of the bs32 decode
// workload): ids[B], positions pos[B]; caches [B][L][kvh][cap][D]; logits
// [B][V]. Weights are streamed once per step for all B rows.
int orc_llama_decode_batch(const OrcLlama *m, const int32_t *ids, const int32_t *pos, int B, float *kcache,
                           float *vcache, int cap, float *logits) {
    const int H = m->hidden, I = m->inter, D = m->head_dim, qh = m->qh, kvh = m->kvh, L = m->layers;
    std::vector<float> x(static_cast<size_t>(B) * H), h(x.size()), o(x.size());
    std::vector<float> q(static_cast<size_t>(B) * qh * D), kk(static_cast<size_t>(B) * kvh * D), vv(kk.size());
    std::vector<float> att(q.size()), g(static_cast<size_t>(B) * I), u(g.size());
    for (int b = 0; b < B; ++b)
        std::memcpy(&x[static_cast<size_t>(b) * H], m->embed + static_cast<int64_t>(ids[b]) * H, sizeof(float) * H);
    const int64_t seq_stride = static_cast<int64_t>(L) * kvh * cap * D;
    for (int l = 0; l < L; ++l) {
        orc_rms_norm(x.data(), m->input_norm[l], h.data(), B, H, m->eps);
        orc_linear(h.data(), m->q_proj[l], q.data(), B, H, qh * D);
        orc_linear(h.data(), m->k_proj[l], kk.data(), B, H, kvh * D);
        orc_linear(h.data(), m->v_proj[l], vv.data(), B, H, kvh * D);
#pragma omp parallel for schedule(dynamic)
        for (int b = 0; b < B; ++b) {
            orc_rope(&q[static_cast<size_t>(b) * qh * D], m->inv_freq, 1, qh, D, pos[b]);
            orc_rope(&kk[static_cast<size_t>(b) * kvh * D], m->inv_freq, 1, kvh, D, pos[b]);
        }
        const double scale = 1.0 / std::sqrt(static_cast<double>(D));
        const int rep = qh / kvh;
#pragma omp parallel for schedule(dynamic) collapse(2)
        for (int b = 0; b < B; ++b)
            for (int hq = 0; hq < qh; ++hq) {
                const int g2 = hq / rep;
                float *kc = kcache + b * seq_stride + (static_cast<int64_t>(l) * kvh + g2) * cap * D;
                float *vc = vcache + b * seq_stride + (static_cast<int64_t>(l) * kvh + g2) * cap * D;
                if (hq % rep == 0)
                    for (int i = 0; i < D; ++i) {
                        kc[static_cast<int64_t>(pos[b]) * D + i] = kk[(static_cast<size_t>(b) * kvh + g2) * D + i];
                        vc[static_cast<int64_t>(pos[b]) * D + i] = vv[(static_cast<size_t>(b) * kvh + g2) * D + i];
                    }
            }
#pragma omp parallel for schedule(dynamic) collapse(2)
        for (int b = 0; b < B; ++b)
            for (int hq = 0; hq < qh; ++hq) {
                const int g2 = hq / rep;
                const float *kc = kcache + b * seq_stride + (static_cast<int64_t>(l) * kvh + g2) * cap * D;
                const float *vc = vcache + b * seq_stride + (static_cast<int64_t>(l) * kvh + g2) * cap * D;
                const float *qv = &q[(static_cast<size_t>(b) * qh + hq) * D];
                const int len = pos[b] + 1;
                std::vector<double> sc(len);
                double mx = -INFINITY;
                for (int s = 0; s < len; ++s) {
                    double d = 0.0;
                    for (int i = 0; i < D; ++i)
                        d += static_cast<double>(qv[i]) * kc[static_cast<int64_t>(s) * D + i];
                    sc[s] = d * scale;
                    mx = std::max(mx, sc[s]);
                }
                double z = 0.0;
                std::vector<double> acc(D, 0.0);
                for (int s = 0; s < len; ++s) {
                    const double p = std::exp(sc[s] - mx);
                    z += p;
                    for (int i = 0; i < D; ++i)
                        acc[i] += p * vc[static_cast<int64_t>(s) * D + i];
                }
                for (int i = 0; i < D; ++i)
                    att[(static_cast<size_t>(b) * qh + hq) * D + i] = static_cast<float>(acc[i] / z);
            }
        orc_linear(att.data(), m->o_proj[l], o.data(), B, qh * D, H);
        for (size_t i = 0; i < x.size(); ++i)
            x[i] += o[i];
        orc_rms_norm(x.data(), m->post_norm[l], h.data(), B, H, m->eps);
        orc_linear(h.data(), m->gate_proj[l], g.data(), B, H, I);
        orc_linear(h.data(), m->up_proj[l], u.data(), B, H, I);
        orc_swiglu(g.data(), u.data(), g.data(), static_cast<int64_t>(B) * I);
        orc_linear(g.data(), m->down_proj[l], o.data(), B, I, H);
        for (size_t i = 0; i < x.size(); ++i)
            x[i] += o[i];
    }
    orc_rms_norm(x.data(), m->final_norm, h.data(), B, H, m->eps);
    orc_linear(h.data(), m->embed, logits, B, H, m->vocab);
    return 0;
}

// -------------------------------------------------------------- sampler

// Host top-p sampler of examples/llama/generate.py:83-109 with numpy's
// Generator.choice(V, p=probs) replaced by its inverse-CDF rule on one uniform
// u in [0, 1): probs = softmax(logits / max(T, 1e-6)) in float64; if
// top_p < 1 keep the sorted prefix with cumsum <= top_p plus the top token and
// the token where the cumsum crosses top_p, renormalise; then
// cdf = cumsum(probs) in index order, cdf /= cdf[-1], return the first index
// with cdf > u. Sort ties: descending probability, then ascending index.
int orc_top_p_sample(const float *logits, int V, double temperature, double top_p, double u) {
    std::vector<double> p(V);
    const double t = std::max(temperature, 1e-6);
    double mx = -INFINITY;
    for (int i = 0; i < V; ++i) {
        p[i] = static_cast<double>(logits[i]) / t;
        mx = std::max(mx, p[i]);
    }
    double z = 0.0;
    for (int i = 0; i < V; ++i) {
        p[i] = std::exp(p[i] - mx);
        z += p[i];
    }
    for (int i = 0; i < V; ++i)
        p[i] /= z;
    if (top_p < 1.0) {
        std::vector<int> order(V);
        for (int i = 0; i < V; ++i)
            order[i] = i;
        std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return p[a] > p[b]; });
        std::vector<char> keep(V, 0);
        double cum = 0.0;
        int cross = V;
        for (int j = 0; j < V; ++j) {
            cum += p[order[j]];
            if (cum <= top_p)
                keep[order[j]] = 1;
            if (cross == V && cum >= top_p)
                cross = j;
        }
        keep[order[0]] = 1;
        if (cross < V)
            keep[order[cross]] = 1;
        double kept = 0.0;
        for (int i = 0; i < V; ++i)
            if (!keep[i])
                p[i] = 0.0;
            else
                kept += p[i];
        for (int i = 0; i < V; ++i)
            p[i] /= kept;
    }
    double cdf = 0.0, total = 0.0;
    for (int i = 0; i < V; ++i)
        total += p[i];
    for (int i = 0; i < V; ++i) {
        cdf += p[i];
        if (cdf / total > u)
            return i;
    }
    return V - 1;
}

} // extern "C"

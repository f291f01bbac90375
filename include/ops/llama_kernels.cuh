#pragma once

// Fused kernels of the B200 Llama forward pass (one launch replaces 2-4 of the
// reference's per-op launches; see include/models/llama.cuh for the step):
//
//   embed_rmsnorm   hidden = table[id]; normed = rms_norm(hidden) * w
//   add_rmsnorm     hidden += sum of split-K partials; normed = rms_norm(hidden) * w
//   qkv_finalize    sum partials -> q, k, v; RoPE(q, k) from a cos/sin table;
//                   k, v written straight into the paged KV cache
//   silu_mul        sum partials of the interleaved gate/up GEMM -> silu(g) * u
//   sample          greedy argmax or exact top-p (float64) per sequence
//
// "normed"/"act" outputs go to an ActOut: bf16 (fast path, the GEMM operand
// directly) or fp32, optionally with the tf32 hi/lo split of the accurate
// (split-precision) GEMM path.

#include <cuda_bf16.h>

#include "../core/block_reduce.cuh"
#include "../core/cuda_utils.cuh"
#include "attention_kernels.cuh"
#include "detail/operand_prep.cuh"

namespace opworks::detail {

// Where a row-wise producer writes the operand of the next GEMM.
struct ActOut {
    __nv_bfloat16 *bf16 = nullptr; // fast path
    float *f32 = nullptr;          // accurate path (tf32 hi part when lo != nullptr)
    float *lo = nullptr;           // tf32 lo part (split-precision GEMM)
    int64_t ld = 0;                // row stride (elements)
    __device__ __forceinline__ void put(int64_t row, int col, float v) const {
        const int64_t i = row * ld + col;
        if (bf16) {
            bf16[i] = __float2bfloat16_rn(v);
        } else if (lo) {
            const float h = tf32_round(v);
            f32[i] = h;
            lo[i] = v - h;
        } else {
            f32[i] = v;
        }
    }
};

constexpr int kRowThreads = 256;

// Sum of the squares of a row held as kPer values per thread, block-wide.
__device__ __forceinline__ float row_sumsq_block(float ss) { return block_reduce_all<ReduceSum>(ss); }

// One CTA per token row; cols == kRowThreads * kPer.
template <int kPer, typename WT>
__global__ void __launch_bounds__(kRowThreads)
    embed_rmsnorm_kernel(const WT *__restrict__ table, const int *__restrict__ ids, float *__restrict__ hidden,
                         const float *__restrict__ w, float eps, ActOut out, int cols) {
    const int64_t row = blockIdx.x;
    const WT *src = table + static_cast<int64_t>(ids[row]) * cols;
    float v[kPer];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int c = threadIdx.x + i * kRowThreads;
        v[i] = to_f32(src[c]);
        hidden[row * cols + c] = v[i];
        ss += v[i] * v[i];
    }
    const float inv = rsqrtf(row_sumsq_block(ss) / cols + eps);
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int c = threadIdx.x + i * kRowThreads;
        out.put(row, c, v[i] * inv * w[c]);
    }
}

// hidden[row] += sum_{s < splits} part[s][row]; normed = rms_norm(hidden) * w.
template <int kPer>
__global__ void __launch_bounds__(kRowThreads)
    add_rmsnorm_kernel(float *__restrict__ hidden, const float *__restrict__ part, int splits, int64_t split_stride,
                       const float *__restrict__ w, float eps, ActOut out, int cols) {
    const int64_t row = blockIdx.x;
    float v[kPer];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int c = threadIdx.x + i * kRowThreads;
        const int64_t idx = row * cols + c;
        float x = hidden[idx];
        for (int s = 0; s < splits; ++s)
            x += part[s * split_stride + idx];
        hidden[idx] = x;
        v[i] = x;
        ss += x * x;
    }
    const float inv = rsqrtf(row_sumsq_block(ss) / cols + eps);
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int c = threadIdx.x + i * kRowThreads;
        out.put(row, c, v[i] * inv * w[c]);
    }
}

// Token rows of a forward step: sequence slot and absolute position.
struct TokenMap {
    const int *seq; // [rows] block-table row
    const int *pos; // [rows] absolute position
};

// part: [splits][rows][qkv] with qkv = (qh + 2 kvh) * 64 columns (q | k | v).
// q_out: [rows][qh][64] fp32. rope: [max_pos][32][2] (cos, sin) fp32.
// One CTA (256 threads) per token row.
static __global__ void __launch_bounds__(256)
    qkv_finalize_kernel(const float *__restrict__ part, int splits, int64_t split_stride, int qh, int kvh,
                        const float2 *__restrict__ rope, TokenMap tm, PagedKV kv, float *__restrict__ kpool,
                        float *__restrict__ vpool, float *__restrict__ q_out) {
    const int64_t row = blockIdx.x;
    const int width = (qh + 2 * kvh) * kAttnD;
    const float *src = part + row * width;
    const int pos = tm.pos[row];
    const int seq = tm.seq[row];
    const float2 *cs = rope + static_cast<int64_t>(pos) * (kAttnD / 2);
    const int blk = kv.table[static_cast<int64_t>(seq) * kv.table_stride + pos / kKvChunk];
    const int slot = pos % kKvChunk;
    // rotated pairs of q and k heads: (head, i) for i < 32
    for (int pi = threadIdx.x; pi < (qh + kvh) * (kAttnD / 2); pi += blockDim.x) {
        const int head = pi / (kAttnD / 2), i = pi % (kAttnD / 2);
        const int c0 = head * kAttnD + i;
        float a = src[c0], b = src[c0 + kAttnD / 2];
        for (int s = 1; s < splits; ++s) {
            a += src[s * split_stride + c0];
            b += src[s * split_stride + c0 + kAttnD / 2];
        }
        const float2 r = cs[i];
        const float ra = a * r.x - b * r.y;
        const float rb = b * r.x + a * r.y;
        if (head < qh) {
            float *q = q_out + row * qh * kAttnD + head * kAttnD;
            q[i] = ra;
            q[i + kAttnD / 2] = rb;
        } else {
            const int h = head - qh;
            float *k = kpool + ((static_cast<int64_t>(blk) * kvh + h) * kKvChunk + slot) * kAttnD;
            k[i] = ra;
            k[i + kAttnD / 2] = rb;
        }
    }
    for (int j = threadIdx.x; j < kvh * kAttnD; j += blockDim.x) {
        const int c = (qh + kvh) * kAttnD + j;
        float x = src[c];
        for (int s = 1; s < splits; ++s)
            x += src[s * split_stride + c];
        const int h = j / kAttnD, d = j % kAttnD;
        vpool[((static_cast<int64_t>(blk) * kvh + h) * kKvChunk + slot) * kAttnD + d] = x;
    }
}

// part: [splits][rows][2 * inter] with interleaved columns (2j = gate_j,
// 2j + 1 = up_j); act[row][j] = silu(g) * u = g / (1 + exp(-g)) * u.
static __global__ void silu_mul_kernel(const float *__restrict__ part, int splits, int64_t split_stride, int rows, int inter,
                                ActOut out) {
    OPWORKS_GRID_LOOP(i, static_cast<int64_t>(rows) * inter) {
        const int64_t row = i / inter;
        const int j = static_cast<int>(i % inter);
        const float2 *src = reinterpret_cast<const float2 *>(part + row * 2 * inter) + j;
        float2 gu = src[0];
        for (int s = 1; s < splits; ++s) {
            const float2 t = *reinterpret_cast<const float2 *>(
                reinterpret_cast<const float *>(src) + s * split_stride);
            gu.x += t.x;
            gu.y += t.y;
        }
        out.put(row, j, gu.x / (1.f + expf(-gu.x)) * gu.y);
    }
}

// cos/sin table of RoPE: table[pos][i] = (cosf(a), sinf(a)), a = fp32(pos) *
// inv_freq[i], the same fp32 expression as ops::rope.
static __global__ void rope_table_kernel(const float *__restrict__ inv_freq, int max_pos, int half, float2 *__restrict__ out) {
    OPWORKS_GRID_LOOP(i, static_cast<int64_t>(max_pos) * half) {
        const int pos = static_cast<int>(i / half), j = static_cast<int>(i % half);
        const float a = static_cast<float>(pos) * inv_freq[j];
        out[i] = make_float2(cosf(a), sinf(a));
    }
}

// fp32 weight -> bf16 copy with optional row interleave of two sources:
// dst row 2j = a[j], 2j + 1 = b[j] (b == nullptr: plain copy of a).
static __global__ void weights_to_bf16_kernel(const float *__restrict__ a, const float *__restrict__ b, int rows, int cols,
                                       __nv_bfloat16 *__restrict__ dst) {
    const int64_t total = static_cast<int64_t>(b ? 2 * rows : rows) * cols;
    OPWORKS_GRID_LOOP(i, total) {
        const int64_t r = i / cols, c = i % cols;
        const float *src = b ? ((r & 1) ? b : a) : a;
        const int64_t sr = b ? (r >> 1) : r;
        dst[i] = __float2bfloat16_rn(src[sr * cols + c]);
    }
}

// Same into a tf32 hi/lo pair.
static __global__ void weights_to_split_kernel(const float *__restrict__ a, const float *__restrict__ b, int rows, int cols,
                                        float *__restrict__ hi, float *__restrict__ lo) {
    const int64_t total = static_cast<int64_t>(b ? 2 * rows : rows) * cols;
    OPWORKS_GRID_LOOP(i, total) {
        const int64_t r = i / cols, c = i % cols;
        const float *src = b ? ((r & 1) ? b : a) : a;
        const int64_t sr = b ? (r >> 1) : r;
        const float x = src[sr * cols + c];
        const float h = tf32_round(x);
        hi[i] = h;
        lo[i] = x - h;
    }
}

// Same into fp32 (interleave only).
static __global__ void weights_interleave_kernel(const float *__restrict__ a, const float *__restrict__ b, int rows, int cols,
                                          float *__restrict__ dst) {
    const int64_t total = static_cast<int64_t>(2 * rows) * cols;
    OPWORKS_GRID_LOOP(i, total) {
        const int64_t r = i / cols, c = i % cols;
        dst[i] = ((r & 1) ? b : a)[(r >> 1) * cols + c];
    }
}

// bf16 weight rows interleave (bf16 packs): dst 2j = a[j], 2j+1 = b[j].
static __global__ void bf16_interleave_kernel(const __nv_bfloat16 *__restrict__ a, const __nv_bfloat16 *__restrict__ b,
                                       int rows, int cols, __nv_bfloat16 *__restrict__ dst) {
    const int64_t total = static_cast<int64_t>(2 * rows) * cols;
    OPWORKS_GRID_LOOP(i, total) {
        const int64_t r = i / cols, c = i % cols;
        dst[i] = ((r & 1) ? b : a)[(r >> 1) * cols + c];
    }
}

// ------------------------------------------------------------------ sampler

// Per-row sampling controls of one decode step.
struct SampleParams {
    const float *temperature; // [rows]; <= 0 selects greedy argmax
    const float *top_p;       // [rows]
    const double *uniform;    // [rows] host-supplied uniforms (< 0: use seed/step), or nullptr
    const uint64_t *seed;     // [rows] counter-based uniforms when uniform == nullptr
    const int *step;          // [rows]
};

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

// Uniform in [0, 1) with 53 random bits from (seed, step).
__device__ __forceinline__ double counter_uniform(uint64_t seed, int step) {
    const uint64_t h = splitmix64(splitmix64(seed) ^ (static_cast<uint64_t>(step) * 0xd1b54a32d192ed03ull));
    return static_cast<double>(h >> 11) * (1.0 / 9007199254740992.0);
}

// Order-preserving key of a float (larger float -> larger key; NaN excluded).
__device__ __forceinline__ uint32_t float_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kSampleThreads = 1024;
constexpr int kRadixBits = 11;
constexpr int kRadixBuckets = 1 << kRadixBits;

__device__ __forceinline__ double block_sum_d(double v, double *scratch) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
        v += __shfl_xor_sync(kFullWarpMask, v, off);
    __syncthreads();
    if ((threadIdx.x & 31) == 0)
        scratch[threadIdx.x >> 5] = v;
    __syncthreads();
    double t = 0.0;
    for (int w = 0; w < kSampleThreads / 32; ++w)
        t += scratch[w];
    return t;
}

// Exclusive prefix (over threads in index order) of a per-thread double and int.
__device__ __forceinline__ void block_exclusive_scan(double v, int c, double *dscr, int *iscr, double &v_before,
                                                     int &c_before, double &v_total, int &c_total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    double vi = v;
    int ci = c;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const double vo = __shfl_up_sync(kFullWarpMask, vi, off);
        const int co = __shfl_up_sync(kFullWarpMask, ci, off);
        if (lane >= off) {
            vi += vo;
            ci += co;
        }
    }
    __syncthreads();
    if (lane == 31) {
        dscr[warp] = vi;
        iscr[warp] = ci;
    }
    __syncthreads();
    double wv = 0.0, tv = 0.0;
    int wc = 0, tc = 0;
    for (int w = 0; w < kSampleThreads / 32; ++w) {
        if (w < warp) {
            wv += dscr[w];
            wc += iscr[w];
        }
        tv += dscr[w];
        tc += iscr[w];
    }
    v_before = wv + vi - v;
    c_before = wc + ci - c;
    v_total = tv;
    c_total = tc;
}

// One CTA per row of `logits` ([rows][vocab] fp32). Greedy: first index of the
// maximum. Top-p: the host sampler of OpWorks examples/llama/generate.py:83-109
// in float64 — p = softmax(logits / max(T, 1e-6)); keep the descending-sorted
// prefix up to and including the first token whose cumulative mass reaches
// top_p (ties at that boundary kept in ascending index order); renormalise;
// return the first index whose cumulative kept mass exceeds u (numpy's
// Generator.choice rule). The sorted order is found by a 3-level radix
// select on the float bits of the logits, so no sort is materialised.
static __global__ void __launch_bounds__(kSampleThreads)
    sample_kernel(const float *__restrict__ logits, int64_t ld, int vocab, SampleParams sp, int *__restrict__ out) {
    __shared__ double hist[kRadixBuckets];
    __shared__ int cnt[kRadixBuckets];
    __shared__ double dscr[32];
    __shared__ int iscr[32];
    __shared__ float best_v[32];
    __shared__ int best_i[32];
    __shared__ uint32_t s_prefix;
    __shared__ double s_above;
    __shared__ int s_above_cnt;

    const int row = blockIdx.x;
    const float *x = logits + static_cast<int64_t>(row) * ld;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // pass 1: max (first index)
    float bv = kNegInf;
    int bi = 0x7fffffff;
    for (int i = tid; i < vocab; i += blockDim.x) {
        const float v = x[i];
        if (v > bv || (v == bv && i < bi)) {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(kFullWarpMask, bv, off);
        const int oi = __shfl_xor_sync(kFullWarpMask, bi, off);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if (lane == 0) {
        best_v[warp] = bv;
        best_i[warp] = bi;
    }
    __syncthreads();
    bv = best_v[0];
    bi = best_i[0];
    for (int w = 1; w < 32; ++w)
        if (best_v[w] > bv || (best_v[w] == bv && best_i[w] < bi)) {
            bv = best_v[w];
            bi = best_i[w];
        }
    const float temp = sp.temperature ? sp.temperature[row] : 0.f;
    if (!(temp > 0.f)) {
        if (tid == 0)
            out[row] = bi;
        return;
    }
    const double t = fmax(static_cast<double>(temp), 1e-6);
    const double zmax = static_cast<double>(bv) / t;
    const double top_p = sp.top_p ? static_cast<double>(sp.top_p[row]) : 1.0;
    // host-supplied uniform when >= 0, else the counter-based stream
    const double u = (sp.uniform && sp.uniform[row] >= 0.0)
                         ? sp.uniform[row]
                         : counter_uniform(sp.seed ? sp.seed[row] : 0ull, sp.step ? sp.step[row] : 0);

    // mass of every token: e_i = exp(l_i / T - zmax)
    double z = 0.0;
    for (int i = tid; i < vocab; i += blockDim.x)
        z += exp(static_cast<double>(x[i]) / t - zmax);
    z = block_sum_d(z, dscr);

    // radix select of the crossing key: largest k with mass(key >= k) >= p z
    uint32_t prefix = 0;
    double above = 0.0; // mass with key above the current prefix range
    int above_cnt = 0;
    uint32_t key_star = 0;
    double e_star = 0.0;
    int n_keep_ties = 0x7fffffff;
    bool filtered = top_p < 1.0;
    if (filtered) {
        const double target = top_p * z;
        for (int level = 0; level < 3; ++level) {
            const int shift = level == 0 ? 21 : (level == 1 ? 10 : 0);
            const int nb = level == 2 ? (1 << 10) : kRadixBuckets;
            const uint32_t mask_hi = level == 0 ? 0u : (0xffffffffu << (level == 1 ? 21 : 10));
            for (int b = tid; b < nb; b += blockDim.x) {
                hist[b] = 0.0;
                cnt[b] = 0;
            }
            __syncthreads();
            for (int i = tid; i < vocab; i += blockDim.x) {
                const float v = x[i];
                const uint32_t k = float_key(v);
                if ((k & mask_hi) == prefix) {
                    const int b = static_cast<int>((k >> shift) & static_cast<uint32_t>(nb - 1));
                    atomicAdd(&hist[b], exp(static_cast<double>(v) / t - zmax));
                    atomicAdd(&cnt[b], 1);
                }
            }
            __syncthreads();
            if (tid == 0) {
                double acc = above;
                int acc_cnt = above_cnt;
                int b = nb - 1;
                for (; b > 0; --b) {
                    if (acc + hist[b] >= target)
                        break;
                    acc += hist[b];
                    acc_cnt += cnt[b];
                }
                s_prefix = prefix | (static_cast<uint32_t>(b) << shift);
                s_above = acc;
                s_above_cnt = acc_cnt;
            }
            __syncthreads();
            prefix = s_prefix;
            above = s_above;
            above_cnt = s_above_cnt;
            __syncthreads();
        }
        key_star = prefix;
        // all tokens with key == key_star share one mass value
        float fstar;
        {
            const uint32_t u32 = (key_star & 0x80000000u) ? (key_star & 0x7fffffffu) : ~key_star;
            fstar = __uint_as_float(u32);
        }
        e_star = exp(static_cast<double>(fstar) / t - zmax);
        const double need = (target - above) / e_star;
        n_keep_ties = need <= 1.0 ? 1 : static_cast<int>(ceil(need - 1e-12));
        if (n_keep_ties < 1)
            n_keep_ties = 1;
    }

    // inverse-CDF over the kept tokens in index order: contiguous chunk/thread
    const int chunk = (vocab + blockDim.x - 1) / blockDim.x;
    const int lo = tid * chunk, hi = min(vocab, lo + chunk);
    double my = 0.0;
    int my_ties = 0;
    for (int i = lo; i < hi; ++i) {
        const float v = x[i];
        if (!filtered) {
            my += exp(static_cast<double>(v) / t - zmax);
        } else {
            const uint32_t k = float_key(v);
            if (k > key_star)
                my += exp(static_cast<double>(v) / t - zmax);
            else if (k == key_star)
                ++my_ties;
        }
    }
    // ties at the boundary: the first n_keep_ties (index order) are kept
    double before, total;
    int ties_before, ties_total;
    block_exclusive_scan(my, my_ties, dscr, iscr, before, ties_before, total, ties_total);
    if (filtered) {
        const int keep_total = min(n_keep_ties, ties_total);
        const int mine = max(0, min(my_ties, keep_total - ties_before));
        // recompute the running mass including this thread's kept ties
        const double tie_mass_before = e_star * static_cast<double>(min(ties_before, keep_total));
        before += tie_mass_before;
        my += e_star * mine;
        total += e_star * static_cast<double>(keep_total);
    }
    const double goal = u * total;
    if (before <= goal && goal < before + my) {
        double run = before;
        int ties_seen = ties_before;
        int pick = hi - 1;
        for (int i = lo; i < hi; ++i) {
            const float v = x[i];
            double e = 0.0;
            if (!filtered) {
                e = exp(static_cast<double>(v) / t - zmax);
            } else {
                const uint32_t k = float_key(v);
                if (k > key_star)
                    e = exp(static_cast<double>(v) / t - zmax);
                else if (k == key_star && ties_seen++ < n_keep_ties)
                    e = e_star;
            }
            if (e > 0.0) {
                run += e;
                if (run > goal) {
                    pick = i;
                    break;
                }
            }
        }
        out[row] = pick;
    }
    // numerical edge: goal at the very top (u -> 1) lands in no interval;
    // the last kept token is the answer (numpy's searchsorted clamps likewise)
    if (tid == blockDim.x - 1 && !(goal < total)) {
        int last = vocab - 1;
        for (int i = vocab - 1; i >= 0; --i) {
            const uint32_t k = float_key(x[i]);
            if (!filtered || k >= key_star) {
                last = i;
                break;
            }
        }
        out[row] = last;
    }
}

} // namespace opworks::detail

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

#include <cooperative_groups.h>
#include <cuda_bf16.h>

#include "../core/block_reduce.cuh"
#include "../core/cuda_utils.cuh"
#include "attention_kernels.cuh"
#include "detail/operand_prep.cuh"

namespace opworks::detail {

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

// Order-preserving key of a float (larger float -> larger key).
__device__ __forceinline__ uint32_t float_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

constexpr int kSampleCluster = 8;    // CTAs per row (portable cluster size)
constexpr int kSampleThreads = 512;  // threads per CTA
constexpr int kSampleChunkMax = 16384; // logits per CTA held in shared memory
constexpr int kRadixBuckets = 2048;

struct SampleShared {
    float x[kSampleChunkMax];      // this CTA's slice of the row
    double hist[kRadixBuckets];    // mass per radix bucket
    int cnt[kRadixBuckets];        // tokens per radix bucket
    double dscr[32];
    int iscr[32];
    float best_v;
    int best_i;
    double part_mass;              // final pass: kept mass of this CTA
    int part_ties;                 // final pass: boundary ties of this CTA
    // results of the leader (rank 0), read by every CTA through DSMEM
    uint32_t prefix;
    double above, z;
    int above_cnt;
};

// Block-wide exclusive prefix (threads in index order) of a double and an int.
__device__ __forceinline__ void block_scan_excl(double v, int c, double *dscr, int *iscr, double &v_before,
                                                int &c_before, double &v_total, int &c_total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
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
    for (int w = 0; w < nw; ++w) {
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

// One 8-CTA cluster per row of logits [rows][ld]. Greedy (temperature <= 0):
// first index of the maximum. Otherwise the host sampler of OpWorks
// examples/llama/generate.py:83-109: p = softmax(logits / max(T, 1e-6));
// keep the descending-sorted prefix up to and including the first token whose
// cumulative mass reaches top_p (tokens tied at that boundary are kept in
// ascending index order); renormalise; return the first index whose
// cumulative kept mass (index order) exceeds u * total, numpy's
// Generator.choice rule. The sorted order is found by a 3-level radix select
// over the float bits of the logits (11 + 11 + 10 bits) with per-bucket mass
// histograms; masses are expf in fp32 accumulated in fp64. Each CTA keeps its
// slice of the row in shared memory; partial results meet in the leader CTA
// through distributed shared memory.
static __global__ void __cluster_dims__(kSampleCluster, 1, 1) __launch_bounds__(kSampleThreads)
    sample_kernel(const float *__restrict__ logits, int64_t ld, int vocab, SampleParams sp, int *__restrict__ out) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(16) uint8_t smem_raw[];
    SampleShared &sh = *reinterpret_cast<SampleShared *>(smem_raw);
    const int rank = static_cast<int>(cluster.block_rank());
    const int row = blockIdx.x / kSampleCluster;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int chunk = (vocab + kSampleCluster - 1) / kSampleCluster;
    const int lo = rank * chunk;
    const int n = max(0, min(vocab, lo + chunk) - lo);
    const float *src = logits + static_cast<int64_t>(row) * ld + lo;
    SampleShared *leader = cluster.map_shared_rank(&sh, 0);

    // pass 0: stage the slice, local (max, first index)
    float bv = kNegInf;
    int bi = 0x7fffffff;
    for (int i = tid; i < n; i += blockDim.x) {
        const float v = src[i];
        sh.x[i] = v;
        if (v > bv) {
            bv = v;
            bi = lo + i;
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
        sh.dscr[warp] = bv;
        sh.iscr[warp] = bi;
    }
    __syncthreads();
    if (tid == 0) {
        float v = kNegInf;
        int i0 = 0x7fffffff;
        for (int w = 0; w < kSampleThreads / 32; ++w) {
            const float ov = static_cast<float>(sh.dscr[w]);
            if (ov > v || (ov == v && sh.iscr[w] < i0)) {
                v = ov;
                i0 = sh.iscr[w];
            }
        }
        sh.best_v = v;
        sh.best_i = i0;
    }
    cluster.sync();
    float gmax = kNegInf;
    int garg = 0x7fffffff;
    for (int r = 0; r < kSampleCluster; ++r) {
        const SampleShared *peer = cluster.map_shared_rank(&sh, r);
        const float v = peer->best_v;
        const int i0 = peer->best_i;
        if (v > gmax || (v == gmax && i0 < garg)) {
            gmax = v;
            garg = i0;
        }
    }
    const float temp = sp.temperature ? sp.temperature[row] : 0.f;
    if (!(temp > 0.f)) {
        if (rank == 0 && tid == 0)
            out[row] = garg;
        cluster.sync(); // peers finished reading this CTA's shared memory
        return;
    }
    const float inv_t = 1.f / fmaxf(temp, 1e-6f);
    const double top_p = sp.top_p ? static_cast<double>(sp.top_p[row]) : 1.0;
    const double u = (sp.uniform && sp.uniform[row] >= 0.0)
                         ? sp.uniform[row]
                         : counter_uniform(sp.seed ? sp.seed[row] : 0ull, sp.step ? sp.step[row] : 0);
    auto mass = [&](float v) { return expf((v - gmax) * inv_t); };

    const bool filtered = top_p < 1.0;
    uint32_t prefix = 0;
    double above = 0.0, z = 0.0;
    for (int level = 0; level < (filtered ? 3 : 1); ++level) {
        const int shift = level == 0 ? 21 : (level == 1 ? 10 : 0);
        const int nb = level == 2 ? 1024 : kRadixBuckets;
        const uint32_t mask_hi = level == 0 ? 0u : (0xffffffffu << (level == 1 ? 21 : 10));
        for (int b = tid; b < nb; b += blockDim.x) {
            sh.hist[b] = 0.0;
            sh.cnt[b] = 0;
        }
        __syncthreads();
        // warp-aggregated histogram: lanes hitting the same bucket are summed
        // in registers and one lane issues the shared-memory atomics (the
        // top-level buckets of a logit row are few and heavily shared)
        const int n_pad = (n + kWarpSize - 1) / kWarpSize * kWarpSize;
        for (int i = tid; i < n_pad; i += blockDim.x) {
            int b = -1;
            float e = 0.f;
            if (i < n) {
                const float v = sh.x[i];
                const uint32_t k = float_key(v);
                if ((k & mask_hi) == prefix) {
                    b = static_cast<int>((k >> shift) & static_cast<uint32_t>(nb - 1));
                    e = mass(v);
                }
            }
            const unsigned peers = __match_any_sync(kFullWarpMask, b);
            double sum = 0.0;
#pragma unroll 4
            for (int j = 0; j < kWarpSize; ++j) {
                const float ej = __shfl_sync(kFullWarpMask, e, j);
                if ((peers >> j) & 1u)
                    sum += static_cast<double>(ej);
            }
            if (b >= 0 && lane == __ffs(peers) - 1) {
                atomicAdd(&sh.hist[b], sum);
                atomicAdd(&sh.cnt[b], __popc(peers));
            }
        }
        cluster.sync();
        if (rank == 0) {
            // leader: sum the cluster's histograms; buckets scanned from the top
            const int per = nb / kSampleThreads; // 4 or 2 buckets per thread
            double my = 0.0;
            int myc = 0;
            double bm[4];
            int bc[4];
            for (int j = 0; j < per; ++j) {
                const int b = nb - 1 - (tid * per + j);
                double m = 0.0;
                int c = 0;
                for (int r = 0; r < kSampleCluster; ++r) {
                    const SampleShared *peer = cluster.map_shared_rank(&sh, r);
                    m += peer->hist[b];
                    c += peer->cnt[b];
                }
                bm[j] = m;
                bc[j] = c;
                my += m;
                myc += c;
            }
            double before, total;
            int cbefore, ctotal;
            block_scan_excl(my, myc, sh.dscr, sh.iscr, before, cbefore, total, ctotal);
            if (level == 0)
                z = total;
            else
                z = leader->z;
            const double target = top_p * z;
            if (!filtered) {
                if (tid == 0) {
                    sh.z = total;
                    sh.prefix = 0;
                    sh.above = 0.0;
                    sh.above_cnt = 0;
                }
            } else {
                // the crossing bucket: first (from the top) where above + cum >= target
                double acc = above + before;
                int accc = cbefore;
                for (int j = 0; j < per; ++j) {
                    const int b = nb - 1 - (tid * per + j);
                    const bool last_bucket = b == 0;
                    if ((acc + bm[j] >= target || last_bucket) && acc < target) {
                        sh.prefix = prefix | (static_cast<uint32_t>(b) << shift);
                        sh.above = acc;
                        sh.above_cnt = accc;
                    }
                    acc += bm[j];
                    accc += bc[j];
                }
                // target beyond everything (rounding): keep the lowest bucket
                if (tid == kSampleThreads - 1 && !(above + total >= target) && level == 0) {
                    sh.prefix = 0;
                    sh.above = above;
                    sh.above_cnt = 0;
                }
                if (tid == 0 && level == 0)
                    sh.z = total;
            }
        }
        cluster.sync();
        prefix = leader->prefix;
        above = leader->above;
        z = leader->z;
    }
    const uint32_t key_star = prefix;
    const double e_star = filtered ? static_cast<double>(mass(key_float(key_star))) : 0.0;
    int n_keep_ties = 0x7fffffff;
    if (filtered) {
        const double need = (top_p * z - above) / e_star;
        n_keep_ties = need <= 1.0 ? 1 : static_cast<int>(ceil(need - 1e-12));
    }

    // final pass: kept mass in index order; each thread owns a contiguous run
    const int per_t = (n + kSampleThreads - 1) / kSampleThreads;
    const int t_lo = min(n, tid * per_t), t_hi = min(n, t_lo + per_t);
    double my = 0.0;
    int my_ties = 0;
    for (int i = t_lo; i < t_hi; ++i) {
        const float v = sh.x[i];
        if (!filtered) {
            my += mass(v);
        } else {
            const uint32_t k = float_key(v);
            if (k > key_star)
                my += mass(v);
            else if (k == key_star)
                ++my_ties;
        }
    }
    double before, total;
    int ties_before, ties_total;
    block_scan_excl(my, my_ties, sh.dscr, sh.iscr, before, ties_before, total, ties_total);
    if (tid == 0) {
        sh.part_mass = total;
        sh.part_ties = ties_total;
    }
    cluster.sync();
    // cluster prefix over ranks (every CTA computes it from the peers)
    double rank_before = 0.0, grand = 0.0;
    int ties_rank_before = 0, ties_grand = 0;
    for (int r = 0; r < kSampleCluster; ++r) {
        const SampleShared *peer = cluster.map_shared_rank(&sh, r);
        if (r < rank) {
            rank_before += peer->part_mass;
            ties_rank_before += peer->part_ties;
        }
        grand += peer->part_mass;
        ties_grand += peer->part_ties;
    }
    const int keep_total = filtered ? min(n_keep_ties, ties_grand) : 0;
    const int tb = ties_rank_before + ties_before; // boundary ties before this thread
    const int mine = filtered ? max(0, min(my_ties, keep_total - tb)) : 0;
    const double t_before = rank_before + before + e_star * static_cast<double>(min(tb, keep_total));
    const double t_mine = my + e_star * static_cast<double>(mine);
    const double all = grand + e_star * static_cast<double>(keep_total);
    const double goal = u * all;
    if (t_before <= goal && goal < t_before + t_mine) {
        double run = t_before;
        int ties_seen = tb;
        int pick = lo + t_hi - 1;
        for (int i = t_lo; i < t_hi; ++i) {
            const float v = sh.x[i];
            double e = 0.0;
            if (!filtered) {
                e = mass(v);
            } else {
                const uint32_t k = float_key(v);
                if (k > key_star)
                    e = mass(v);
                else if (k == key_star && ties_seen++ < keep_total)
                    e = e_star;
            }
            if (e > 0.0) {
                run += e;
                if (run > goal) {
                    pick = lo + i;
                    break;
                }
            }
        }
        out[row] = pick;
    }
    // u -> 1 rounding: the goal lands past the last kept token
    if (rank == kSampleCluster - 1 && tid == 0 && !(goal < all)) {
        int last = vocab - 1;
        for (int r = kSampleCluster - 1; r >= 0 && last == vocab - 1; --r) {
            const SampleShared *peer = cluster.map_shared_rank(&sh, r);
            const int plo = r * chunk, pn = max(0, min(vocab, plo + chunk) - plo);
            for (int i = pn - 1; i >= 0; --i)
                if (!filtered || float_key(peer->x[i]) >= key_star) {
                    last = plo + i;
                    break;
                }
        }
        out[row] = last;
    }
    cluster.sync(); // keep shared memory alive until every peer is done with it
}

inline size_t sample_smem_bytes() { return sizeof(SampleShared); }

inline void sample_launch(const float *logits, int64_t ld, int rows, int vocab, const SampleParams &sp, int *out,
                          cudaStream_t stream) {
    require((vocab + kSampleCluster - 1) / kSampleCluster <= kSampleChunkMax, "vocabulary too large for the sampler");
    static thread_local int done = -1;
    int dev = 0;
    OPWORKS_CUDA_CHECK(cudaGetDevice(&dev));
    if (done != dev) {
        OPWORKS_CUDA_CHECK(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(sample_smem_bytes())));
        done = dev;
    }
    sample_kernel<<<rows * kSampleCluster, kSampleThreads, sample_smem_bytes(), stream>>>(logits, ld, vocab, sp, out);
    OPWORKS_CUDA_CHECK(cudaGetLastError());
}

} // namespace opworks::detail

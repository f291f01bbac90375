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
// "normed"/"act" outputs go to an ActOut: two-term 16-bit words (fast path,
// the GEMM operand directly; fp16 or bf16 by the model's format) or fp32,
// optionally with the tf32 hi/lo split of the accurate (split-precision) GEMM
// path.

#include <cooperative_groups.h>
#include <cuda_bf16.h>

#include "../core/block_reduce.cuh"
#include "../core/cuda_utils.cuh"
#include "attention_kernels.cuh"
#include "detail/operand_prep.cuh"
#include "gemm_sm100.cuh"

namespace opworks::detail {

constexpr int kRowThreads = 256;

// Sum of the squares of a row held as kPer values per thread, block-wide.
__device__ __forceinline__ float row_sumsq_block(float ss) { return block_reduce_all<ReduceSum>(ss); }

// Deferred RMSNorm of the residual stream (fast path). The per-token factor
// rsqrt(sum(h^2) / H + eps) commutes with the projection that consumes the
// normalised row, W (h * g * r) = r (W (h * g)), so the producer of h writes
// the GEMM operand h * g (no norm yet) plus one partial sum of squares per
// 128-feature tile, part[tile][row], and the consuming GEMM's epilogue scales
// its output by r, summing the tiles in order (deterministic).
struct RowSumSq {
    float *part = nullptr; // [tiles][ld]
    int64_t ld = 0;
    int tiles = 0;
    int cols = 0; // H
    float eps = 0.f;
    __device__ __forceinline__ float inv_rms(int64_t row) const {
        // unrolled so that the tiles' loads are in flight together (the
        // additions keep their order)
        float s = 0.f;
#pragma unroll 16
        for (int t = 0; t < tiles; ++t)
            s += part[t * ld + row];
        return rsqrtf(s / static_cast<float>(cols) + eps);
    }
};

// One CTA per token row; cols == kRowThreads * kPer. With rs.part set the
// norm is deferred (see RowSumSq): out = h * w and part[0][row] = sum(h^2),
// the other tiles 0.
template <int kPer, typename WT>
__global__ void __launch_bounds__(kRowThreads)
    embed_rmsnorm_kernel(const WT *__restrict__ table, const int *__restrict__ ids, float *__restrict__ hidden,
                         const float *__restrict__ w, float eps, ActOut out, int cols, RowSumSq rs) {
    pdl_trigger();
    pdl_wait();
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
    const float total = row_sumsq_block(ss);
    if (rs.part) {
        for (int t = threadIdx.x; t < rs.tiles; t += blockDim.x)
            rs.part[t * rs.ld + row] = t == 0 ? total : 0.f;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int c = threadIdx.x + i * kRowThreads;
            out.put(row, c, v[i] * w[c]);
        }
        return;
    }
    const float inv = rsqrtf(total / cols + eps);
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
    pdl_trigger();
    pdl_wait();
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
    pdl_trigger();
    pdl_wait();
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
    pdl_trigger();
    pdl_wait();
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

// ------------------------------------------------- fused GEMM tile epilogues
//
// Tile epilogues of the tcgen05 GEMM (sm100::umma_gemm_kernel): they receive
// finished fp32 values of tokens [tok0, tok0 + ntok) x features
// [f0, f0 + nfeat) as a shared-memory tile [ntok][128], on the 128 epilogue
// threads (tid), after the split-K reduction, plus 2 KB of shared scratch
// filled by their optional prepare().

// hidden[tok][f] += value: the o and down projections' residual add. With
// `gain` set it also writes the next projection's operand h * gain (two-term
// 16-bit) and, per token, the tile's partial sum of squares of h (RowSumSq).
struct ResidualTileEpi {
    static constexpr bool kTile = true;
    // scratch: [4 warps][kPreTok] sums of squares | gain[128] | rows[kPreTok][128]
    static constexpr int kPreTok = static_cast<int>((sm100::kEpiScratchNarrow - 1024) / 512);
    float *hidden;
    int64_t ld;
    const float *gain = nullptr;
    ActOut normed{};
    RowSumSq rs{};
    bool preload = false; // the GEMM's scratch is kEpiScratchNarrow bytes (BN <= 64)
    // while the main loop streams: the slice's residual rows and the gains
    // go to shared memory, so the epilogue does no global load
    __device__ __forceinline__ void prepare(int tok0, int ntok, int f0, int nfeat, int tid, void *scratch) const {
        if (!preload || ntok > kPreTok)
            return;
        float *sg = static_cast<float *>(scratch) + 4 * kPreTok;
        float *sh = sg + 128;
        const int c = tid;
        const bool col_ok = c < nfeat;
        sg[c] = (gain && col_ok) ? gain[f0 + c] : 0.f;
        const float *col = hidden + static_cast<int64_t>(tok0) * ld + f0 + c;
        // four rows in flight per step (a decode slice is one step): short
        // code, few instruction-cache lines on a cold SM
        for (int j0 = 0; j0 < ntok; j0 += 4) {
            float hv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                hv[u] = (col_ok && j0 + u < ntok) ? col[static_cast<int64_t>(j0 + u) * ld] : 0.f;
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (j0 + u < ntok)
                    sh[(j0 + u) * 128 + c] = hv[u];
        }
    }
    __device__ __forceinline__ void operator()(const float *tile, int tok0, int ntok, int f0, int nfeat, int tid,
                                               void *scratch) const {
        // warp w takes tokens w, w + 4, ...; lane l owns columns 4l .. 4l + 3
        // (16-byte loads and stores), so a token's sum of squares is one warp
        // reduction. The residual rows of kChunk tokens per warp are loaded
        // together (one memory latency per chunk), from the rows staged in
        // shared memory by prepare() when they fit.
        constexpr int kChunk = 2;
        const bool staged = preload && ntok <= kPreTok;
        const float *sg = static_cast<const float *>(scratch) + 4 * kPreTok;
        const float *sh = sg + 128;
        const int warp = tid >> 5, lane = tid & 31, c = 4 * lane;
        const bool vec = c + 3 < nfeat; // whole vector in range (nfeat is 128 on the model's shapes)
        float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
        if (gain) {
            if (staged)
                g = *reinterpret_cast<const float4 *>(sg + c);
            else if (vec)
                g = *reinterpret_cast<const float4 *>(gain + f0 + c);
            else {
                g.x = c < nfeat ? gain[f0 + c] : 0.f;
                g.y = c + 1 < nfeat ? gain[f0 + c + 1] : 0.f;
                g.z = c + 2 < nfeat ? gain[f0 + c + 2] : 0.f;
                g.w = c + 3 < nfeat ? gain[f0 + c + 3] : 0.f;
            }
        }
        float *base = hidden + static_cast<int64_t>(tok0) * ld + f0 + c;
        for (int tb = warp; tb < ntok; tb += 4 * kChunk) {
            float4 hv[kChunk];
#pragma unroll
            for (int j = 0; j < kChunk; ++j) {
                const int t = tb + 4 * j;
                hv[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (t < ntok) {
                    if (staged)
                        hv[j] = *reinterpret_cast<const float4 *>(sh + t * 128 + c);
                    else if (vec)
                        hv[j] = *reinterpret_cast<const float4 *>(base + static_cast<int64_t>(t) * ld);
                    else {
                        const float *r = base + static_cast<int64_t>(t) * ld;
                        hv[j].x = c < nfeat ? r[0] : 0.f;
                        hv[j].y = c + 1 < nfeat ? r[1] : 0.f;
                        hv[j].z = c + 2 < nfeat ? r[2] : 0.f;
                        hv[j].w = c + 3 < nfeat ? r[3] : 0.f;
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < kChunk; ++j) {
                const int t = tb + 4 * j;
                if (t >= ntok) // the same for every lane of the warp
                    break;
                const float4 v = *reinterpret_cast<const float4 *>(tile + t * 128 + c);
                const float4 h = make_float4(hv[j].x + v.x, hv[j].y + v.y, hv[j].z + v.z, hv[j].w + v.w);
                float *r = base + static_cast<int64_t>(t) * ld;
                if (vec) {
                    *reinterpret_cast<float4 *>(r) = h;
                    if (gain)
                        normed.put4c(tok0 + t, f0 + c, make_float4(h.x * g.x, h.y * g.y, h.z * g.z, h.w * g.w));
                } else {
                    const float hh[4] = {h.x, h.y, h.z, h.w}, gg[4] = {g.x, g.y, g.z, g.w};
                    for (int e = 0; e < 4; ++e)
                        if (c + e < nfeat) {
                            r[e] = hh[e];
                            if (gain)
                                normed.put(tok0 + t, f0 + c + e, hh[e] * gg[e]);
                        }
                }
                if (rs.part) {
                    // columns past nfeat hold 0 (zero-filled operands)
                    float sq = (h.x * h.x + h.y * h.y) + (h.z * h.z + h.w * h.w);
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1)
                        sq += __shfl_xor_sync(kFullWarpMask, sq, off);
                    if (lane == 0)
                        rs.part[(f0 / 128) * rs.ld + tok0 + t] = sq;
                }
            }
        }
    }
};

// Interleaved gate/up columns (2j = gate_j, 2j + 1 = up_j) -> act[tok][j] =
// silu(g) * u = g / (1 + exp(-g)) * u, the expression of silu_mul_kernel
// (evaluated with the SFU exponential and a fast division: fast path only).
// With rs.part set the operand was h * gain (deferred norm): both columns are
// first scaled by the token's rsqrt(mean(h^2) + eps).
struct SiluMulTileEpi {
    static constexpr bool kTile = true;
    ActOut act;
    RowSumSq rs{};
    __device__ __forceinline__ void prepare(int tok0, int ntok, int, int, int tid, void *scratch) const {
        float *inv = static_cast<float *>(scratch);
        for (int t = tid; t < ntok; t += 128)
            inv[t] = rs.part ? rs.inv_rms(tok0 + t) : 1.f;
    }
    __device__ __forceinline__ void operator()(const float *tile, int tok0, int ntok, int f0, int nfeat, int tid,
                                               void *scratch) const {
        // warp w takes tokens w, w + 4, ...; lane l reads the 16-byte group
        // (g, u, g, u) of outputs 2l, 2l + 1 and writes them as one pair
        // four tokens per warp iteration (independent chains); SiLU by the
        // SFU exponential and a fast reciprocal (the fast path's outputs are
        // 16-bit pairs: their rounding dwarfs these few-ulp differences)
        const float *inv = static_cast<const float *>(scratch);
        const int warp = tid >> 5, lane = tid & 31;
        const bool vec = 4 * lane + 3 < nfeat;
        constexpr int kU = 2;
        for (int tb = warp; tb < ntok; tb += 4 * kU) {
            float a0[kU], a1[kU];
#pragma unroll
            for (int j = 0; j < kU; ++j) {
                const int t = tb + 4 * j;
                a0[j] = a1[j] = 0.f;
                if (t < ntok) {
                    const float sc = inv[t];
                    const float4 v = *reinterpret_cast<const float4 *>(tile + t * 128 + 4 * lane);
                    const float g0 = v.x * sc, u0 = v.y * sc, g1 = v.z * sc, u1 = v.w * sc;
                    a0[j] = __fdividef(g0, 1.f + __expf(-g0)) * u0;
                    a1[j] = __fdividef(g1, 1.f + __expf(-g1)) * u1;
                }
            }
#pragma unroll
            for (int j = 0; j < kU; ++j) {
                const int t = tb + 4 * j;
                if (t >= ntok)
                    break;
                if (vec) {
                    act.put2c(tok0 + t, f0 / 2 + 2 * lane, a0[j], a1[j]);
                } else if (4 * lane + 1 < nfeat) {
                    act.put(tok0 + t, f0 / 2 + 2 * lane, a0[j]);
                }
            }
        }
    }
};

// LM head logits out[tok][f] = value * rsqrt(mean(h^2) + eps) of the token
// (deferred final norm); ss_row0 maps tile tokens to RowSumSq rows.
struct LogitsTileEpi {
    static constexpr bool kTile = true;
    float *out;
    int64_t ld;
    RowSumSq rs;
    int64_t ss_row0 = 0;
    __device__ __forceinline__ void prepare(int tok0, int ntok, int, int, int tid, void *scratch) const {
        float *inv = static_cast<float *>(scratch);
        for (int t = tid; t < ntok; t += 128)
            inv[t] = rs.inv_rms(ss_row0 + tok0 + t);
    }
    __device__ __forceinline__ void operator()(const float *tile, int tok0, int ntok, int f0, int nfeat, int tid,
                                               void *scratch) const {
        const float *inv = static_cast<const float *>(scratch);
        for (int idx = tid; idx < ntok * 128; idx += 128) {
            const int t = idx >> 7, c = idx & 127;
            if (c < nfeat)
                out[static_cast<int64_t>(tok0 + t) * ld + f0 + c] = tile[idx] * inv[t];
        }
    }
};

// q | k | v columns of the fused QKV projection (two 64-wide heads per tile):
// RoPE on q and k heads (the pairs (i, i + 32) and the cos/sin table of
// qkv_finalize_kernel), q to q_out [rows][qh][64], k and v into the paged
// cache at the token's position.
struct QkvTileEpi {
    static constexpr bool kTile = true;
    float *q_out;
    int qh, kvh;
    const float2 *rope;
    TokenMap tm;
    PagedKV kv;
    float *kpool, *vpool;
    // per token of the slice: position, KV block and slot in it (loaded while
    // the GEMM main loop streams)
    RowSumSq rs{}; // deferred input norm when rs.part is set
    // scratch: meta [ntok][4] | cos/sin [ntok][32] (staged when preload is
    // set, the GEMM's scratch is kEpiScratchNarrow bytes and ntok fits)
    static constexpr int kPreTok = static_cast<int>(sm100::kEpiScratchNarrow / (16 + 8 * (kAttnD / 2)));
    bool preload = false;
    __device__ __forceinline__ void prepare(int tok0, int ntok, int, int, int tid, void *scratch) const {
        int *meta = static_cast<int *>(scratch); // [ntok][4]: pos, block, slot, rsqrt scale (float bits)
        for (int t = tid; t < ntok; t += 128) {
            const int64_t row = tok0 + t;
            const int pos = tm.pos[row];
            meta[4 * t] = pos;
            meta[4 * t + 1] = kv.table[static_cast<int64_t>(tm.seq[row]) * kv.table_stride + pos / kKvChunk];
            meta[4 * t + 2] = pos % kKvChunk;
            meta[4 * t + 3] = __float_as_int(rs.part ? rs.inv_rms(row) : 1.f);
        }
        if (preload && ntok <= kPreTok) {
            // read in operator() by other threads: the cluster barrier (or
            // the block barrier of an unsplit tile) orders these writes
            float2 *cs = reinterpret_cast<float2 *>(meta + 4 * kPreTok);
            for (int idx = tid; idx < ntok * 32; idx += 128)
                cs[idx] = rope[static_cast<int64_t>(tm.pos[tok0 + (idx >> 5)]) * (kAttnD / 2) + (idx & 31)];
        }
    }
    __device__ __forceinline__ void operator()(const float *tile, int tok0, int ntok, int f0, int nfeat, int tid,
                                               void *scratch) const {
        const int *meta = static_cast<const int *>(scratch);
        const bool staged = preload && ntok <= kPreTok;
        const float2 *cs = reinterpret_cast<const float2 *>(meta + 4 * kPreTok);
        // kChunk items per thread at a time: their cos/sin loads are issued
        // together (one memory latency per chunk)
        constexpr int kChunk = 4;
        const int items = ntok * 64;
        for (int base = 0; base < items; base += kChunk * 128) {
            float2 rv[kChunk];
#pragma unroll
            for (int j = 0; j < kChunk; ++j) {
                const int idx = base + j * 128 + tid;
                rv[j] = make_float2(1.f, 0.f);
                if (idx < items && f0 / kAttnD + ((idx >> 5) & 1) < qh + kvh)
                    rv[j] = staged ? cs[(idx >> 6) * 32 + (idx & 31)]
                                   : rope[static_cast<int64_t>(meta[4 * (idx >> 6)]) * (kAttnD / 2) + (idx & 31)];
            }
#pragma unroll
            for (int j = 0; j < kChunk; ++j) {
                const int idx = base + j * 128 + tid;
                if (idx >= items)
                    break;
                const int t = idx >> 6, hh = (idx >> 5) & 1, i = idx & 31;
                if (hh * 64 + 64 > nfeat)
                    continue;
                const int head = f0 / kAttnD + hh;
                const int64_t row = tok0 + t;
                const float sc = __int_as_float(meta[4 * t + 3]);
                const float a = tile[t * 128 + hh * 64 + i] * sc, b = tile[t * 128 + hh * 64 + i + 32] * sc;
                const float2 r = rv[j];
                if (head < qh) {
                    float *q = q_out + row * qh * kAttnD + head * kAttnD;
                    q[i] = a * r.x - b * r.y;
                    q[i + kAttnD / 2] = b * r.x + a * r.y;
                    continue;
                }
                const int blk = meta[4 * t + 1];
                const int slot = meta[4 * t + 2];
                if (head < qh + kvh) {
                    float *k = kpool + ((static_cast<int64_t>(blk) * kvh + (head - qh)) * kKvChunk + slot) * kAttnD;
                    k[i] = a * r.x - b * r.y;
                    k[i + kAttnD / 2] = b * r.x + a * r.y;
                } else {
                    float *v =
                        vpool + ((static_cast<int64_t>(blk) * kvh + (head - qh - kvh)) * kKvChunk + slot) * kAttnD;
                    v[i] = a;
                    v[i + kAttnD / 2] = b;
                }
            }
        }
    }
};

// Tensor-parallel residual step: y is the projection's output summed over the
// ranks (all-reduce). hidden[row] += y[row]; with `gain` set, normed[row] =
// hidden[row] * gain (the next projection's two-term 16-bit operand, deferred
// norm) and rs.part[tile][row] = the tile's sum of squares of hidden, as the
// fused residual epilogue writes them. One block of 128 threads per row: warp
// w takes the 128-feature tiles w, w + 4, ...; lane l owns features 4l..4l+3.
// cols must be a multiple of 128.
static __global__ void __launch_bounds__(128)
    tp_residual_kernel(float *__restrict__ hidden, const float *__restrict__ y, int cols,
                       const float *__restrict__ gain, ActOut normed, RowSumSq rs) {
    pdl_trigger();
    pdl_wait();
    const int64_t row = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int t = warp; t < cols / 128; t += 4) {
        const int c = t * 128 + 4 * lane;
        float4 *hp = reinterpret_cast<float4 *>(hidden + row * cols + c);
        const float4 v = *reinterpret_cast<const float4 *>(y + row * cols + c);
        float4 h = *hp;
        h.x += v.x;
        h.y += v.y;
        h.z += v.z;
        h.w += v.w;
        *hp = h;
        if (gain) {
            const float4 g = *reinterpret_cast<const float4 *>(gain + c);
            normed.put4c(row, c, make_float4(h.x * g.x, h.y * g.y, h.z * g.z, h.w * g.w));
        }
        if (rs.part) {
            float sq = (h.x * h.x + h.y * h.y) + (h.z * h.z + h.w * h.w);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
                sq += __shfl_xor_sync(kFullWarpMask, sq, off);
            if (lane == 0)
                rs.part[t * rs.ld + row] = sq;
        }
    }
}

// Tensor parallelism without a library collective: the o / down GEMM's tile
// epilogue stores its partial tile straight into slot `rank` of every rank's
// receive buffer (peer memory over NVLink, CUDA IPC mappings) and then adds
// the tile's token count to every rank's arrival counter (system-scope
// atomics after a system fence); tp_p2p_residual_kernel waits for the
// counter to reach rows x (H / 128) x world, sums the slots in rank order
// (the same order on every rank: identical results) and runs the residual
// step. Receive buffers and counters are double-buffered by `parity` (o: 0,
// down: 1), and the last block of the consumer re-arms the parity's counter.
constexpr int kTpMaxWorld = 8;
// The ranks' hosts drift apart by more than a kernel-local wait (first-launch
// module loads, graph captures), so the cross-rank wait allows 10 s by
// default before it reports error 6 and returns. After error 6 the receive
// counters are left as they are (partial tiles of slow ranks may still
// arrive), and the engine that launched the wait refuses further steps: its
// tensor-parallel exchange must be rebuilt (a new batch on every rank).
constexpr unsigned long long kTpPeerWaitNs = 10000000000ull;
constexpr int kErrTpPeerTimeout = 6;
struct TpPeers {
    float *recv[kTpMaxWorld];        // each rank's receive buffer [2][world][rows_max][H]
    unsigned int *cnt[kTpMaxWorld];  // each rank's counters [2]
    int world = 1, rank = 0;
    int64_t slot_floats = 0;         // rows_max * H
};

struct PeerStoreTileEpi {
    static constexpr bool kTile = true;
    TpPeers peers;
    int parity = 0;
    int64_t ld = 0; // H
    __device__ __forceinline__ void operator()(const float *tile, int tok0, int ntok, int f0, int nfeat, int tid,
                                               void *) const {
        const int warp = tid >> 5, lane = tid & 31, c = 4 * lane;
        const int64_t base = (static_cast<int64_t>(parity) * peers.world + peers.rank) * peers.slot_floats;
        for (int t = warp; t < ntok; t += 4) {
            const float4 v = *reinterpret_cast<const float4 *>(tile + t * 128 + c);
            const int64_t off = base + static_cast<int64_t>(tok0 + t) * ld + f0 + c;
            for (int r = 0; r < peers.world; ++r) {
                if (c + 3 < nfeat) {
                    *reinterpret_cast<float4 *>(peers.recv[r] + off) = v;
                } else {
                    const float vv[4] = {v.x, v.y, v.z, v.w};
                    for (int e = 0; e < 4; ++e)
                        if (c + e < nfeat)
                            peers.recv[r][off + e] = vv[e];
                }
            }
        }
        sm100::epilogue_bar(); // every epilogue thread's stores are issued
        if (tid == 0 && ntok > 0) {
            __threadfence_system();
            for (int r = 0; r < peers.world; ++r)
                atomicAdd_system(peers.cnt[r] + parity, static_cast<unsigned>(ntok));
        }
    }
};

// One block of 128 threads per row (see tp_residual_kernel); waits (bounded)
// for the partial tiles of all ranks, y = sum of the slots in rank order.
static __global__ void __launch_bounds__(128)
    tp_p2p_residual_kernel(float *__restrict__ hidden, const float *__restrict__ recv, unsigned int *cnt,
                           unsigned int *done, int parity, int world, int64_t slot_floats, int rows, int cols,
                           const float *__restrict__ gain, ActOut normed, RowSumSq rs, int *err,
                           unsigned long long wait_ns) {
    pdl_trigger();
    pdl_wait();
    __shared__ int ok;
    if (threadIdx.x == 0) {
        const unsigned target = static_cast<unsigned>(rows) * static_cast<unsigned>(cols / 128) * world;
        const uint64_t start = sm100::global_timer_ns();
        unsigned seen = 0;
        bool good = true;
        while (true) {
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(seen) : "l"(cnt + parity) : "memory");
            if (seen >= target)
                break;
            // a wait that already ran out (this launch or an earlier one of
            // the step) ends the others at once: one 10 s stall per step
            if (*static_cast<volatile int *>(err) == kErrTpPeerTimeout || sm100::global_timer_ns() - start > wait_ns) {
                good = false;
                break;
            }
        }
        ok = good;
        if (!good)
            atomicExch(err, kErrTpPeerTimeout);
    }
    __syncthreads();
    if (ok) {
        const int64_t row = blockIdx.x;
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        const float *slots = recv + static_cast<int64_t>(parity) * world * slot_floats + row * cols;
        for (int t = warp; t < cols / 128; t += 4) {
            const int c = t * 128 + 4 * lane;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int r = 0; r < world; ++r) {
                const float4 x = __ldcv(reinterpret_cast<const float4 *>(slots + r * slot_floats + c));
                v.x += x.x;
                v.y += x.y;
                v.z += x.z;
                v.w += x.w;
            }
            float4 *hp = reinterpret_cast<float4 *>(hidden + row * cols + c);
            float4 h = *hp;
            h.x += v.x;
            h.y += v.y;
            h.z += v.z;
            h.w += v.w;
            *hp = h;
            if (gain) {
                const float4 g = *reinterpret_cast<const float4 *>(gain + c);
                normed.put4c(row, c, make_float4(h.x * g.x, h.y * g.y, h.z * g.z, h.w * g.w));
            }
            if (rs.part) {
                float sq = (h.x * h.x + h.y * h.y) + (h.z * h.z + h.w * h.w);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1)
                    sq += __shfl_xor_sync(kFullWarpMask, sq, off);
                if (lane == 0)
                    rs.part[t * rs.ld + row] = sq;
            }
        }
    }
    // the last block of the launch re-arms this parity's counter (no rank
    // writes it again before this rank's next GEMM of the other parity ran);
    // a block whose wait ran out takes no part, so the counters stay as the
    // ranks left them
    __syncthreads();
    if (threadIdx.x == 0 && ok) {
        __threadfence();
        if (atomicAdd(done + parity, 1u) == gridDim.x - 1) {
            atomicExch(cnt + parity, 0u);
            atomicExch(done + parity, 0u);
        }
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

// fp32 weight -> 16-bit operand copy (fp16 when f16, else bf16; nearest even)
// with optional row interleave of two sources: dst row 2j = a[j], 2j + 1 =
// b[j] (b == nullptr: plain copy of a).
static __global__ void weights_to_16_kernel(const float *__restrict__ a, const float *__restrict__ b, int rows, int cols,
                                            uint16_t *__restrict__ dst, bool f16) {
    const int64_t total = static_cast<int64_t>(b ? 2 * rows : rows) * cols;
    OPWORKS_GRID_LOOP(i, total) {
        const int64_t r = i / cols, c = i % cols;
        const float *src = b ? ((r & 1) ? b : a) : a;
        const int64_t sr = b ? (r >> 1) : r;
        dst[i] = to16(src[sr * cols + c], f16);
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

// 16-bit weight rows interleave (bf16 packs): dst 2j = a[j], 2j+1 = b[j].
static __global__ void interleave16_kernel(const uint16_t *__restrict__ a, const uint16_t *__restrict__ b, int rows,
                                           int cols, uint16_t *__restrict__ dst) {
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

// Device-side step feedback of a multi-step decode, done by the thread that
// writes a row's token (ids == nullptr: plain sampling). Row i's token of
// step k = taken[i] goes to out[k][i] (-1 once the row has emitted `eos`,
// which ends its count) and becomes the row's next input; position, length
// and the sampling step advance; the next step's uniform comes from
// uniforms[k + 1][i] when given (uniforms holds one row more than the
// steps of a call).
struct SampleAdvance {
    int32_t *ids = nullptr, *pos = nullptr, *lens = nullptr, *step = nullptr; // the next step's inputs
    double *uniform = nullptr;                                                 // the next step's uniform
    const double *uniforms = nullptr;                                          // [steps + 1][n], or nullptr
    int32_t *done = nullptr, *count = nullptr, *taken = nullptr;               // per row
    int32_t *out = nullptr;                                                    // [steps][n]
    int n = 0, eos = -1;
};

// A row's advance state as read at kernel start (every CTA of the row reads
// it while the row is being sampled, so the one writer only stores).
struct SampleAdvanceIn {
    int taken, done, pos, lens, step;
    double next_uniform; // valid when has_uniform
    bool has_uniform;
};

__device__ __forceinline__ void sample_advance_load(const SampleAdvance &adv, int row, SampleAdvanceIn &in) {
    in.taken = adv.taken[row];
    in.done = adv.done[row];
    in.pos = adv.pos[row];
    in.lens = adv.lens[row];
    in.step = adv.step[row];
    in.has_uniform = adv.uniforms != nullptr;
    in.next_uniform = in.has_uniform ? adv.uniforms[static_cast<int64_t>(in.taken + 1) * adv.n + row] : 0.0;
}

// Every CTA of a row has read the row's sampling inputs (uniform, step)
// before the one writer gets here (after the row's last cluster barrier).
__device__ __forceinline__ void sample_emit(int *out, int row, int tok, const SampleAdvance &adv,
                                            const SampleAdvanceIn &in) {
    out[row] = tok;
    if (adv.ids == nullptr)
        return;
    const int k = in.taken;
    int32_t emitted = -1;
    if (!in.done) {
        emitted = tok;
        adv.count[row] = k + 1;
        if (tok == adv.eos)
            adv.done[row] = 1;
    }
    adv.out[static_cast<int64_t>(k) * adv.n + row] = emitted;
    adv.ids[row] = tok;
    adv.pos[row] = in.pos + 1;
    adv.lens[row] = in.lens + 1;
    adv.step[row] = in.step + 1;
    if (in.has_uniform)
        adv.uniform[row] = in.next_uniform;
    adv.taken[row] = k + 1;
}

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

constexpr int kSampleCluster = 8;      // CTAs per row (portable cluster size)
constexpr int kSampleThreads = 512;    // threads per CTA
constexpr int kSampleChunkMax = 16384; // logits per CTA held in shared memory
constexpr int kSampleBuckets = 256;    // buckets per select level
constexpr int kSampleCandMax = 2048;   // compacted boundary-band tokens per CTA
constexpr float kSampleDistScale = 8.f;           // level-0 buckets per nat of (max - logit) / T
constexpr float kSampleTailDist = 23.f * 8.f;     // beyond 23 nats a token's fixed-point mass is 0
constexpr float kSampleMassScale = 2147483648.f;  // 2^31: masses in fixed point
static_assert(kSampleChunkMax % (4 * kSampleThreads) == 0, "each thread's run of the slice is whole 4-token words");

// Scaled distance of logit v from the row max, (max - v) / T * 8, and its
// level-0 band (monotone in v: a larger logit never lands in a later band).
__device__ __forceinline__ float sample_dist(float v, float gmax, float dscale) { return (gmax - v) * dscale; }
constexpr int kSampleBandCap = 251; // last distance band; byte codes above it mark boundary-band tokens
constexpr uint8_t kBandKept = 252, kBandTie = 253, kBandDrop = 254;
__device__ __forceinline__ int sample_bucket(float t) {
    return t < static_cast<float>(kSampleBandCap) ? static_cast<int>(t) : kSampleBandCap;
}

// Token mass exp((v - max) / T) in fixed point: round(e * 2^31) with e the
// fp32 exp (so the top token weighs exactly 2^31), 0 beyond 23 nats (where it
// rounds to 0 anyway). A row's total stays below 2^17 * 2^31, and integer sums
// are exact and independent of summation order, so the kept set and the draw
// are deterministic.
__device__ __forceinline__ uint32_t sample_qmass(float v, float t, float gmax, float inv_t) {
    return t < kSampleTailDist ? __float2uint_rn(expf((v - gmax) * inv_t) * kSampleMassScale) : 0u;
}

// Shared-memory positions of slice element i in the 32-bit array (one pad
// word per 32) and in the byte array (one pad word per 128): a thread walking
// a contiguous run and a warp walking consecutive elements are both free of
// bank conflicts.
__device__ __forceinline__ int sample_pos(int i) { return i + (i >> 5); }
__device__ __forceinline__ int sample_bpos(int i) { return i + ((i >> 7) << 2); }

struct SampleShared {
    // this CTA's slice of the row: the logits, replaced by their fixed-point
    // masses once the row max is known
    union {
        float x[kSampleChunkMax + kSampleChunkMax / 32];
        uint32_t q[kSampleChunkMax + kSampleChunkMax / 32];
    };
    uint8_t band[kSampleChunkMax + kSampleChunkMax / 32]; // level-0 bucket of every token
    // histograms: per bucket the sums of mass bits [0,16) and [16,32) in
    // 32-bit counters (no overflow for 16384 tokens; two native 32-bit
    // shared-memory atomics per token measured 5x faster than one 64-bit
    // one); level 0, then levels 1-4 alternating between two buffers
    uint32_t h0[2][kSampleBuckets];
    uint32_t hk[2][2][kSampleBuckets];
    uint32_t cand_key[kSampleCandMax];                     // boundary-band tokens: float key,
    uint32_t cand_q[kSampleCandMax];                       //   mass
    uint16_t cand_pos[kSampleCandMax];                     //   and slice position
    unsigned long long uscr[kSampleThreads / 32];
    int iscr[kSampleThreads / 32];
    float best_v;
    int best_i;
    unsigned long long part_mass; // final pass: kept mass of this CTA
    int part_ties;                // final pass: boundary ties of this CTA
    SampleAdvanceIn adv_in;       // the row's multi-step state (thread 0 reads it)
    int res_bucket;               // crossing bucket of the current level
    unsigned long long res_above; // mass above it
};

// Block-wide exclusive prefix (threads in index order) of a u64 and an int.
__device__ __forceinline__ void block_scan_excl(unsigned long long v, int c, unsigned long long *uscr, int *iscr,
                                                unsigned long long &v_before, int &c_before,
                                                unsigned long long &v_total, int &c_total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
    unsigned long long vi = v;
    int ci = c;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const unsigned long long vo = __shfl_up_sync(kFullWarpMask, vi, off);
        const int co = __shfl_up_sync(kFullWarpMask, ci, off);
        if (lane >= off) {
            vi += vo;
            ci += co;
        }
    }
    __syncthreads();
    if (lane == 31) {
        uscr[warp] = vi;
        iscr[warp] = ci;
    }
    __syncthreads();
    unsigned long long wv = 0, tv = 0;
    int wc = 0, tc = 0;
    for (int w = 0; w < nw; ++w) {
        if (w < warp) {
            wv += uscr[w];
            wc += iscr[w];
        }
        tv += uscr[w];
        tc += iscr[w];
    }
    v_before = wv + vi - v;
    c_before = wc + ci - c;
    v_total = tv;
    c_total = tc;
}

// Histogram add of a 31-bit mass as two 16-bit halves in 32-bit counters
// (native shared-memory atomics); a warp whose lanes all hit one bucket
// (flat rows) adds once. Whole warps must call it.
__device__ __forceinline__ void sample_hist_add(uint32_t (*h)[kSampleBuckets], int bkt, uint32_t q, int lane) {
    const int b0 = __shfl_sync(kFullWarpMask, bkt, 0);
    if (__all_sync(kFullWarpMask, bkt == b0)) {
        const uint32_t lo = __reduce_add_sync(kFullWarpMask, q & 0xffffu);
        const uint32_t hi = __reduce_add_sync(kFullWarpMask, q >> 16);
        if (lane == 0 && b0 >= 0 && (lo | hi)) {
            atomicAdd(&h[0][b0], lo);
            atomicAdd(&h[1][b0], hi);
        }
    } else if (bkt >= 0 && q) {
        atomicAdd(&h[0][bkt], q & 0xffffu);
        atomicAdd(&h[1][bkt], q >> 16);
    }
}

// One 8-CTA cluster per row of logits [rows][ld]. Greedy (temperature <= 0):
// first index of the maximum. Otherwise the host sampler of OpWorks
// examples/llama/generate.py:83-109: p = softmax(logits / max(T, 1e-6));
// keep the descending-sorted prefix up to and including the first token whose
// cumulative mass reaches top_p (tokens tied at that boundary are kept in
// ascending index order); renormalise; return the first index whose
// cumulative kept mass (index order) exceeds u * total, numpy's
// Generator.choice rule.
//
// The boundary token is found by a 5-level select over 256-bucket
// histograms. Level 0 buckets every token by its distance from the max in
// 1/8 nat, floor((max - v) / T * 8) (capped at 255), and replaces the
// logits in shared memory by their masses and bands; the tokens of the
// crossing band are compacted into a short list (float key, mass) and levels
// 1-4 refine it by the float bits of the logit, 8 bits at a time. Each CTA keeps its slice of
// the row in shared memory and builds a histogram of its slice; after a
// cluster barrier every CTA sums the 8 histograms through distributed shared
// memory (256 x 8 loads) and finds the crossing bucket itself (identical
// integer arithmetic everywhere), so one barrier per level suffices.
static __global__ void __cluster_dims__(kSampleCluster, 1, 1) __launch_bounds__(kSampleThreads, 2)
    sample_kernel(const float *__restrict__ logits, int64_t ld, int vocab, SampleParams sp, int *__restrict__ out,
                  SampleAdvance adv) {
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
    const int n_pad = (n + kWarpSize - 1) / kWarpSize * kWarpSize;
    const float *src = logits + static_cast<int64_t>(row) * ld + lo;
    pdl_trigger();
    pdl_wait();
    if (adv.ids != nullptr && tid == 0)
        sample_advance_load(adv, row, sh.adv_in);

    // pass 0: stage the slice, local (max, first index)
    float bv = kNegInf;
    int bi = 0x7fffffff;
    auto take = [&](int i, float v) {
        sh.x[sample_pos(i)] = v;
        if (v > bv) {
            bv = v;
            bi = lo + i;
        }
    };
    int head = 0;
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        for (int i4 = tid; i4 < n / 4; i4 += blockDim.x) {
            const float4 f = __ldg(s4 + i4);
            take(4 * i4, f.x);
            take(4 * i4 + 1, f.y);
            take(4 * i4 + 2, f.z);
            take(4 * i4 + 3, f.w);
        }
        head = (n / 4) * 4;
    }
    for (int i = head + tid; i < n; i += blockDim.x)
        take(i, __ldg(src + i));
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
        sh.uscr[warp] = __float_as_uint(bv);
        sh.iscr[warp] = bi;
    }
    for (int b = tid; b < kSampleBuckets; b += blockDim.x)
        sh.h0[0][b] = sh.h0[1][b] = 0u;
    __syncthreads();
    if (tid == 0) {
        float v = kNegInf;
        int i0 = 0x7fffffff;
        for (int w = 0; w < kSampleThreads / 32; ++w) {
            const float ov = __uint_as_float(static_cast<uint32_t>(sh.uscr[w]));
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
#pragma unroll
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
        cluster.sync(); // peers finished reading this CTA's shared memory
        if (rank == 0 && tid == 0)
            sample_emit(out, row, garg, adv, sh.adv_in);
        return;
    }
    const float inv_t = 1.f / fmaxf(temp, 1e-6f);
    const float dscale = inv_t * kSampleDistScale;
    const double top_p = sp.top_p ? static_cast<double>(sp.top_p[row]) : 1.0;
    const double u = (sp.uniform && sp.uniform[row] >= 0.0)
                         ? sp.uniform[row]
                         : counter_uniform(sp.seed ? sp.seed[row] : 0ull, sp.step ? sp.step[row] : 0);

    const bool filtered = top_p < 1.0;
    // level 0: the mass and band of every token (masses replace the logits
    // in shared memory); the band histogram when filtering. Two tokens per
    // thread per iteration; whole warps iterate together.
    for (int i = tid; i < n_pad; i += 2 * kSampleThreads) {
        const int i2 = i + kSampleThreads;
        const float v0 = i < n ? sh.x[sample_pos(i)] : kNegInf;
        const float v1 = i2 < n ? sh.x[sample_pos(i2)] : kNegInf;
        const float t0 = sample_dist(v0, gmax, dscale), t1 = sample_dist(v1, gmax, dscale);
        const uint32_t q0 = i < n ? sample_qmass(v0, t0, gmax, inv_t) : 0u;
        const uint32_t q1 = i2 < n ? sample_qmass(v1, t1, gmax, inv_t) : 0u;
        const int b0 = sample_bucket(t0), b1 = sample_bucket(t1);
        if (i < n) {
            sh.q[sample_pos(i)] = q0;
            sh.band[sample_bpos(i)] = static_cast<uint8_t>(b0);
        }
        if (i2 < n) {
            sh.q[sample_pos(i2)] = q1;
            sh.band[sample_bpos(i2)] = static_cast<uint8_t>(b1);
        }
        if (filtered) {
            sample_hist_add(sh.h0, i < n ? b0 : -1, q0, lane);
            sample_hist_add(sh.h0, i2 < n ? b1 : -1, q1, lane);
        }
    }
    uint32_t key_star = 0;
    int bstar = kSampleBuckets;
    unsigned long long above = 0, z = 0;
    if (filtered) {
        uint32_t prefix = 0;
        bool listed = true; // band compacted (else levels 1-4 rescan the slice)
        int n_cand = 0;
        for (int level = 0; level < 5; ++level) {
            uint32_t(*hk)[kSampleBuckets] = sh.hk[level & 1];
            const int shift = level == 0 ? 0 : 32 - 8 * level;
            const uint32_t mask_hi = level <= 1 ? 0u : (0xffffffffu << (shift + 8));
            if (level > 0) {
                for (int b = tid; b < kSampleBuckets; b += blockDim.x)
                    hk[0][b] = hk[1][b] = 0u;
                __syncthreads();
                if (listed) {
                    const int nc_pad = (n_cand + kWarpSize - 1) / kWarpSize * kWarpSize;
                    for (int c = tid; c < nc_pad; c += kSampleThreads) {
                        int bkt = -1;
                        uint32_t q = 0;
                        if (c < n_cand) {
                            const uint32_t k = sh.cand_key[c];
                            if ((k & mask_hi) == prefix) {
                                bkt = static_cast<int>((k >> shift) & 0xffu);
                                q = sh.cand_q[c];
                            }
                        }
                        sample_hist_add(hk, bkt, q, lane);
                    }
                } else {
                    // band too large to list (flat rows): scan the slice,
                    // keys from global memory, 8 loads in flight per thread
                    for (int base = tid; base < n_pad; base += 8 * kSampleThreads) {
                        uint32_t key[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const int i = base + j * kSampleThreads;
                            key[j] = i < n && sh.band[sample_bpos(i)] == bstar ? float_key(__ldg(src + i)) : 0u;
                        }
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const int i = base + j * kSampleThreads;
                            int bkt = -1;
                            uint32_t q = 0;
                            if (i < n && sh.band[sample_bpos(i)] == bstar && (key[j] & mask_hi) == prefix) {
                                bkt = static_cast<int>((key[j] >> shift) & 0xffu);
                                q = sh.q[sample_pos(i)];
                            }
                            sample_hist_add(hk, bkt, q, lane);
                        }
                    }
                }
            }
            cluster.sync();
            // every CTA: the cluster's histogram (thread t < 256 sums bucket
            // t of the 8 slices), scanned from the heaviest bucket: distance 0
            // first, then the largest float bits first
            unsigned long long bm = 0;
            if (tid < kSampleBuckets) {
                const int b = level == 0 ? tid : kSampleBuckets - 1 - tid;
#pragma unroll
                for (int r = 0; r < kSampleCluster; ++r) {
                    const SampleShared *peer = cluster.map_shared_rank(&sh, r);
                    const uint32_t(*h)[kSampleBuckets] = level == 0 ? peer->h0 : peer->hk[level & 1];
                    bm += (static_cast<unsigned long long>(h[1][b]) << 16) + h[0][b];
                }
            }
            unsigned long long before, total;
            int ib, it;
            block_scan_excl(bm, 0, sh.uscr, sh.iscr, before, ib, total, it);
            if (level == 0)
                z = total;
            const double target = top_p * static_cast<double>(z);
            if (tid < kSampleBuckets) {
                const unsigned long long acc = above + before;
                const bool last = tid == kSampleBuckets - 1;
                if ((static_cast<double>(acc + bm) >= target || last) && static_cast<double>(acc) < target) {
                    sh.res_bucket = level == 0 ? tid : kSampleBuckets - 1 - tid;
                    sh.res_above = acc;
                }
            }
            __syncthreads();
            if (level == 0)
                bstar = sh.res_bucket;
            else
                prefix |= static_cast<uint32_t>(sh.res_bucket) << shift;
            above = sh.res_above;
            if (level == 0) {
                // compact the crossing band's positions in index order: each
                // thread tests its run of 32 tokens four band bytes per load,
                // a block scan of the counts gives its first slot; then the
                // keys are fetched, all loads in flight
                constexpr int kRun = kSampleChunkMax / kSampleThreads;
                const int r_lo = min(n, tid * kRun), r_hi = min(n, r_lo + kRun);
                const uint32_t pat = 0x01010101u * static_cast<uint32_t>(bstar);
                uint32_t hit[kRun / 4];
                int cnt = 0;
#pragma unroll
                for (int w = 0; w < kRun / 4; ++w) {
                    const int i = r_lo + 4 * w; // 4-aligned: one 32-bit word of band bytes
                    uint32_t m = 0;
                    if (i < r_hi) {
                        m = __vcmpeq4(*reinterpret_cast<const uint32_t *>(&sh.band[sample_bpos(i)]), pat) & 0x01010101u;
                        if (r_hi - i < 4)
                            m &= (1u << (8 * (r_hi - i))) - 1u;
                    }
                    hit[w] = m;
                    cnt += __popc(m);
                }
                unsigned long long ub, ut;
                int slot;
                block_scan_excl(0ull, cnt, sh.uscr, sh.iscr, ub, slot, ut, n_cand);
#pragma unroll
                for (int w = 0; w < kRun / 4; ++w)
                    for (uint32_t m = hit[w]; m; m &= m - 1u, ++slot)
                        if (slot < kSampleCandMax)
                            sh.cand_pos[slot] = static_cast<uint16_t>(r_lo + 4 * w + ((__ffs(m) - 1) >> 3));
                __syncthreads();
                listed = n_cand <= kSampleCandMax;
                if (listed)
                    for (int c = tid; c < n_cand; c += kSampleThreads) {
                        const int i = sh.cand_pos[c];
                        sh.cand_key[c] = float_key(__ldg(src + i));
                        sh.cand_q[c] = sh.q[sample_pos(i)];
                    }
            }
            __syncthreads(); // res_* is rewritten by the next level
        }
        key_star = prefix;
        // mark the boundary band's tokens kept / tied / dropped, so the
        // final pass reads only shared memory
        if (listed) {
            for (int c = tid; c < n_cand; c += kSampleThreads) {
                const uint32_t k = sh.cand_key[c];
                sh.band[sample_bpos(sh.cand_pos[c])] = k > key_star ? kBandKept : (k == key_star ? kBandTie : kBandDrop);
            }
        } else {
            for (int base = tid; base < n; base += 8 * kSampleThreads) {
                uint32_t key[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int i = base + j * kSampleThreads;
                    key[j] = i < n && sh.band[sample_bpos(i)] == bstar ? float_key(__ldg(src + i)) : 0u;
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int i = base + j * kSampleThreads;
                    if (i < n && sh.band[sample_bpos(i)] == bstar)
                        sh.band[sample_bpos(i)] =
                            key[j] > key_star ? kBandKept : (key[j] == key_star ? kBandTie : kBandDrop);
                }
            }
        }
        __syncthreads();
    }
    const float v_star = key_float(key_star);
    const unsigned long long q_star =
        filtered ? sample_qmass(v_star, sample_dist(v_star, gmax, dscale), gmax, inv_t) : 0ull;
    int n_keep_ties = 0x7fffffff;
    if (filtered && q_star > 0) {
        const double need =
            (top_p * static_cast<double>(z) - static_cast<double>(above)) / static_cast<double>(q_star);
        n_keep_ties = need <= 1.0 ? 1 : (need >= 2e9 ? 0x7fffffff : static_cast<int>(ceil(need - 1e-12)));
    }

    // final pass: kept mass in index order; each thread owns a contiguous
    // run. A token is kept when its logit's key is above key_star: bands
    // before the boundary band are kept whole, later ones dropped, and the
    // boundary band's tokens carry their mark. `tie` flags a boundary tie.
    auto kept_mass = [&](int i, bool &tie) -> uint32_t {
        const uint32_t q = sh.q[sample_pos(i)];
        if (!filtered) {
            tie = false;
            return q;
        }
        const int b = sh.band[sample_bpos(i)];
        tie = b == kBandTie;
        return (b < bstar || b == kBandKept) ? q : 0u;
    };
    const int per_t = (n + kSampleThreads - 1) / kSampleThreads;
    const int t_lo = min(n, tid * per_t), t_hi = min(n, t_lo + per_t);
    unsigned long long my = 0, my1 = 0;
    int my_ties = 0;
    {
        bool tie0, tie1;
        int i = t_lo;
        for (; i + 1 < t_hi; i += 2) {
            my += kept_mass(i, tie0);
            my1 += kept_mass(i + 1, tie1);
            my_ties += tie0 + tie1;
        }
        if (i < t_hi) {
            my += kept_mass(i, tie0);
            my_ties += tie0;
        }
        my += my1;
    }
    unsigned long long before, total;
    int ties_before, ties_total;
    block_scan_excl(my, my_ties, sh.uscr, sh.iscr, before, ties_before, total, ties_total);
    if (tid == 0) {
        sh.part_mass = total;
        sh.part_ties = ties_total;
    }
    cluster.sync();
    // cluster prefix over ranks (every CTA computes it from the peers)
    unsigned long long rank_before = 0, grand = 0;
    int ties_rank_before = 0, ties_grand = 0;
#pragma unroll
    for (int r = 0; r < kSampleCluster; ++r) {
        const SampleShared *peer = cluster.map_shared_rank(&sh, r);
        const unsigned long long pm = peer->part_mass;
        const int pt = peer->part_ties;
        if (r < rank) {
            rank_before += pm;
            ties_rank_before += pt;
        }
        grand += pm;
        ties_grand += pt;
    }
    const int keep_total = filtered ? min(n_keep_ties, ties_grand) : 0;
    const int tb = ties_rank_before + ties_before; // boundary ties before this thread
    const int mine = filtered ? max(0, min(my_ties, keep_total - tb)) : 0;
    const unsigned long long t_before =
        rank_before + before + q_star * static_cast<unsigned long long>(min(tb, keep_total));
    const unsigned long long t_mine = my + q_star * static_cast<unsigned long long>(mine);
    const unsigned long long all = grand + q_star * static_cast<unsigned long long>(keep_total);
    const double goal = u * static_cast<double>(all);
    if (static_cast<double>(t_before) <= goal && goal < static_cast<double>(t_before + t_mine)) {
        unsigned long long run = t_before;
        int ties_seen = tb;
        int pick = lo + t_hi - 1;
        for (int i = t_lo; i < t_hi; ++i) {
            bool tie;
            unsigned long long e = kept_mass(i, tie);
            if (tie && ties_seen++ < keep_total)
                e = q_star;
            if (e > 0) {
                run += e;
                if (static_cast<double>(run) > goal) {
                    pick = lo + i;
                    break;
                }
            }
        }
        sample_emit(out, row, pick, adv, sh.adv_in);
    }
    // u -> 1 rounding: the goal lands past the last kept token
    if (rank == kSampleCluster - 1 && tid == 0 && !(goal < static_cast<double>(all))) {
        const float *rowp = logits + static_cast<int64_t>(row) * ld;
        int last = vocab - 1;
        for (int i = vocab - 1; i >= 0; --i)
            if (!filtered || float_key(rowp[i]) >= key_star) {
                last = i;
                break;
            }
        sample_emit(out, row, last, adv, sh.adv_in);
    }
    cluster.sync(); // keep shared memory alive until every peer is done with it
}

inline size_t sample_smem_bytes() { return sizeof(SampleShared); }

inline void sample_launch(const float *logits, int64_t ld, int rows, int vocab, const SampleParams &sp, int *out,
                          cudaStream_t stream, const SampleAdvance &adv = {}) {
    require((vocab + kSampleCluster - 1) / kSampleCluster <= kSampleChunkMax, "vocabulary too large for the sampler");
    static thread_local int done = -1;
    int dev = 0;
    OPWORKS_CUDA_CHECK(cudaGetDevice(&dev));
    if (done != dev) {
        OPWORKS_CUDA_CHECK(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(sample_smem_bytes())));
        done = dev;
    }
    launch_ex(sample_kernel, dim3(rows * kSampleCluster), dim3(kSampleThreads), sample_smem_bytes(), stream, logits, ld,
              vocab, sp, out, adv);
}

} // namespace opworks::detail

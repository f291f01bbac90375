#pragma once

// GQA attention kernels over fp32 K/V, head_dim 64, shared by the OpWorks
// operator API (attention_decode / attention_prefill_chunked) and the Llama
// runtime's paged KV cache.
//
// K/V are addressed in 16-token chunks of 16 x 64 contiguous floats (4 KB):
// a chunk of the contiguous per-head cache [kvh][cap][64], or one block of
// the paged pool [blocks][kvh][16][64] looked up through a block table. Each
// 64-token tile is staged into shared memory with 1D bulk async copies (TMA
// engine, mbarrier completion), double/triple buffered.
//
// Decode (one query per sequence): split-KV. CTA = (KV split, kv head,
// sequence); all kRep query heads of the group share every K/V tile, so each
// K/V byte is read from HBM once. Partials (m, l, o) go to scratch and a
// combine kernel merges the splits.
//
// Prefill: CTA = (64/kRep query positions x kRep heads = 64 query rows, kv
// head). S = Q K^T and O += P V run as 4x4 register tiles per thread with
// online softmax; fully masked tiles beyond the causal diagonal are skipped.
// This fp32 SIMT kernel is the accurate path.

#include <type_traits>
#include <cuda_bf16.h>

#include "../core/block_reduce.cuh"
#include "../core/cuda_utils.cuh"
#include "detail/operand16.cuh"
#include "detail/sm100.cuh"

namespace opworks::detail {

constexpr int kAttnD = 64;      // head dim supported by these kernels

// Attention output writer into fp32 memory: out(t, head, d) = v for query
// token t (the operator API's layouts).
template <typename T> struct StridedOut {
    static_assert(std::is_same_v<T, float>, "attention outputs of the operator API are fp32");
    T *p;
    int64_t tok, head; // element strides
    __device__ __forceinline__ void put(int64_t t, int h, int d, float v) const { p[t * tok + h * head + d] = v; }
    __device__ __forceinline__ void put4(int64_t t, int h, int d0, float a, float b, float c, float e) const {
        *reinterpret_cast<float4 *>(p + t * tok + h * head + d0) = make_float4(a, b, c, e);
    }
};

// Row-major activation [tokens][cols] written as the next GEMM's operand:
// 16-bit words (fp16 when f16, else bf16; with h16_lo also the remainder
// term r(x - hi)), or fp32 (with lo: split into a tf32 hi part and x - hi).
struct ActOut {
    uint16_t *h16 = nullptr;    // hi term of a 16-bit operand
    uint16_t *h16_lo = nullptr; // optional remainder term
    bool f16 = false;           // format of the 16-bit terms
    float *f32 = nullptr;       // tf32 hi part when lo != nullptr
    float *lo = nullptr;        // x - tf32(x)
    int64_t ld = 0;             // row stride (elements)
    __device__ __forceinline__ static float tf32_rn(float x) {
        uint32_t u = __float_as_uint(x);
        if ((u & 0x7f800000u) == 0x7f800000u)
            return x;
        u += 0xfffu + ((u >> 13) & 1u);
        return __uint_as_float(u & 0xffffe000u);
    }
    __device__ __forceinline__ void put(int64_t row, int col, float v) const {
        const int64_t i = row * ld + col;
        if (h16) {
            const uint16_t h = to16(v, f16);
            h16[i] = h;
            if (h16_lo)
                h16_lo[i] = to16(v - from16(h, f16), f16);
        } else if (lo) {
            const float h = tf32_rn(v);
            f32[i] = h;
            lo[i] = v - h;
        } else {
            f32[i] = v;
        }
    }
    // two consecutive columns col, col + 1 (col and ld even)
    __device__ __forceinline__ void put2c(int64_t row, int col, float a, float b) const {
        const int64_t i = row * ld + col;
        if (h16) {
            const uint32_t h = pack16x2(a, b, f16);
            *reinterpret_cast<uint32_t *>(h16 + i) = h;
            if (h16_lo) {
                const float2 f = unpack16x2(h, f16);
                *reinterpret_cast<uint32_t *>(h16_lo + i) = pack16x2(a - f.x, b - f.y, f16);
            }
        } else {
            put(row, col, a);
            put(row, col + 1, b);
        }
    }
    // four consecutive columns col .. col + 3 (col and ld multiples of 4)
    __device__ __forceinline__ void put4c(int64_t row, int col, float4 v) const {
        const int64_t i = row * ld + col;
        if (h16) {
            const uint32_t h01 = pack16x2(v.x, v.y, f16), h23 = pack16x2(v.z, v.w, f16);
            *reinterpret_cast<uint2 *>(h16 + i) = make_uint2(h01, h23);
            if (h16_lo) {
                const float2 f01 = unpack16x2(h01, f16), f23 = unpack16x2(h23, f16);
                *reinterpret_cast<uint2 *>(h16_lo + i) =
                    make_uint2(pack16x2(v.x - f01.x, v.y - f01.y, f16), pack16x2(v.z - f23.x, v.w - f23.y, f16));
            }
        } else {
            put(row, col, v.x);
            put(row, col + 1, v.y);
            put(row, col + 2, v.z);
            put(row, col + 3, v.w);
        }
    }
    // attention-writer form (head-major columns)
    __device__ __forceinline__ void put(int64_t t, int h, int d, float v) const { put(t, h * 64 + d, v); }
    __device__ __forceinline__ void put4(int64_t t, int h, int d0, float a, float b, float c, float e) const {
        const int col = h * 64 + d0;
        if ((col & 3) == 0 && (ld & 3) == 0) {
            put4c(t, col, make_float4(a, b, c, e));
        } else {
            put(t, col, a);
            put(t, col + 1, b);
            put(t, col + 2, c);
            put(t, col + 3, e);
        }
    }
};
constexpr int kKvChunk = 16;    // tokens per chunk / paged block
constexpr int kAttnTile = 64;   // keys per staged tile (4 chunks)

// Contiguous per-head cache [kvh][cap][64] of one sequence.
struct ContigKV {
    const float *k;
    const float *v;
    int cap;
    __device__ __forceinline__ int64_t chunk_offset(int, int h, int chunk) const {
        return (static_cast<int64_t>(h) * cap + static_cast<int64_t>(chunk) * kKvChunk) * kAttnD;
    }
    __device__ __forceinline__ int chunk_tokens(int chunk) const {
        const int r = cap - chunk * kKvChunk;
        return r < kKvChunk ? r : kKvChunk;
    }
};

// Paged pool [blocks][kvh][16][64]; table[b * table_stride + i] is the
// physical block holding tokens [16 i, 16 i + 16) of sequence b.
struct PagedKV {
    const float *k;
    const float *v;
    const int *table;
    int table_stride;
    int kvh;
    __device__ __forceinline__ int64_t chunk_offset(int b, int h, int chunk) const {
        const int blk = table[static_cast<int64_t>(b) * table_stride + chunk];
        return ((static_cast<int64_t>(blk) * kvh + h) * kKvChunk) * kAttnD;
    }
    __device__ __forceinline__ int chunk_tokens(int) const { return kKvChunk; }
};

// Stage the K/V tile starting at token t0 (multiple of 64) into smem; only
// chunks holding tokens below t_end are copied. Thread 0 only.
template <class KV>
__device__ __forceinline__ void stage_kv_tile(const KV &kv, int b, int h, int t0, int t_end, float *ks, float *vs,
                                              uint64_t *bar) {
    uint32_t bytes = 0;
    int ntok[4];
    int64_t off[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const int chunk = t0 / kKvChunk + c;
        ntok[c] = 0;
        if (chunk * kKvChunk < t_end) {
            ntok[c] = kv.chunk_tokens(chunk);
            off[c] = kv.chunk_offset(b, h, chunk);
            bytes += 2u * static_cast<uint32_t>(ntok[c]) * kAttnD * 4u;
        }
    }
    sm100::mbar_arrive_expect_tx(bar, bytes);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        if (ntok[c] > 0) {
            const uint32_t n = static_cast<uint32_t>(ntok[c]) * kAttnD * 4u;
            sm100::bulk_load(ks + c * kKvChunk * kAttnD, kv.k + off[c], n, bar);
            sm100::bulk_load(vs + c * kKvChunk * kAttnD, kv.v + off[c], n, bar);
        }
    }
}

// ------------------------------------------------------------------ decode

constexpr float kLog2e = 1.4426950408889634f; // log2(e): exp(x) = 2^(x log2 e)

// 2^x by the SFU's ex2.approx (relative error ~2^-22; 2^-inf = 0).
__device__ __forceinline__ float exp2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Decode: one producer warp streams 32-token K/V tiles (2 chunks) through a
// kDecodeStages-deep ring of bulk copies; 8 consumer warps take 4 tokens of
// every tile each. A token's 64 dims are spread over kDG lanes (8, or 16 for
// 8 query heads per KV head) and every lane keeps the query heads' dims and
// its own online-softmax state (m, l, o) for all kRep heads of the KV head in
// registers. So every staged K/V element is read from shared memory exactly
// once, the softmax needs no per-tile cross-lane reduction beyond the QK dot
// product, and a warp releases a stage with one mbarrier arrive. Lane states
// are merged once, at the end of the split.
#ifndef OPWORKS_DECODE_STAGES
#define OPWORKS_DECODE_STAGES 6
#endif
constexpr int kDecodeStages = OPWORKS_DECODE_STAGES;
constexpr int kDecodeTile = 32;
constexpr int kDecodeWarps = 8;
constexpr int kDecodeThreads = (kDecodeWarps + 1) * 32;
constexpr int kDecodeCtasPerSm = kDecodeStages <= 4 ? 3 : 2; // shared-memory bound residency

template <int kRep> struct DecodeGeo {
    static constexpr int kDG = kRep == 8 ? 16 : 8;          // lanes per token
    static constexpr int kTL = 32 / kDG;                    // tokens a warp holds at once
    static constexpr int kVec = kAttnD / (4 * kDG);         // float4 per lane per K/V row
    static constexpr int kDims = 4 * kVec;                  // dims per lane
    static constexpr int kTPW = kDecodeTile / kDecodeWarps; // tokens per warp per tile
    static constexpr int kSteps = kTPW / kTL;
    static constexpr int kTileFloats = kDecodeTile * kAttnD;
    static constexpr int kPipeFloats = 2 * kDecodeStages * kTileFloats;
    static constexpr int kRedFloats = kDecodeWarps * kRep * (kAttnD + 2);
    static constexpr size_t kBytes =
        sizeof(float) * (kPipeFloats > kRedFloats ? kPipeFloats : kRedFloats) + 8 * kDecodeStages * 2 + 64;
    static_assert(kTL * kDG == 32 && kSteps * kTL == kTPW && kVec >= 1, "decode geometry");
};

// Issue the bulk copies of one tile (chunks of `kDecodeTile / kKvChunk`),
// given the per-chunk source offsets and token counts (0 = past t_end).
template <class KV>
__device__ __forceinline__ void stage_kv_tile_offsets(const KV &kv, const int64_t *off, const int *ntok, float *ks,
                                                      float *vs, uint64_t *bar) {
    constexpr int kChunks = kDecodeTile / kKvChunk;
    uint32_t bytes = 0;
#pragma unroll
    for (int c = 0; c < kChunks; ++c)
        bytes += 2u * static_cast<uint32_t>(ntok[c]) * kAttnD * 4u;
    sm100::mbar_arrive_expect_tx(bar, bytes);
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
        if (ntok[c] > 0) {
            const uint32_t n = static_cast<uint32_t>(ntok[c]) * kAttnD * 4u;
            sm100::bulk_load(ks + c * kKvChunk * kAttnD, kv.k + off[c], n, bar);
            sm100::bulk_load(vs + c * kKvChunk * kAttnD, kv.v + off[c], n, bar);
        }
    }
}

// q: [B][q_stride] with heads at h*64; sequence b holds lens[b] tokens (or
// len_all when lens is null). grid = (splits, kvh, B). With one
// split the normalised result goes straight to `out`; otherwise part_o
// [B][qh][splits][64] and part_ml [B][qh][splits][2] (running max in log2 units, running
// sum) hold the split partials for attn_decode_combine_kernel.
template <class KV, int kRep, typename Out>
__global__ void __launch_bounds__(kDecodeThreads, kDecodeCtasPerSm)
    attn_decode_partial_kernel(const float *__restrict__ q, int64_t q_stride, KV kv, const int *__restrict__ lens,
                               int len_all, int tokens_per_split, float scale, float *__restrict__ part_o,
                               float *__restrict__ part_ml, Out out, int *err) {
    using G = DecodeGeo<kRep>;
    constexpr int kChunks = kDecodeTile / kKvChunk;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    float *ks = reinterpret_cast<float *>(smem_raw);
    float *vs = ks + kDecodeStages * G::kTileFloats;
    float *red = ks;                                // [warps][kRep][64], reuses the ring after the loop
    float *mls = red + kDecodeWarps * kRep * kAttnD; // [warps][kRep][2]
    const int pipe_floats = G::kPipeFloats > G::kRedFloats ? G::kPipeFloats : G::kRedFloats;
    uint64_t *full = reinterpret_cast<uint64_t *>(ks + pipe_floats);
    uint64_t *empty = full + kDecodeStages;

    const int b = blockIdx.z, h = blockIdx.y, split = blockIdx.x, splits = gridDim.x;
    const int qh_total = gridDim.y * kRep;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_trigger();
    // lens and the block table are step inputs (copied before the step's
    // first kernel); q and the newest token's K/V come from the kernel
    // before this one, so only the producer's first tiles of OLDER tokens
    // may be fetched before the programmatic-launch wait
    const int len = lens != nullptr ? lens[b] : len_all;
    const int t_begin = split * tokens_per_split;
    const int t_end = min(len, t_begin + tokens_per_split);
    const int n_tiles = t_end > t_begin ? (t_end - t_begin + kDecodeTile - 1) / kDecodeTile : 0;

    if (tid == 0) {
        for (int s = 0; s < kDecodeStages; ++s) {
            sm100::mbar_init(&full[s], 1);
            sm100::mbar_init(&empty[s], kDecodeWarps);
        }
        sm100::fence_mbarrier_init();
    }
    __syncthreads();

    bool ok = true;
    const int tl = lane / G::kDG, dq = lane % G::kDG;
    float m_run[kRep], l_run[kRep], acc[kRep][G::kDims];
    if (warp == kDecodeWarps) {
        // producer warp: the lanes look up 32 chunks' block offsets at a time,
        // lane 0 issues the copies
        int issued = 0;
        bool waited = false;
        const int chunk0 = t_begin / kKvChunk;
        for (int base = 0; base < n_tiles && ok; base += 32 / kChunks) {
            const int my_chunk = chunk0 + base * kChunks + lane;
            int64_t my_off = 0;
            int my_tok = 0;
            if (my_chunk * kKvChunk < t_end) {
                my_off = kv.chunk_offset(b, h, my_chunk);
                my_tok = kv.chunk_tokens(my_chunk);
            }
            const int stop = min(n_tiles, base + 32 / kChunks);
            for (int tile = base; tile < stop; ++tile) {
                int64_t off[kChunks];
                int ntok[kChunks];
#pragma unroll
                for (int c = 0; c < kChunks; ++c) {
                    off[c] = __shfl_sync(kFullWarpMask, my_off, (tile - base) * kChunks + c);
                    ntok[c] = __shfl_sync(kFullWarpMask, my_tok, (tile - base) * kChunks + c);
                }
                const int s = tile % kDecodeStages;
                // a tile that reaches the step's new token (position len - 1,
                // written by the previous kernel) or needs a recycled stage
                // waits for the previous kernel (warp-uniform condition)
                if (!waited && (tile >= kDecodeStages || t_begin + (tile + 1) * kDecodeTile >= len)) {
                    pdl_wait();
                    waited = true;
                }
                bool go = true;
                if (lane == 0) {
                    if (tile >= kDecodeStages)
                        go = sm100::mbar_wait(&empty[s], static_cast<uint32_t>((tile / kDecodeStages) - 1) & 1u);
                    if (go)
                        stage_kv_tile_offsets(kv, off, ntok, ks + s * G::kTileFloats, vs + s * G::kTileFloats,
                                              &full[s]);
                }
                go = __shfl_sync(kFullWarpMask, go, 0);
                if (!go) {
                    ok = false;
                    break;
                }
                ++issued;
            }
        }
        // every issued copy must land before the CTA may exit or reuse the ring
        if (lane == 0)
            for (int j = (issued > kDecodeStages ? issued - kDecodeStages : 0); j < issued; ++j)
                if (!sm100::mbar_wait(&full[j % kDecodeStages], static_cast<uint32_t>(j / kDecodeStages) & 1u))
                    ok = false;
    } else {
        pdl_wait(); // q is the previous kernel's output
        // this lane's slice of the query heads, in registers, pre-scaled so
        // that scores come out in log2 units (softmax by exp2)
        const float qscale = scale * kLog2e;
        float qr[kRep][G::kDims];
        const float *qb = q + static_cast<int64_t>(b) * q_stride + static_cast<int64_t>(h) * kRep * kAttnD;
#pragma unroll
        for (int j = 0; j < kRep; ++j) {
            m_run[j] = kNegInf;
            l_run[j] = 0.f;
#pragma unroll
            for (int c = 0; c < G::kVec; ++c)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    qr[j][4 * c + e] = qb[j * kAttnD + c * 4 * G::kDG + dq * 4 + e] * qscale;
                    acc[j][4 * c + e] = 0.f;
                }
        }
        for (int tile = 0; tile < n_tiles; ++tile) {
            const int s = tile % kDecodeStages;
            if (!sm100::mbar_wait(&full[s], static_cast<uint32_t>(tile / kDecodeStages) & 1u)) {
                ok = false;
                break;
            }
            const float4 *K = reinterpret_cast<const float4 *>(ks + s * G::kTileFloats);
            const float4 *V = reinterpret_cast<const float4 *>(vs + s * G::kTileFloats);
            const int t0 = t_begin + tile * kDecodeTile;
#pragma unroll
            for (int st = 0; st < G::kSteps; ++st) {
                const int tok = warp * G::kTPW + st * G::kTL + tl;
                const bool valid = t0 + tok < t_end;
                float4 kk[G::kVec], vv[G::kVec];
#pragma unroll
                for (int c = 0; c < G::kVec; ++c) {
                    kk[c] = K[tok * (kAttnD / 4) + c * G::kDG + dq];
                    vv[c] = V[tok * (kAttnD / 4) + c * G::kDG + dq];
                }
                float d[kRep];
#pragma unroll
                for (int j = 0; j < kRep; ++j) {
                    float x = 0.f;
#pragma unroll
                    for (int c = 0; c < G::kVec; ++c) {
                        x = fmaf(qr[j][4 * c + 0], kk[c].x, x);
                        x = fmaf(qr[j][4 * c + 1], kk[c].y, x);
                        x = fmaf(qr[j][4 * c + 2], kk[c].z, x);
                        x = fmaf(qr[j][4 * c + 3], kk[c].w, x);
                    }
                    d[j] = x;
                }
#pragma unroll
                for (int j = 0; j < kRep; ++j)
#pragma unroll
                    for (int off = 1; off < G::kDG; off <<= 1)
                        d[j] += __shfl_xor_sync(kFullWarpMask, d[j], off);
                if (valid) {
#pragma unroll
                    for (int j = 0; j < kRep; ++j) {
                        float p;
                        if (d[j] > m_run[j]) {
                            const float a = exp2_approx(m_run[j] - d[j]);
                            m_run[j] = d[j];
                            l_run[j] *= a;
#pragma unroll
                            for (int e = 0; e < G::kDims; ++e)
                                acc[j][e] *= a;
                            p = 1.f;
                        } else {
                            p = exp2_approx(d[j] - m_run[j]);
                        }
                        l_run[j] += p;
#pragma unroll
                        for (int c = 0; c < G::kVec; ++c) {
                            acc[j][4 * c + 0] = fmaf(p, vv[c].x, acc[j][4 * c + 0]);
                            acc[j][4 * c + 1] = fmaf(p, vv[c].y, acc[j][4 * c + 1]);
                            acc[j][4 * c + 2] = fmaf(p, vv[c].z, acc[j][4 * c + 2]);
                            acc[j][4 * c + 3] = fmaf(p, vv[c].w, acc[j][4 * c + 3]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0)
                sm100::mbar_arrive(&empty[s]);
        }
        // merge the token lanes of the warp (lanes with the same dq)
#pragma unroll
        for (int j = 0; j < kRep; ++j) {
            float M = m_run[j];
#pragma unroll
            for (int off = G::kDG; off < 32; off <<= 1)
                M = fmaxf(M, __shfl_xor_sync(kFullWarpMask, M, off));
            const float a = m_run[j] == kNegInf ? 0.f : exp2_approx(m_run[j] - M);
            float L = l_run[j] * a;
#pragma unroll
            for (int off = G::kDG; off < 32; off <<= 1)
                L += __shfl_xor_sync(kFullWarpMask, L, off);
#pragma unroll
            for (int e = 0; e < G::kDims; ++e) {
                float o = acc[j][e] * a;
#pragma unroll
                for (int off = G::kDG; off < 32; off <<= 1)
                    o += __shfl_xor_sync(kFullWarpMask, o, off);
                acc[j][e] = o;
            }
            m_run[j] = M;
            l_run[j] = L;
        }
    }
    ok = __syncthreads_and(ok);
    if (!ok) {
        if (tid == 0)
            atomicExch(err, 2);
        return;
    }
    // the ring is idle: every warp publishes its (m, l, o) there
    if (warp < kDecodeWarps && tl == 0) {
#pragma unroll
        for (int j = 0; j < kRep; ++j) {
            float *o = red + (warp * kRep + j) * kAttnD;
#pragma unroll
            for (int c = 0; c < G::kVec; ++c)
                *reinterpret_cast<float4 *>(o + c * 4 * G::kDG + dq * 4) =
                    make_float4(acc[j][4 * c], acc[j][4 * c + 1], acc[j][4 * c + 2], acc[j][4 * c + 3]);
            if (dq == 0) {
                mls[(warp * kRep + j) * 2] = m_run[j];
                mls[(warp * kRep + j) * 2 + 1] = l_run[j];
            }
        }
    }
    __syncthreads();
    for (int i = tid; i < kRep * kAttnD; i += blockDim.x) {
        const int head = i / kAttnD, dd = i % kAttnD;
        float M = kNegInf;
        for (int g = 0; g < kDecodeWarps; ++g)
            M = fmaxf(M, mls[(g * kRep + head) * 2]);
        float L = 0.f, O = 0.f;
        if (M != kNegInf) {
            for (int g = 0; g < kDecodeWarps; ++g) {
                const float mg = mls[(g * kRep + head) * 2];
                if (mg == kNegInf)
                    continue;
                const float w = exp2_approx(mg - M);
                L += w * mls[(g * kRep + head) * 2 + 1];
                O += w * red[(g * kRep + head) * kAttnD + dd];
            }
        }
        if (splits == 1) {
            out.put(b, h * kRep + head, dd, L > 0.f ? O / L : 0.f);
        } else {
            const int64_t row = (static_cast<int64_t>(b) * qh_total + h * kRep + head) * splits + split;
            part_o[row * kAttnD + dd] = O;
            if (dd == 0) {
                part_ml[2 * row] = M;
                part_ml[2 * row + 1] = L;
            }
        }
    }
}

// Merge the split partials of every (sequence, q head): block = 64 threads
// (one per dim), grid = (qh, B); out(b, hq, d).
template <typename Out>
__global__ void __launch_bounds__(64)
    attn_decode_combine_kernel(const float *__restrict__ part_o, const float *__restrict__ part_ml, int splits,
                               Out out) {
    const int hq = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    pdl_trigger();
    pdl_wait();
    const int64_t base = (static_cast<int64_t>(b) * gridDim.x + hq) * splits;
    float M = kNegInf;
    for (int s = 0; s < splits; ++s)
        M = fmaxf(M, part_ml[2 * (base + s)]);
    float L = 0.f, o = 0.f;
    if (M != kNegInf) {
        for (int s = 0; s < splits; ++s) {
            const float m = part_ml[2 * (base + s)];
            if (m == kNegInf)
                continue;
            const float w = exp2_approx(m - M);
            L += w * part_ml[2 * (base + s) + 1];
            o += w * part_o[(base + s) * kAttnD + d];
        }
    }
    out.put(b, hq, d, L > 0.f ? o / L : 0.f);
}

// ----------------------------------------------------------------- prefill

constexpr int kPrefillStages = 2;
constexpr int kPad = 68; // padded row (floats) of the transposed smem tiles

struct PrefillSmem {
    static constexpr int kTileFloats = kAttnTile * kAttnD;
    static constexpr size_t kBytes = sizeof(float) * (2 * kPrefillStages * kTileFloats // K, V stages
                                                      + 3 * kAttnD * kPad)           // Qt, Kt, P
                                     + 8 * kPrefillStages + 64;
};

// q[t * q_tok + head * q_head + d], out[t * o_tok + head * o_head + d] for
// query t in [0, T) at absolute position q_offset + t; keys [0, q_offset + T)
// of sequence `b` in `kv`. grid = (ceil(T / (64 / kRep)), kvh).
template <class KV, int kRep, typename Out>
__global__ void __launch_bounds__(256)
    attn_prefill_kernel(const float *__restrict__ q, int64_t q_tok, int64_t q_head, Out out, KV kv, int b, int T,
                        int q_offset, float scale, int *err) {
    constexpr int kPos = kAttnTile / kRep; // query positions per CTA
    using SM = PrefillSmem;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    float *ks = reinterpret_cast<float *>(smem_raw);
    float *vs = ks + kPrefillStages * SM::kTileFloats;
    float *qt = vs + kPrefillStages * SM::kTileFloats; // [64 d][kPad]
    float *kt = qt + kAttnD * kPad;                    // [64 d][kPad]
    float *pm = kt + kAttnD * kPad;                    // [64 rows][kPad]
    uint64_t *full = reinterpret_cast<uint64_t *>(pm + kAttnD * kPad);
    pdl_trigger();
    pdl_wait();

    const int h = blockIdx.y;
    const int tid = threadIdx.x;
    const int p0 = blockIdx.x * kPos; // first query (relative) of this CTA
    const int S = q_offset + T;       // keys visible to the last query

    // Q^T tile: row r = hd * kPos + pi
    for (int i = tid; i < kAttnTile * kAttnD; i += blockDim.x) {
        const int r = i / kAttnD, d = i % kAttnD;
        const int hd = r / kPos, pi = r % kPos;
        const int t = p0 + pi;
        qt[d * kPad + r] = t < T ? q[static_cast<int64_t>(t) * q_tok + static_cast<int64_t>(h * kRep + hd) * q_head + d]
                                 : 0.f;
    }
    if (tid == 0) {
        for (int s = 0; s < kPrefillStages; ++s)
            sm100::mbar_init(&full[s], 1);
        sm100::fence_mbarrier_init();
    }
    __syncthreads();

    const int q_last = q_offset + min(T, p0 + kPos) - 1; // furthest query position in the CTA
    const int n_tiles = min(S, q_last + 1) > 0 ? (min(S, q_last + 1) + kAttnTile - 1) / kAttnTile : 0;
    int issued = 0;
    if (tid == 0)
        for (; issued < kPrefillStages && issued < n_tiles; ++issued)
            stage_kv_tile(kv, b, h, issued * kAttnTile, S, ks + issued * SM::kTileFloats,
                          vs + issued * SM::kTileFloats, &full[issued]);

    const int rg = tid / 16, cg = tid % 16;
    const int r0 = rg * 4, c0 = cg * 4;
    int qpos[4];
    bool rvalid[4];
#pragma unroll
    for (int jr = 0; jr < 4; ++jr) {
        const int pi = (r0 + jr) % kPos;
        rvalid[jr] = p0 + pi < T;
        qpos[jr] = q_offset + p0 + pi;
    }
    float m_run[4], l_run[4], o[4][4];
#pragma unroll
    for (int jr = 0; jr < 4; ++jr) {
        m_run[jr] = kNegInf;
        l_run[jr] = 0.f;
#pragma unroll
        for (int jd = 0; jd < 4; ++jd)
            o[jr][jd] = 0.f;
    }

    bool ok = true;
    int consumed = 0;
    for (int tile = 0; tile < n_tiles; ++tile) {
        const int s = tile % kPrefillStages;
        const bool landed = sm100::mbar_wait(&full[s], static_cast<uint32_t>(tile / kPrefillStages) & 1u);
        if (!__syncthreads_and(landed)) {
            ok = false;
            break;
        }
        consumed = tile + 1;
        const int k0 = tile * kAttnTile;
        const float *K = ks + s * SM::kTileFloats;
        const float *V = vs + s * SM::kTileFloats;
        const int kvalid = min(kAttnTile, S - k0);
        // K^T into padded smem (rows beyond kvalid are never used unmasked)
        for (int i = tid; i < kAttnTile * (kAttnD / 4); i += blockDim.x) {
            const int c = i % kAttnTile, d4 = (i / kAttnTile) * 4;
            const float4 v4 = c < kvalid ? *reinterpret_cast<const float4 *>(K + c * kAttnD + d4)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
            kt[(d4 + 0) * kPad + c] = v4.x;
            kt[(d4 + 1) * kPad + c] = v4.y;
            kt[(d4 + 2) * kPad + c] = v4.z;
            kt[(d4 + 3) * kPad + c] = v4.w;
        }
        __syncthreads();
        float sv[4][4];
#pragma unroll
        for (int jr = 0; jr < 4; ++jr)
#pragma unroll
            for (int jc = 0; jc < 4; ++jc)
                sv[jr][jc] = 0.f;
#pragma unroll 8
        for (int d = 0; d < kAttnD; ++d) {
            const float4 a = *reinterpret_cast<const float4 *>(qt + d * kPad + r0);
            const float4 kk = *reinterpret_cast<const float4 *>(kt + d * kPad + c0);
            const float av[4] = {a.x, a.y, a.z, a.w};
            const float kv4[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
            for (int jr = 0; jr < 4; ++jr)
#pragma unroll
                for (int jc = 0; jc < 4; ++jc)
                    sv[jr][jc] += av[jr] * kv4[jc];
        }
        float alpha[4];
#pragma unroll
        for (int jr = 0; jr < 4; ++jr) {
            float mx = kNegInf;
#pragma unroll
            for (int jc = 0; jc < 4; ++jc) {
                const int kp = k0 + c0 + jc;
                const bool vis = rvalid[jr] && kp < S && kp <= qpos[jr];
                sv[jr][jc] = vis ? sv[jr][jc] * scale : kNegInf;
                mx = fmaxf(mx, sv[jr][jc]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1)
                mx = fmaxf(mx, __shfl_xor_sync(kFullWarpMask, mx, off));
            const float m_new = fmaxf(m_run[jr], mx);
            alpha[jr] = (m_run[jr] == kNegInf) ? 0.f : expf(m_run[jr] - m_new);
            float psum = 0.f;
#pragma unroll
            for (int jc = 0; jc < 4; ++jc) {
                const float p = sv[jr][jc] == kNegInf ? 0.f : expf(sv[jr][jc] - m_new);
                sv[jr][jc] = p;
                psum += p;
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1)
                psum += __shfl_xor_sync(kFullWarpMask, psum, off);
            l_run[jr] = l_run[jr] * alpha[jr] + psum;
            m_run[jr] = m_new;
            *reinterpret_cast<float4 *>(pm + (r0 + jr) * kPad + c0) = make_float4(sv[jr][0], sv[jr][1], sv[jr][2],
                                                                                  sv[jr][3]);
        }
        __syncthreads();
#pragma unroll
        for (int jr = 0; jr < 4; ++jr)
#pragma unroll
            for (int jd = 0; jd < 4; ++jd)
                o[jr][jd] *= alpha[jr];
        const int cmax = kvalid;
#pragma unroll 4
        for (int c = 0; c < cmax; ++c) {
            const float4 v4 = *reinterpret_cast<const float4 *>(V + c * kAttnD + c0);
#pragma unroll
            for (int jr = 0; jr < 4; ++jr) {
                const float p = pm[(r0 + jr) * kPad + c];
                o[jr][0] += p * v4.x;
                o[jr][1] += p * v4.y;
                o[jr][2] += p * v4.z;
                o[jr][3] += p * v4.w;
            }
        }
        __syncthreads(); // stage, K^T and P are free again
        if (tid == 0 && issued < n_tiles) {
            const int ns = issued % kPrefillStages;
            stage_kv_tile(kv, b, h, issued * kAttnTile, S, ks + ns * SM::kTileFloats, vs + ns * SM::kTileFloats,
                          &full[ns]);
            ++issued;
        }
    }
    if (!ok) {
        if (tid == 0) {
            for (int j = consumed; j < issued; ++j)
                sm100::mbar_wait(&full[j % kPrefillStages], static_cast<uint32_t>(j / kPrefillStages) & 1u);
            atomicExch(err, 3);
        }
        return;
    }
#pragma unroll
    for (int jr = 0; jr < 4; ++jr) {
        if (!rvalid[jr])
            continue;
        const int r = r0 + jr;
        const int hd = r / kPos, pi = r % kPos;
        const float inv = l_run[jr] > 0.f ? 1.f / l_run[jr] : 0.f;
        out.put4(p0 + pi, h * kRep + hd, c0, o[jr][0] * inv, o[jr][1] * inv, o[jr][2] * inv, o[jr][3] * inv);
    }
}

// ----------------------------------------------------------- host helpers

template <class KV, int kRep, typename Out> inline void prepare_decode_kernel() {
    static thread_local int done = -1;
    int dev = 0;
    OPWORKS_CUDA_CHECK(cudaGetDevice(&dev));
    if (done != dev) {
        OPWORKS_CUDA_CHECK(cudaFuncSetAttribute(attn_decode_partial_kernel<KV, kRep, Out>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(DecodeGeo<kRep>::kBytes)));
        done = dev;
    }
}

template <class KV, int kRep, typename Out> inline void prepare_prefill_kernel() {
    static thread_local int done = -1;
    int dev = 0;
    OPWORKS_CUDA_CHECK(cudaGetDevice(&dev));
    if (done != dev) {
        OPWORKS_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_kernel<KV, kRep, Out>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(PrefillSmem::kBytes)));
        done = dev;
    }
}

// Split-KV geometry for `pairs` (sequence, kv head) pairs whose longest
// visible length is max_len: as many splits as keep every CTA resident in one
// wave (kDecodeCtasPerSm per SM), so the KV stream is one pass over HBM with
// no tail wave; tokens per split is a multiple of the tile.
inline int decode_tokens_per_split(int pairs, int max_len, int sm_count) {
    const int tiles = (max_len + kDecodeTile - 1) / kDecodeTile;
    const int slots = kDecodeCtasPerSm * sm_count;
    int splits = slots / (pairs > 0 ? pairs : 1);
    if (splits > tiles)
        splits = tiles;
    if (splits < 1)
        splits = 1;
    const int tiles_per_split = (tiles + splits - 1) / splits;
    return (tiles_per_split > 0 ? tiles_per_split : 1) * kDecodeTile;
}

template <class KV, int kRep, typename Out>
inline void attn_decode_launch(const float *q, int64_t q_stride, const KV &kv, const int *lens, int batch, int kvh,
                               int tokens_per_split, int splits, float scale, float *part_o, float *part_ml,
                               const Out &out, cudaStream_t stream, int len_all = 0) {
    prepare_decode_kernel<KV, kRep, Out>();
    const dim3 grid(splits, kvh, batch);
    launch_ex(attn_decode_partial_kernel<KV, kRep, Out>, grid, dim3(kDecodeThreads), DecodeGeo<kRep>::kBytes, stream, q,
              q_stride, kv, lens, len_all, tokens_per_split, scale, part_o, part_ml, out, sm100::device_error_word());
    if (splits > 1)
        launch_ex(attn_decode_combine_kernel<Out>, dim3(kvh * kRep, batch), dim3(64), 0, stream,
                  static_cast<const float *>(part_o), static_cast<const float *>(part_ml), splits, out);
}

template <class KV, int kRep, typename Out>
inline void attn_prefill_launch(const float *q, int64_t q_tok, int64_t q_head, const Out &out, const KV &kv, int b,
                                int T, int q_offset, int kvh, float scale, cudaStream_t stream) {
    prepare_prefill_kernel<KV, kRep, Out>();
    constexpr int kPos = kAttnTile / kRep;
    const dim3 grid((T + kPos - 1) / kPos, kvh);
    launch_ex(attn_prefill_kernel<KV, kRep, Out>, grid, dim3(256), PrefillSmem::kBytes, stream, q, q_tok, q_head, out,
              kv, b, T, q_offset, scale, sm100::device_error_word());
}

} // namespace opworks::detail

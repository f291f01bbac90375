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
#include "detail/sm100.cuh"

namespace opworks::detail {

constexpr int kAttnD = 64;      // head dim supported by these kernels
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

constexpr int kDecodeStages = 3;

template <int kRep> struct DecodeSmem {
    static constexpr int kTileFloats = kAttnTile * kAttnD;
    static constexpr size_t kBytes =
        sizeof(float) * (2 * kDecodeStages * kTileFloats // K, V stages
                         + kRep * kAttnD                 // q
                         + 2 * kRep * kAttnTile          // score halves
                         + kRep * kAttnTile              // probabilities
                         + 4 * kRep * kAttnD             // cross-warp reduction
                         + 4 * kRep)                     // alpha, m, l
        + 8 * kDecodeStages + 64;
};

// q: [B][q_stride] with heads at h*64; part_o [B][qh][splits][64]; part_ml
// [B][qh][splits][2] (running max, running sum).
template <class KV, int kRep>
__global__ void __launch_bounds__(128)
    attn_decode_partial_kernel(const float *__restrict__ q, int64_t q_stride, KV kv, const int *__restrict__ lens,
                               int tokens_per_split, float scale, float *__restrict__ part_o,
                               float *__restrict__ part_ml, int *err) {
    using SM = DecodeSmem<kRep>;
    constexpr int kHPW = (kRep + 3) / 4; // heads per softmax warp
    extern __shared__ __align__(128) uint8_t smem_raw[];
    float *ks = reinterpret_cast<float *>(smem_raw);
    float *vs = ks + kDecodeStages * SM::kTileFloats;
    float *qs = vs + kDecodeStages * SM::kTileFloats;
    float *sc = qs + kRep * kAttnD;
    float *ps = sc + 2 * kRep * kAttnTile;
    float *red = ps + kRep * kAttnTile;
    float *al = red + 4 * kRep * kAttnD;
    float *mls = al + kRep;
    uint64_t *full = reinterpret_cast<uint64_t *>(
        (reinterpret_cast<uintptr_t>(mls + 3 * kRep) + 7) & ~static_cast<uintptr_t>(7));

    const int b = blockIdx.z, h = blockIdx.y, split = blockIdx.x, splits = gridDim.x;
    const int qh_total = gridDim.y * kRep;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int len = lens[b];
    const int t_begin = split * tokens_per_split;
    const int t_end = min(len, t_begin + tokens_per_split);
    const int n_tiles = t_end > t_begin ? (t_end - t_begin + kAttnTile - 1) / kAttnTile : 0;

    for (int i = tid; i < kRep * kAttnD; i += blockDim.x)
        qs[i] = q[static_cast<int64_t>(b) * q_stride + static_cast<int64_t>(h) * kRep * kAttnD + i];
    if (tid == 0) {
        for (int s = 0; s < kDecodeStages; ++s)
            sm100::mbar_init(&full[s], 1);
        sm100::fence_mbarrier_init();
    }
    __syncthreads();
    int issued = 0;
    if (tid == 0) {
        for (; issued < kDecodeStages && issued < n_tiles; ++issued)
            stage_kv_tile(kv, b, h, t_begin + issued * kAttnTile, t_end, ks + issued * SM::kTileFloats,
                          vs + issued * SM::kTileFloats, &full[issued]);
    }

    float m_run[kHPW], l_run[kHPW];
#pragma unroll
    for (int j = 0; j < kHPW; ++j) {
        m_run[j] = kNegInf;
        l_run[j] = 0.f;
    }
    float acc[kRep][2];
#pragma unroll
    for (int hd = 0; hd < kRep; ++hd)
        acc[hd][0] = acc[hd][1] = 0.f;

    bool ok = true;
    int consumed = 0;
    for (int tile = 0; tile < n_tiles; ++tile) {
        const int s = tile % kDecodeStages;
        const bool landed = sm100::mbar_wait(&full[s], static_cast<uint32_t>(tile / kDecodeStages) & 1u);
        if (!__syncthreads_and(landed)) {
            ok = false;
            break;
        }
        consumed = tile + 1;
        const int t0 = t_begin + tile * kAttnTile;
        const int valid = min(kAttnTile, t_end - t0);
        const float *K = ks + s * SM::kTileFloats;
        const float *V = vs + s * SM::kTileFloats;

        { // partial scores: thread = (token, half of the head dim)
            const int t = tid & 63, half = tid >> 6;
            float d[kRep];
#pragma unroll
            for (int hd = 0; hd < kRep; ++hd)
                d[hd] = 0.f;
            if (t < valid) {
                const float4 *kr = reinterpret_cast<const float4 *>(K + t * kAttnD + half * 32);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int c = (j + t) & 7; // staggered to spread smem banks
                    const float4 kv4 = kr[c];
#pragma unroll
                    for (int hd = 0; hd < kRep; ++hd) {
                        const float4 qv = reinterpret_cast<const float4 *>(qs + hd * kAttnD + half * 32)[c];
                        d[hd] += kv4.x * qv.x + kv4.y * qv.y + kv4.z * qv.z + kv4.w * qv.w;
                    }
                }
            }
#pragma unroll
            for (int hd = 0; hd < kRep; ++hd)
                sc[(half * kRep + hd) * kAttnTile + t] = d[hd];
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kHPW; ++j) { // online softmax, one warp per head
            const int hd = warp + 4 * j;
            if (hd < kRep) {
                const float s0 = lane < valid
                                     ? (sc[hd * kAttnTile + lane] + sc[(kRep + hd) * kAttnTile + lane]) * scale
                                     : kNegInf;
                const float s1 = lane + 32 < valid ? (sc[hd * kAttnTile + lane + 32] +
                                                      sc[(kRep + hd) * kAttnTile + lane + 32]) *
                                                         scale
                                                   : kNegInf;
                const float mt = warp_reduce<ReduceMax>(fmaxf(s0, s1));
                const float m_new = fmaxf(m_run[j], mt);
                const float alpha = m_run[j] == kNegInf ? 0.f : expf(m_run[j] - m_new);
                const float p0 = lane < valid ? expf(s0 - m_new) : 0.f;
                const float p1 = lane + 32 < valid ? expf(s1 - m_new) : 0.f;
                l_run[j] = l_run[j] * alpha + warp_reduce<ReduceSum>(p0 + p1);
                m_run[j] = m_new;
                ps[hd * kAttnTile + lane] = p0;
                ps[hd * kAttnTile + lane + 32] = p1;
                if (lane == 0)
                    al[hd] = alpha;
            }
        }
        __syncthreads();
        { // P V: warp w takes tokens [16w, 16w+16), lane owns dims 2*lane, 2*lane+1
#pragma unroll
            for (int hd = 0; hd < kRep; ++hd) {
                const float a = al[hd];
                acc[hd][0] *= a;
                acc[hd][1] *= a;
            }
#pragma unroll 4
            for (int tt = 0; tt < 16; ++tt) {
                const int t = warp * 16 + tt;
                if (t < valid) {
                    const float2 v2 = *reinterpret_cast<const float2 *>(V + t * kAttnD + 2 * lane);
#pragma unroll
                    for (int hd = 0; hd < kRep; ++hd) {
                        const float p = ps[hd * kAttnTile + t];
                        acc[hd][0] += p * v2.x;
                        acc[hd][1] += p * v2.y;
                    }
                }
            }
        }
        __syncthreads(); // stage s, scores and probabilities are free again
        if (tid == 0 && issued < n_tiles) {
            const int ns = issued % kDecodeStages;
            stage_kv_tile(kv, b, h, t_begin + issued * kAttnTile, t_end, ks + ns * SM::kTileFloats,
                          vs + ns * SM::kTileFloats, &full[ns]);
            ++issued;
        }
    }

    if (!ok) {
        // drain copies still in flight before the CTA exits
        if (tid == 0) {
            for (int j = consumed; j < issued; ++j)
                sm100::mbar_wait(&full[j % kDecodeStages], static_cast<uint32_t>(j / kDecodeStages) & 1u);
            atomicExch(err, 2);
        }
        return;
    }
#pragma unroll
    for (int hd = 0; hd < kRep; ++hd) {
        red[(warp * kRep + hd) * kAttnD + 2 * lane] = acc[hd][0];
        red[(warp * kRep + hd) * kAttnD + 2 * lane + 1] = acc[hd][1];
    }
#pragma unroll
    for (int j = 0; j < kHPW; ++j) {
        const int hd = warp + 4 * j;
        if (hd < kRep && lane == 0) {
            mls[2 * hd] = m_run[j];
            mls[2 * hd + 1] = l_run[j];
        }
    }
    __syncthreads();
    for (int i = tid; i < kRep * kAttnD; i += blockDim.x) {
        const int hd = i / kAttnD, d = i % kAttnD;
        const float o = red[(0 * kRep + hd) * kAttnD + d] + red[(1 * kRep + hd) * kAttnD + d] +
                        red[(2 * kRep + hd) * kAttnD + d] + red[(3 * kRep + hd) * kAttnD + d];
        const int64_t row = (static_cast<int64_t>(b) * qh_total + h * kRep + hd) * splits + split;
        part_o[row * kAttnD + d] = o;
    }
    if (tid < kRep) {
        const int64_t row = (static_cast<int64_t>(b) * qh_total + h * kRep + tid) * splits + split;
        part_ml[2 * row] = mls[2 * tid];
        part_ml[2 * row + 1] = mls[2 * tid + 1];
    }
}

__device__ __forceinline__ void store_out(float *p, float v) { *p = v; }
__device__ __forceinline__ void store_out(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }

// Merge the split partials of every (sequence, q head): block = 64 threads
// (one per dim), grid = (qh, B). out[b * out_stride + hq * 64 + d].
template <typename OutT>
__global__ void __launch_bounds__(64)
    attn_decode_combine_kernel(const float *__restrict__ part_o, const float *__restrict__ part_ml, int splits,
                               OutT *__restrict__ out, int64_t out_stride) {
    const int hq = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
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
            const float w = expf(m - M);
            L += w * part_ml[2 * (base + s) + 1];
            o += w * part_o[(base + s) * kAttnD + d];
        }
    }
    store_out(out + static_cast<int64_t>(b) * out_stride + static_cast<int64_t>(hq) * kAttnD + d,
              L > 0.f ? o / L : 0.f);
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
template <class KV, int kRep, typename OutT>
__global__ void __launch_bounds__(256)
    attn_prefill_kernel(const float *__restrict__ q, int64_t q_tok, int64_t q_head, OutT *__restrict__ out,
                        int64_t o_tok, int64_t o_head, KV kv, int b, int T, int q_offset, float scale, int *err) {
    constexpr int kPos = kAttnTile / kRep; // query positions per CTA
    using SM = PrefillSmem;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    float *ks = reinterpret_cast<float *>(smem_raw);
    float *vs = ks + kPrefillStages * SM::kTileFloats;
    float *qt = vs + kPrefillStages * SM::kTileFloats; // [64 d][kPad]
    float *kt = qt + kAttnD * kPad;                    // [64 d][kPad]
    float *pm = kt + kAttnD * kPad;                    // [64 rows][kPad]
    uint64_t *full = reinterpret_cast<uint64_t *>(pm + kAttnD * kPad);

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
        OutT *dst = out + static_cast<int64_t>(p0 + pi) * o_tok + static_cast<int64_t>(h * kRep + hd) * o_head + c0;
        if constexpr (std::is_same_v<OutT, float>) {
            *reinterpret_cast<float4 *>(dst) =
                make_float4(o[jr][0] * inv, o[jr][1] * inv, o[jr][2] * inv, o[jr][3] * inv);
        } else {
            __nv_bfloat162 *d2 = reinterpret_cast<__nv_bfloat162 *>(dst);
            d2[0] = __floats2bfloat162_rn(o[jr][0] * inv, o[jr][1] * inv);
            d2[1] = __floats2bfloat162_rn(o[jr][2] * inv, o[jr][3] * inv);
        }
    }
}

// ----------------------------------------------------------- host helpers

template <class KV, int kRep> inline void prepare_decode_kernel() {
    static thread_local int done = -1;
    int dev = 0;
    OPWORKS_CUDA_CHECK(cudaGetDevice(&dev));
    if (done != dev) {
        OPWORKS_CUDA_CHECK(cudaFuncSetAttribute(attn_decode_partial_kernel<KV, kRep>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(DecodeSmem<kRep>::kBytes)));
        done = dev;
    }
}

template <class KV, int kRep, typename OutT> inline void prepare_prefill_kernel() {
    static thread_local int done = -1;
    int dev = 0;
    OPWORKS_CUDA_CHECK(cudaGetDevice(&dev));
    if (done != dev) {
        OPWORKS_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_kernel<KV, kRep, OutT>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(PrefillSmem::kBytes)));
        done = dev;
    }
}

// Split-KV geometry for `pairs` (sequence, kv head) pairs whose longest
// visible length is max_len: tokens per split is a multiple of the tile.
inline int decode_tokens_per_split(int pairs, int max_len, int sm_count) {
    const int tiles = (max_len + kAttnTile - 1) / kAttnTile;
    const int target = 4 * sm_count; // ~2 waves at 2 CTAs per SM
    int splits = (target + pairs - 1) / pairs;
    if (splits > tiles)
        splits = tiles;
    if (splits < 1)
        splits = 1;
    const int tiles_per_split = (tiles + splits - 1) / splits;
    return (tiles_per_split > 0 ? tiles_per_split : 1) * kAttnTile;
}

template <class KV, int kRep, typename OutT>
inline void attn_decode_launch(const float *q, int64_t q_stride, const KV &kv, const int *lens, int batch, int kvh,
                               int tokens_per_split, int splits, float scale, float *part_o, float *part_ml,
                               OutT *out, int64_t out_stride, cudaStream_t stream) {
    prepare_decode_kernel<KV, kRep>();
    const dim3 grid(splits, kvh, batch);
    attn_decode_partial_kernel<KV, kRep><<<grid, 128, DecodeSmem<kRep>::kBytes, stream>>>(
        q, q_stride, kv, lens, tokens_per_split, scale, part_o, part_ml, sm100::device_error_word());
    OPWORKS_CUDA_CHECK(cudaGetLastError());
    attn_decode_combine_kernel<OutT><<<dim3(kvh * kRep, batch), 64, 0, stream>>>(part_o, part_ml, splits, out,
                                                                                 out_stride);
    OPWORKS_CUDA_CHECK(cudaGetLastError());
}

template <class KV, int kRep, typename OutT = float>
inline void attn_prefill_launch(const float *q, int64_t q_tok, int64_t q_head, OutT *out, int64_t o_tok,
                                int64_t o_head, const KV &kv, int b, int T, int q_offset, int kvh, float scale,
                                cudaStream_t stream) {
    prepare_prefill_kernel<KV, kRep, OutT>();
    constexpr int kPos = kAttnTile / kRep;
    const dim3 grid((T + kPos - 1) / kPos, kvh);
    attn_prefill_kernel<KV, kRep, OutT><<<grid, 256, PrefillSmem::kBytes, stream>>>(
        q, q_tok, q_head, out, o_tok, o_head, kv, b, T, q_offset, scale, sm100::device_error_word());
    OPWORKS_CUDA_CHECK(cudaGetLastError());
}

} // namespace opworks::detail

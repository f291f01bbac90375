#pragma once

// Causal GQA prefill attention on the 5th-generation tensor cores (sm_100a).
//
// One CTA owns 128 query rows of one KV head: 128 / kRep positions x the kRep
// query heads that share the KV head (rows ordered position-major, exactly as
// a 3-D TMA box {32 dims, kRep heads, 128 / kRep positions} lands them). It
// walks the KV range in 128-key tiles staged by TMA straight from the paged
// fp32 cache (16-token pages, one 2 KB box per page and 32-dim half). A tile
// whose eight pages are consecutive physical blocks (the block allocator
// hands a prefill ascending blocks) is staged with three copies instead of
// 24: one 8-page box per K half and one for V, through run tensor maps that
// step over blocks instead of (block, head) rows; both land the same bytes at
// the same shared-memory addresses.
//
//   S = Q K^T   tcgen05.mma kind::tf32, A = Q (K-major, smem), B = K (K-major,
//               smem: the cache's [token][dim] rows), D in TMEM (128 x 128)
//   P = softmax  8 warps, two per TMEM lane quarter: a thread owns half of a
//               query row (64 of the 128 keys), the pair exchanges half-row
//               maxima; scores in log2 units (one FFMA + exp2 on the SFU per
//               score), causal mask on diagonal tiles only, running max /
//               sum; P truncated to tf32 as the MMA reads it
//   O += P V    tcgen05.mma kind::tf32, A = P (TMEM, written back over S),
//               B = V (MN-major smem: the same [token][dim] rows), D in TMEM
//               (128 x 64, double-buffered); the softmax warps fold tile n-1's
//               P V into fp32 registers (running rescale) after publishing
//               tile n's P, so they never wait for the P V of the tile they
//               just handed over
//
// Roles (320 threads): warp 0 TMA producer (four lanes), warp 1 TMEM
// allocator and single-thread MMA issuer, warps 2-9 softmax + epilogue. S is
// double-buffered in TMEM, so QK^T of tile n+1 runs while tile n's softmax
// does; three KV stages (226 KB of shared memory with Q) keep the reload of a
// stage (PV commit, 32 page copies, their latency) off the softmax's path.
// Every mbarrier wait is bounded (device error word on timeout).
//
// Precision: TF32 operands (10-bit mantissa) with fp32 accumulation; used by
// the fast (bf16-weight) model path only.

#include "attention_kernels.cuh"
#include "detail/sm100.cuh"

namespace opworks::detail {

constexpr int kPfKvTile = 128;   // keys per KV tile (8 pages)
constexpr int kPfStages = 3;     // KV tiles in flight
constexpr int kPfThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 softmax
constexpr int kPfSoftmaxThreads = 256;
constexpr uint32_t kPfTmemCols = 512; // S0 [0,128), S1 [128,256), O0 [256,320), O1 [320,384)

struct PrefillTcSmem {
    static constexpr uint32_t kSlab = 128 * 128;          // [128 rows][32 fp32], 16 KB
    static constexpr uint32_t kQBytes = 2 * kSlab;         // dims 0-31, 32-63
    static constexpr uint32_t kStageBytes = 4 * kSlab;     // K halves, V halves
    // Q | KV stages | barriers (256 B) | half-row max exchange [2][2][128]
    // floats. No alignment slack: the kernel checks that the dynamic
    // shared-memory base is 1024-byte aligned (128B-swizzled operands)
    static constexpr size_t kBytes = kQBytes + kPfStages * kStageBytes + 256 + 4 * 128 * 4;
};

using sm100::sdesc_mn128_32b;

// sm_100 packed fp32 pairs (one instruction for two lanes' worth of work)
// and the three-input max: the softmax's per-score instruction count.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// D[tmem] (+)= A[tmem] * B[smem desc], tf32 (A from tensor memory, K-major).
__device__ __forceinline__ void umma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
                 "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
                 : "memory");
}

__device__ __forceinline__ void tmem_st_32x16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
                 "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
                 "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tma_load_4d(void *smem_dst, const CUtensorMap *tm, uint64_t *bar, int c0, int c1,
                                            int c2, int c3) {
    asm volatile("cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(sm100::smem_u32(smem_dst)),
                 "l"(reinterpret_cast<uint64_t>(tm)), "r"(sm100::smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}

__device__ __forceinline__ void tma_load_5d(void *smem_dst, const CUtensorMap *tm, uint64_t *bar, int c0, int c1,
                                            int c2, int c3, int c4) {
    asm volatile("cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(sm100::smem_u32(smem_dst)),
                 "l"(reinterpret_cast<uint64_t>(tm)), "r"(sm100::smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
                 "r"(c4)
                 : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *smem_dst, const CUtensorMap *tm, uint64_t *bar, int c0, int c1,
                                            int c2) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(sm100::smem_u32(smem_dst)),
                 "l"(reinterpret_cast<uint64_t>(tm)), "r"(sm100::smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}

// Causal prefill of `T` query rows of sequence `b` (absolute positions
// q_offset + t), grid = (ceil(T / (128 / kRep)), kvh); the heaviest query
// tiles are scheduled first. tmQ covers q as {64 dims, qh heads, T rows};
// tmK / tmV cover the KV pool as {64 dims, 16 tokens, blocks * kvh}; tmKr /
// tmVr (the run maps) as {64 dims, 16 tokens, kvh, blocks} with 8-block boxes.
template <int kRep, typename Out>
__global__ void __launch_bounds__(kPfThreads, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmKr,
                           const __grid_constant__ CUtensorMap tmVr, const int *__restrict__ table, int table_stride,
                           int kvh, int b, int T, int q_offset, float scale, Out out, int *err) {
    using SM = PrefillTcSmem;
    constexpr int kPos = 128 / kRep; // query positions per CTA
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    if ((sm100::smem_u32(smem_raw) & 1023u) != 0) { // never taken on sm_100a (no static shared memory)
        if (threadIdx.x == 0)
            atomicExch(err, 5);
        return;
    }
    uint8_t *smem = smem_raw;
    uint8_t *qs = smem;
    uint8_t *stages = smem + SM::kQBytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(stages + kPfStages * SM::kStageBytes);
    uint64_t *full_q = bars;
    uint64_t *full_kv = bars + 1;              // [kPfStages]
    uint64_t *empty_kv = full_kv + kPfStages;  // [kPfStages]
    uint64_t *s_ready = empty_kv + kPfStages;  // [2]
    uint64_t *p_ready = s_ready + 2;           // [2]
    uint64_t *o_ready = p_ready + 2;           // [2]
    uint64_t *o_free = o_ready + 2;            // [2]
    uint64_t *drain = o_free + 2;
    uint64_t *xch = drain + 1;                 // [2 tile parities][4 quarters]: half-row max exchange
    uint64_t *xch_l = xch + 8;                 // [4 quarters]: row-sum exchange
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(xch_l + 4);
    float *xv = reinterpret_cast<float *>(bars + 32); // [2 parities][2 halves][128 rows]

    const int warp = threadIdx.x / kWarpSize, lane = threadIdx.x % kWarpSize;
    const int qt = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x); // heaviest first
    const int h = blockIdx.y;
    const int t0 = qt * kPos;
    const int t_last = min(T, t0 + kPos) - 1;           // last query row of the tile
    const int keys = q_offset + t_last + 1;             // keys any row of the tile may see
    const int n_tiles = (keys + kPfKvTile - 1) / kPfKvTile;
    const int last_page = (keys - 1) / kKvChunk;

    if (threadIdx.x == 0) {
        sm100::mbar_init(full_q, 1);
        for (int s = 0; s < kPfStages; ++s) {
            sm100::mbar_init(&full_kv[s], 1);
            sm100::mbar_init(&empty_kv[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            sm100::mbar_init(&s_ready[i], 1);
            sm100::mbar_init(&p_ready[i], kPfSoftmaxThreads);
        }
        for (int i = 0; i < 2; ++i) {
            sm100::mbar_init(&o_ready[i], 1);
            sm100::mbar_init(&o_free[i], kPfSoftmaxThreads);
        }
        sm100::mbar_init(drain, 1);
        for (int i = 0; i < 8; ++i)
            sm100::mbar_init(&xch[i], 64);
        for (int i = 0; i < 4; ++i)
            sm100::mbar_init(&xch_l[i], 64);
        sm100::fence_mbarrier_init();
        sm100::prefetch_tmap(&tmQ);
        sm100::prefetch_tmap(&tmK);
        sm100::prefetch_tmap(&tmV);
        sm100::prefetch_tmap(&tmKr);
        sm100::prefetch_tmap(&tmVr);
    }
    if (warp == 1) {
        sm100::tmem_alloc(tmem_slot, kPfTmemCols);
        sm100::tmem_relinquish();
    }
    pdl_trigger();
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        // producer: lanes 0-3 each copy two of a tile's eight pages (K and V,
        // two 32-dim halves each); lane 0 posts the tile's byte count
        constexpr int kIssuers = 4;
        constexpr int kPagesPerLane = kPfKvTile / kKvChunk / kIssuers;
        if (lane < kIssuers) {
            pdl_wait(); // q and the cache are written by earlier kernels
            if (lane == 0) {
                sm100::mbar_arrive_expect_tx(full_q, SM::kQBytes);
                tma_load_3d(qs, &tmQ, full_q, 0, h * kRep, t0);
                tma_load_3d(qs + SM::kSlab, &tmQ, full_q, 32, h * kRep, t0);
            }
            int issued = 0;
            for (int n = 0; n < n_tiles; ++n, ++issued) {
                const int s = n % kPfStages;
                const bool freed =
                    n < kPfStages || sm100::mbar_wait(&empty_kv[s], static_cast<uint32_t>((n / kPfStages) - 1) & 1u);
                if (!__all_sync(0xFu, freed)) { // the four lanes leave together (they shuffle below)
                    ok = false;
                    break;
                }
                uint8_t *st = stages + s * SM::kStageBytes;
                // block-table entries first (their loads overlap; the copies
                // are ordered after them); pages past the last key still load
                // (a valid page): their keys are masked and P = 0 there
                int rows[kPagesPerLane];
#pragma unroll
                for (int i = 0; i < kPagesPerLane; ++i)
                    rows[i] = table[static_cast<int64_t>(b) * table_stride +
                                    min(n * (kPfKvTile / kKvChunk) + lane * kPagesPerLane + i, last_page)] * kvh + h;
                // a run: the tile's eight pages are consecutive blocks, all
                // at or before the last page (rows[] = block * kvh + h)
                const int row0 = __shfl_sync(0xFu, rows[0], 0);
                bool mine = n * (kPfKvTile / kKvChunk) + kPfKvTile / kKvChunk - 1 <= last_page;
#pragma unroll
                for (int i = 0; i < kPagesPerLane; ++i)
                    mine = mine && rows[i] == row0 + (lane * kPagesPerLane + i) * kvh;
                const bool run = __all_sync(0xFu, mine);
                if (lane == 0)
                    sm100::mbar_arrive_expect_tx(&full_kv[s], SM::kStageBytes);
                if (run) {
                    const int blk0 = (row0 - h) / kvh;
                    if (lane == 0)
                        tma_load_4d(st, &tmKr, &full_kv[s], 0, 0, h, blk0);
                    else if (lane == 1)
                        tma_load_4d(st + SM::kSlab, &tmKr, &full_kv[s], 32, 0, h, blk0);
                    else if (lane == 2) // [block][half][16 keys][32], as the page copies land
                        tma_load_5d(st + 2 * SM::kSlab, &tmVr, &full_kv[s], 0, 0, 0, h, blk0);
                } else {
#pragma unroll
                    for (int i = 0; i < kPagesPerLane; ++i) {
                        const int row = rows[i];
                        const uint32_t off = static_cast<uint32_t>(lane * kPagesPerLane + i) * kKvChunk * 128;
                        tma_load_3d(st + off, &tmK, &full_kv[s], 0, 0, row);
                        tma_load_3d(st + SM::kSlab + off, &tmK, &full_kv[s], 32, 0, row);
                        // V page: both 32-dim halves in one copy, [half][16 keys][32]
                        tma_load_4d(st + 2 * SM::kSlab + 2 * off, &tmV, &full_kv[s], 0, 0, 0, row);
                    }
                }
            }
            // no copy may be in flight when the CTA exits (each phase of a
            // stage completes only when all four lanes' copies landed)
            if (lane == 0) {
                if (!sm100::mbar_wait(full_q, 0))
                    ok = false;
                for (int j = (issued > kPfStages ? issued - kPfStages : 0); j < issued; ++j)
                    if (!sm100::mbar_wait(&full_kv[j % kPfStages], static_cast<uint32_t>(j / kPfStages) & 1u))
                        ok = false;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = sm100::idesc_make(sm100::kFmtTF32, 128, kPfKvTile);
            constexpr uint32_t idesc_o = sm100::idesc_make(sm100::kFmtTF32, 128, 64) | (1u << 16); // B MN-major
            const uint32_t qa = sm100::smem_u32(qs);
            auto issue_s = [&](int n) {
                const int s = n % kPfStages;
                const uint32_t kb = sm100::smem_u32(stages + s * SM::kStageBytes);
                const uint32_t d = tmem + static_cast<uint32_t>((n & 1) * kPfKvTile);
                for (int ks = 0; ks < 8; ++ks) { // 8 dims per step: 2 halves x 4 steps of 32 bytes
                    const uint32_t o = static_cast<uint32_t>(ks / 4) * SM::kSlab + static_cast<uint32_t>(ks % 4) * 32u;
                    sm100::umma_tf32(d, sm100::sdesc_k128(qa + o), sm100::sdesc_k128(kb + o), idesc_s, ks > 0);
                }
                sm100::umma_commit(&s_ready[n & 1]);
            };
            if (!sm100::mbar_wait(full_q, 0)) {
                ok = false;
            } else if (n_tiles > 0) {
                if (!sm100::mbar_wait(&full_kv[0], 0)) {
                    ok = false;
                } else {
                    sm100::tc_fence_after();
                    issue_s(0);
                }
            }
            for (int n = 0; ok && n < n_tiles; ++n) {
                if (n + 1 < n_tiles) {
                    const int s1 = (n + 1) % kPfStages;
                    if (!sm100::mbar_wait(&full_kv[s1], static_cast<uint32_t>((n + 1) / kPfStages) & 1u)) {
                        ok = false;
                        break;
                    }
                    sm100::tc_fence_after();
                    issue_s(n + 1);
                }
                // O buffer n & 1 was last folded after P V of tile n - 2
                if (!sm100::mbar_wait(&p_ready[n & 1], static_cast<uint32_t>(n >> 1) & 1u) ||
                    (n >= 2 && !sm100::mbar_wait(&o_free[n & 1], static_cast<uint32_t>((n >> 1) - 1) & 1u))) {
                    ok = false;
                    break;
                }
                sm100::tc_fence_after();
                const int s = n % kPfStages;
                const uint32_t vb = sm100::smem_u32(stages + s * SM::kStageBytes + 2 * SM::kSlab);
                const uint32_t pa = tmem + static_cast<uint32_t>((n & 1) * kPfKvTile);
                const uint32_t od = tmem + 256u + static_cast<uint32_t>((n & 1) * 64);
                // 8 keys per step: half a V page ([half][16 keys][32 dims],
                // 4 KB per page, the 32-dim halves 2 KB apart)
                for (int ks = 0; ks < kPfKvTile / 8; ++ks)
                    umma_tf32_ts(od, pa + static_cast<uint32_t>(ks * 8),
                                 sdesc_mn128_32b(vb + static_cast<uint32_t>(ks >> 1) * 4096u +
                                                     static_cast<uint32_t>(ks & 1) * 1024u,
                                                 2048u, 512u),
                                 idesc_o, ks > 0);
                sm100::umma_commit(&o_ready[n & 1]);
                sm100::umma_commit(&empty_kv[s]);
            }
            // every issued MMA completes before tensor memory is released
            sm100::umma_commit(drain);
            if (!sm100::mbar_wait(drain, 0))
                ok = false;
        }
    } else {
        // softmax warps 2-9: warp w reads TMEM lane quarter w % 4 (row
        // r = 32 (w % 4) + lane) and column half (w - 2) / 4 of every tile:
        // S / P columns [64 half, +64), O dims [32 half, +32). The two warps
        // of a row exchange their half-row maxima through shared memory (an
        // mbarrier per quarter and tile parity, bounded waits) so both use
        // the same running max; each keeps its half of the row sum.
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int r = quarter * 32 + lane;
        const int p = r / kRep, hh = r % kRep;
        const int t = t0 + p;
        const int qpos = q_offset + t;
        const int qpos_min = q_offset + t0; // first row of the CTA: tiles below it need no mask
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        const float c = scale * kLog2e; // scores in log2 units: p = 2^(s c - m c)
        float m_run = kNegInf, l_run = 0.f, alpha_prev = 0.f;
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i)
            o[i] = 0.f;
        // o = o * alpha + (P V of tile k)[dims 32 half ..] (buffer k & 1)
        auto fold = [&](int k, float alpha) -> bool {
            if (!sm100::mbar_wait_warp(&o_ready[k & 1], static_cast<uint32_t>(k >> 1) & 1u)) {
                ok = false;
                return false;
            }
            sm100::tc_fence_after();
            uint32_t rr[2][16];
#pragma unroll
            for (int cc = 0; cc < 2; ++cc)
                sm100::tmem_ld_32x16(tmem + lane_addr + 256u + static_cast<uint32_t>((k & 1) * 64 + 32 * half + cc * 16),
                                     rr[cc]);
            sm100::tmem_wait_ld();
            const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                sm100::tmem_reg_fence(rr[cc]);
#pragma unroll
                for (int i = 0; i < 16; i += 2) {
                    const float2 r = ffma2(make_float2(o[cc * 16 + i], o[cc * 16 + i + 1]), a2,
                                           make_float2(__uint_as_float(rr[cc][i]), __uint_as_float(rr[cc][i + 1])));
                    o[cc * 16 + i] = r.x;
                    o[cc * 16 + i + 1] = r.y;
                }
            }
            sm100::tc_fence_before();
            sm100::mbar_arrive(&o_free[k & 1]);
            return true;
        };
        for (int n = 0; n < n_tiles; ++n) {
            const uint32_t sb = tmem + lane_addr + static_cast<uint32_t>((n & 1) * kPfKvTile + 64 * half);
            if (!sm100::mbar_wait_warp(&s_ready[n & 1], static_cast<uint32_t>(n >> 1) & 1u)) {
                ok = false;
                break;
            }
            sm100::tc_fence_after();
            const int k0 = n * kPfKvTile + 64 * half; // first key of this warp's columns
            uint32_t v[4][16];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc)
                sm100::tmem_ld_32x16(sb + static_cast<uint32_t>(cc * 16), v[cc]);
            sm100::tmem_wait_ld();
            // raw-score max, one accumulator per 16 columns (short chains);
            // the causal mask only on tiles that reach past the CTA's first row
            const bool masked = n * kPfKvTile + kPfKvTile - 1 > qpos_min;
            float mg[4];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                sm100::tmem_reg_fence(v[cc]);
                mg[cc] = kNegInf;
                if (masked) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float sv = k0 + cc * 16 + i <= qpos ? __uint_as_float(v[cc][i]) : kNegInf;
                        v[cc][i] = __float_as_uint(sv);
                        mg[cc] = fmaxf(mg[cc], sv);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 16; i += 2)
                        mg[cc] = fmax3(mg[cc], __uint_as_float(v[cc][i]), __uint_as_float(v[cc][i + 1]));
                }
            }
            float mt = fmaxf(fmaxf(mg[0], mg[1]), fmaxf(mg[2], mg[3]));
            // exchange with the other half of the row
            xv[((n & 1) * 2 + half) * 128 + r] = mt;
            sm100::mbar_arrive(&xch[(n & 1) * 4 + quarter]);
            if (!sm100::mbar_wait_warp(&xch[(n & 1) * 4 + quarter], static_cast<uint32_t>(n >> 1) & 1u)) {
                ok = false;
                break;
            }
            mt = fmaxf(mt, xv[((n & 1) * 2 + (half ^ 1)) * 128 + r]);
            const float m_new = fmaxf(m_run, mt);
            const float alpha = m_run == kNegInf ? 0.f : exp2_approx((m_run - m_new) * c);
            const float mc = m_new == kNegInf ? 0.f : m_new * c;
            float2 lg[4];
            const float2 c2 = make_float2(c, c), nmc2 = make_float2(-mc, -mc);
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                lg[cc] = make_float2(0.f, 0.f);
#pragma unroll
                for (int i = 0; i < 16; i += 2) {
                    // masked scores are -inf: 2^-inf = 0. The MMA reads P as
                    // tf32 by dropping the 13 low mantissa bits, so the row
                    // sum adds P truncated the same way: the weights the P V
                    // product uses are exactly the ones normalised. Pairs of
                    // scores go through the packed fp32x2 FMA and add.
                    const float2 t =
                        ffma2(make_float2(__uint_as_float(v[cc][i]), __uint_as_float(v[cc][i + 1])), c2, nmc2);
                    const uint32_t u0 = __float_as_uint(exp2_approx(t.x)), u1 = __float_as_uint(exp2_approx(t.y));
                    lg[cc] = fadd2(lg[cc], make_float2(__uint_as_float(u0 & 0xffffe000u),
                                                       __uint_as_float(u1 & 0xffffe000u)));
                    v[cc][i] = u0;
                    v[cc][i + 1] = u1;
                }
                tmem_st_32x16(sb + static_cast<uint32_t>(cc * 16), v[cc]);
            }
            tmem_wait_st();
            l_run = l_run * alpha + (((lg[0].x + lg[0].y) + (lg[1].x + lg[1].y)) +
                                     ((lg[2].x + lg[2].y) + (lg[3].x + lg[3].y)));
            m_run = m_new;
            sm100::tc_fence_before();
            sm100::mbar_arrive(&p_ready[n & 1]);
            // fold the previous tile's P V (its MMA ran while this tile's
            // softmax did)
            if (n > 0 && !fold(n - 1, alpha_prev))
                break;
            alpha_prev = alpha;
        }
        if (ok && n_tiles > 0)
            fold(n_tiles - 1, alpha_prev);
        // row sum = half 0 + half 1 (the same order in both warps), through
        // the exchange buffer of parity n_tiles & 1: its last readers (tile
        // n_tiles - 2) finished before the partner arrived on tile n_tiles - 1
        float *xl = xv + (n_tiles & 1) * 256;
        xl[half * 128 + r] = l_run;
        sm100::mbar_arrive(&xch_l[quarter]);
        if (!sm100::mbar_wait_warp(&xch_l[quarter], 0))
            ok = false;
        if (ok && t < T) {
            const float l_tot = xl[r] + xl[128 + r];
            const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
#pragma unroll
            for (int d = 0; d < 32; d += 4)
                out.put4(t, h * kRep + hh, 32 * half + d, o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
        }
    }
    if (!ok)
        atomicExch(err, 4);
    sm100::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        sm100::tc_fence_after();
        sm100::tmem_dealloc(tmem, kPfTmemCols);
    }
}

// 3-D fp32 tensor map with a 128-byte-wide innermost box (32 floats) and
// 128B swizzle: dims / strides in elements / bytes, innermost first.
inline CUtensorMap make_tmap_3d_f32(const void *base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_bytes,
                                    uint64_t stride2_bytes, uint32_t box1, uint32_t box2,
                                    CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    require(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
    require(stride1_bytes % 16 == 0 && stride2_bytes % 16 == 0, "TMA strides must be multiples of 16 bytes");
    CUtensorMap tm;
    std::memset(&tm, 0, sizeof(tm));
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
    const cuuint32_t box[3] = {32, box1, box2};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = sm100::tensor_map_encoder()(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void *>(base),
                                                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                                   swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    require(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (3-D) failed");
    return tm;
}

// Tensor maps of one K or V pool [blocks][kvh][16][64] fp32. K pages land in
// the K-major 128B-swizzle layout, one copy per 32-dim half ({32 dims, 16
// tokens, page}); V pages in the MN-major one (32-byte swizzle atoms), both
// halves in one copy: dims {32 dims, 16 tokens (256 B apart), 2 halves
// (128 B apart), page}, landing as [half][16 tokens][32].
inline CUtensorMap make_kv_pool_tmap(const float *pool, int64_t blocks, int kvh, bool v_operand) {
    if (!v_operand)
        return make_tmap_3d_f32(pool, kAttnD, kKvChunk, static_cast<uint64_t>(blocks) * kvh, kAttnD * 4,
                                kKvChunk * kAttnD * 4, kKvChunk, 1, CU_TENSOR_MAP_SWIZZLE_128B);
    require(reinterpret_cast<uintptr_t>(pool) % 16 == 0, "TMA base must be 16-byte aligned");
    CUtensorMap tm;
    std::memset(&tm, 0, sizeof(tm));
    const cuuint64_t dims[4] = {32, kKvChunk, 2, static_cast<cuuint64_t>(blocks) * kvh};
    const cuuint64_t strides[3] = {kAttnD * 4, 32 * 4, kKvChunk * kAttnD * 4};
    const cuuint32_t box[4] = {32, kKvChunk, 2, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = sm100::tensor_map_encoder()(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float *>(pool),
                                                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                                   CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    require(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (4-D V pages) failed");
    return tm;
}

// Run maps of the same pool: K as {64 dims, 16 tokens, kvh, blocks} with box
// {32, 16, 1, 8} (eight consecutive blocks of one head land as [128 keys][32],
// one copy per 32-dim half), V as {32 dims, 16 tokens, 2 halves, kvh, blocks}
// with box {32, 16, 2, 1, 8} (landing as [block][half][16 keys][32]).
inline CUtensorMap make_kv_run_tmap(const float *pool, int64_t blocks, int kvh, bool v_operand) {
    require(reinterpret_cast<uintptr_t>(pool) % 16 == 0, "TMA base must be 16-byte aligned");
    CUtensorMap tm;
    std::memset(&tm, 0, sizeof(tm));
    const cuuint64_t page_bytes = kKvChunk * kAttnD * 4;
    CUresult r;
    if (!v_operand) {
        const cuuint64_t dims[4] = {kAttnD, kKvChunk, static_cast<cuuint64_t>(kvh), static_cast<cuuint64_t>(blocks)};
        const cuuint64_t strides[3] = {kAttnD * 4, page_bytes, page_bytes * static_cast<cuuint64_t>(kvh)};
        const cuuint32_t box[4] = {32, kKvChunk, 1, kPfKvTile / kKvChunk};
        const cuuint32_t estr[4] = {1, 1, 1, 1};
        r = sm100::tensor_map_encoder()(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float *>(pool), dims,
                                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        const cuuint64_t dims[5] = {32, kKvChunk, 2, static_cast<cuuint64_t>(kvh), static_cast<cuuint64_t>(blocks)};
        const cuuint64_t strides[4] = {kAttnD * 4, 32 * 4, page_bytes, page_bytes * static_cast<cuuint64_t>(kvh)};
        const cuuint32_t box[5] = {32, kKvChunk, 2, 1, kPfKvTile / kKvChunk};
        const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
        r = sm100::tensor_map_encoder()(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, const_cast<float *>(pool), dims,
                                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                        CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    require(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (KV run map) failed");
    return tm;
}

// The four tensor maps of one layer's K and V pools.
struct KvPoolMaps {
    CUtensorMap k, v, k_run, v_run;
};
inline KvPoolMaps make_kv_pool_maps(const float *kpool, const float *vpool, int64_t blocks, int kvh) {
    return {make_kv_pool_tmap(kpool, blocks, kvh, false), make_kv_pool_tmap(vpool, blocks, kvh, true),
            make_kv_run_tmap(kpool, blocks, kvh, false), make_kv_run_tmap(vpool, blocks, kvh, true)};
}

template <int kRep, typename Out> inline void prepare_prefill_tc_kernel() {
    static thread_local int done = -1;
    int dev = 0;
    OPWORKS_CUDA_CHECK(cudaGetDevice(&dev));
    if (done != dev) {
        OPWORKS_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_tc_kernel<kRep, Out>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(PrefillTcSmem::kBytes)));
        done = dev;
    }
}

// q: [T][qh * 64] fp32 rows with row stride q_tok floats; maps from
// make_kv_pool_maps of the layer's pools.
template <int kRep, typename Out>
inline void attn_prefill_tc_launch(const float *q, int64_t q_tok, int qh, const KvPoolMaps &maps, const int *table,
                                   int table_stride, int kvh, int b, int T, int q_offset, float scale, const Out &out,
                                   cudaStream_t stream) {
    static_assert(kRep == 1 || kRep == 2 || kRep == 4 || kRep == 8, "GQA ratio must divide 128 rows");
    require(T > 0 && qh == kvh * kRep, "prefill attention: bad shape");
    prepare_prefill_tc_kernel<kRep, Out>();
    const CUtensorMap qmap = make_tmap_3d_f32(q, kAttnD, static_cast<uint64_t>(qh), static_cast<uint64_t>(T),
                                              kAttnD * 4, static_cast<uint64_t>(q_tok) * 4, kRep, 128 / kRep);
    const dim3 grid((T + 128 / kRep - 1) / (128 / kRep), kvh);
    launch_ex(attn_prefill_tc_kernel<kRep, Out>, grid, dim3(kPfThreads), PrefillTcSmem::kBytes, stream, qmap, maps.k,
              maps.v, maps.k_run, maps.v_run, table, table_stride, kvh, b, T, q_offset, scale, out,
              sm100::device_error_word());
}

} // namespace opworks::detail

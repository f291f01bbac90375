#pragma once

// Two-SM (cta_group::2) tcgen05 GEMM for prefill-sized projections of the
// fast path: bf16 weights times two-term bf16 activations (kBF16x2), fp32
// accumulate, tile epilogue fused.
//
//   out[tok][feat] = epi( sum_k W[feat][k] * (Xhi + Xlo)[tok][k] )
//
// A pair of CTAs (a cluster of 2 along the feature tiles) computes one
// 256-feature x 256-token tile with tcgen05.mma.cta_group::2 (M = 256,
// N = 256): CTA rank r stages the 128 weight rows f0 + 128 r .. and the 128
// token rows t0 + 128 r .. (hi and lo) of every 64-element K block, and the
// leader CTA (rank 0) issues the MMAs, which read both CTAs' shared memory
// and leave rank r's 128 features x 256 tokens in rank r's tensor memory.
// Per CTA and K block that is 48 KB of operands for 128 x 256 x 64 x 2 MACs:
// half the shared-memory traffic per MAC of a one-CTA 128 x 128 tile, which
// is what keeps the tensor cores fed from L2 at prefill sizes.
//
// Protocol (every wait bounded; on a timeout the error word is set and the
// CTA still takes every cluster barrier):
//   * both producers wait on their own empty[s]; the leader's producer
//     posts the expected bytes of BOTH CTAs on the leader's full[s]; both
//     CTAs' TMA loads (.cta_group::2) complete on the leader's full[s];
//   * the leader's MMA thread waits full[s], issues 4 K steps x 2 terms,
//     and commits to empty[s] of both CTAs (multicast commit); after the
//     last block it commits to accum of both CTAs;
//   * each CTA's epilogue warps read their own tensor memory into a
//     [256][128] fp32 tile in shared memory and run the tile epilogue.
// Loads carry no cluster multicast: each CTA fetches its own operands.

#include <algorithm>

#include "gemm_sm100.cuh"

namespace opworks::sm100 {

// kTerms = 2: activations as hi + lo terms (two MMAs per K step); 1: one
// term (one MMA per K step, 32 KB stages, so the ring is 6 deep).
template <int kTerms> struct PairShape {
    static constexpr int BN = 256;                   // tokens per pair tile (128 per CTA staged)
    static constexpr uint32_t kABytes = kUmmaM * kUmmaKBytes; // 128 weight rows x 128 B
    static constexpr uint32_t kBBytes = 128 * kUmmaKBytes;    // 128 token rows x 128 B (one term)
    static constexpr uint32_t kStageBytes = kABytes + kTerms * kBBytes;
    static constexpr int kStages = kTerms == 2 ? 4 : 6;
    static constexpr uint32_t kTmemCols = BN;
    static constexpr size_t kEpiScratchBytes = 16u * BN;
    static constexpr size_t kSmemBytes = 1024 + static_cast<size_t>(kStages) * kStageBytes + 256 + kEpiScratchBytes;
    static_assert(static_cast<size_t>(BN) * kUmmaM * 4 <= static_cast<size_t>(kStages) * kStageBytes,
                  "the fp32 output tile must fit in the pipeline stages");
};

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Shared-memory address of the same variable in cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}

// 2D TMA load into this CTA's shared memory whose completion is counted on
// an mbarrier of either CTA of the pair (shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void *smem_dst, const CUtensorMap *tm, uint32_t bar_cluster, int c0,
                                                 int c1) {
    asm volatile("cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
                 "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar_cluster), "r"(c0), "r"(c1)
                 : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t *slot_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A * B^T over the CTA pair (M = 256 split across the pair,
// N split across the pair's B halves), bf16 inputs.
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
                 "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
                 : "memory");
}

// Arrive once on `bar` (same shared-memory offset) of every CTA in `mask`
// when the MMAs issued so far by this thread have completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t *bar, uint16_t mask) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                     smem_u32(bar)),
                 "h"(mask)
                 : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
    cluster_arrive();
    cluster_wait();
}

// grid = (feature tiles rounded up to even, token tiles of 256), cluster
// (2, 1, 1), 192 threads: warp 0 TMA producer, warp 1 TMEM + MMA issuer
// (leader only), warps 2-5 epilogue.
template <typename Epi, int kTerms>
__global__ void __launch_bounds__(192, 1)
    umma_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmB_lo, GemmParams p, Epi epi) {
    using S = PairShape<kTerms>;
    constexpr int kStages = S::kStages;
    static_assert(is_tile_epilogue<Epi>::value, "the pair GEMM runs tile epilogues");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * S::kStageBytes);
    uint64_t *empty = full + kStages;
    uint64_t *accum = empty + kStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum + 1);
    void *epi_scratch = smem + kStages * S::kStageBytes + 256;

    const int warp = threadIdx.x / kWarpSize;
    const int lane = threadIdx.x % kWarpSize;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int f0 = blockIdx.x * kUmmaM;        // this CTA's 128 features
    const int t0 = blockIdx.y * S::BN;         // the pair's 256 tokens
    const int tb = t0 + static_cast<int>(rank) * 128; // this CTA's staged token rows

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        fence_mbarrier_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        if constexpr (kTerms == 2)
            prefetch_tmap(&tmB_lo);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, S::kTmemCols);
        tmem_relinquish_pair();
    }
    pdl_trigger();
    tc_fence_before();
    cluster_sync_all(); // barriers initialised and tensor memory allocated in both CTAs
    tc_fence_after();
    const uint32_t tmem_d = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t full0 = map_to_rank(smem_u32(full), 0); // the leader's full[0]
            auto bar = [&](int s) { return full0 + static_cast<uint32_t>(s) * 8u; };
            auto load_a = [&](int kb, int s) {
                tma_load_2d_pair(smem + s * S::kStageBytes, &tmA, bar(s), kb * 64, f0);
            };
            auto load_b = [&](int kb, int s) {
                uint8_t *st = smem + s * S::kStageBytes;
                tma_load_2d_pair(st + S::kABytes, &tmB, bar(s), kb * 64, tb);
                if constexpr (kTerms == 2)
                    tma_load_2d_pair(st + S::kABytes + S::kBBytes, &tmB_lo, bar(s), kb * 64, tb);
            };
            // weights of the first stages stream before the programmatic-
            // launch wait; activations after it
            const int pre = min(kStages, p.num_kb);
            for (int j = 0; j < pre; ++j) {
                if (leader)
                    mbar_arrive_expect_tx(&full[j], 2u * S::kStageBytes);
                load_a(j, j);
            }
            pdl_wait();
            for (int j = 0; j < pre; ++j)
                load_b(j, j);
            for (int kb = pre; kb < p.num_kb; ++kb) {
                const int s = kb % kStages;
                const uint32_t ph = static_cast<uint32_t>(kb / kStages) & 1u;
                if (!mbar_wait(&empty[s], ph ^ 1u)) {
                    ok = false;
                    break;
                }
                if (leader)
                    mbar_arrive_expect_tx(&full[s], 2u * S::kStageBytes);
                load_a(kb, s);
                load_b(kb, s);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            const uint32_t idesc = idesc_make(p.ab_fmt, 2 * kUmmaM, S::BN);
            for (int kb = 0; kb < p.num_kb; ++kb) {
                const int s = kb % kStages;
                const uint32_t ph = static_cast<uint32_t>(kb / kStages) & 1u;
                if (!mbar_wait(&full[s], ph)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a = smem_u32(smem + s * S::kStageBytes);
                const uint32_t b = a + S::kABytes;
#pragma unroll
                for (int k = 0; k < 4; ++k) { // four 32-byte K steps per 128-byte block
                    const uint64_t ad = sdesc_k128(a + 32 * k);
                    const uint64_t bd = sdesc_k128(b + 32 * k);
                    const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
                    if constexpr (kTerms == 2) {
                        const uint64_t bd_lo = sdesc_k128(b + S::kBBytes + 32 * k);
                        umma_bf16_pair(tmem_d, ad, bd_lo, idesc, acc);
                        umma_bf16_pair(tmem_d, ad, bd, idesc, 1u);
                    } else {
                        umma_bf16_pair(tmem_d, ad, bd, idesc, acc);
                    }
                }
                umma_commit_pair(&empty[s], 0x3);
            }
            // also on the error path: the epilogues of both CTAs wait on it
            umma_commit_pair(accum, 0x3);
        }
    } else {
        pdl_wait(); // the output may still be read by an earlier kernel
        const int q = warp & 3;
        const int col = q * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        const int ntok = max(0, min(S::BN, p.m_tok - t0));
        const int nfeat = min(kUmmaM, p.n_feat - f0);
        if constexpr (has_prepare<Epi>::value)
            if (f0 < p.n_feat)
                epi.prepare(t0, ntok, f0, nfeat, static_cast<int>(threadIdx.x) - 64, epi_scratch);
        if (!mbar_wait_warp(accum, 0))
            ok = false;
        tc_fence_after();
        // [256 tokens][128 features] fp32 over the idle stages (every MMA
        // reading either CTA's stages has completed: accum follows them)
        float *ptile = reinterpret_cast<float *>(smem);
#pragma unroll 1
        for (int c = 0; c < S::BN; c += 64) {
            uint32_t r[4][16];
#pragma unroll
            for (int g = 0; g < 4; ++g)
                tmem_ld_32x16(tmem_d + lane_base + static_cast<uint32_t>(c + 16 * g), r[g]);
            tmem_wait_ld();
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                tmem_reg_fence(r[g]);
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    ptile[(c + 16 * g + i) * kUmmaM + col] = __uint_as_float(r[g][i]);
            }
        }
    }
    __syncthreads(); // the output tile is complete
    if (warp >= 2 && f0 < p.n_feat) { // the last pair may hold one tile past the features
        const int ntok = max(0, min(S::BN, p.m_tok - t0));
        epi(reinterpret_cast<const float *>(smem), t0, ntok, f0, min(kUmmaM, p.n_feat - f0),
            static_cast<int>(threadIdx.x) - 64, epi_scratch);
    }
    if (!ok)
        atomicExch(p.err, 1);
    // neither CTA frees tensor memory or exits while its peer may still use
    // the pair's resources (MMA reads of shared memory, commits)
    tc_fence_before();
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_d, S::kTmemCols);
    }
}

// ------------------------------------------------------------ persistent ---
//
// The same pair tile (256 features x 256 tokens, cta_group::2) on a
// persistent grid: one cluster of 2 per SM pair, each looping over tiles
// w = cluster, cluster + clusters, ... (tile w: feature pair w / ntt, token
// tile w % ntt, so the clusters running at one time share a few weight
// tiles and stream the activations from L2). The K-block ring runs on across
// tiles, and the accumulator is double-buffered in tensor memory (2 x 256
// columns): the MMAs of tile i + 1 run while two groups of four epilogue
// warps drain tile i in alternate 32-token chunks, each through its own
// [32][128] fp32 shared tile (one group alone took ~1.8x the MMA time of a
// K = 2048 tile and set the kernel's pace).
//
// Extra protocol over the one-tile kernel: tmem_empty[b] lives in the
// leader; each epilogue warp of both CTAs arrives on it (remote arrive for
// rank 1) once its last TMEM load of buffer b has completed, and the leader's
// MMA thread waits on it before it reuses buffer b.
// kBN: tokens per pair tile (256, or 192 where it leaves a smaller last
// wave); each CTA stages half of them.
template <int kTerms, int kBN = 256> struct PairPShape {
    static constexpr int BN = kBN;
    static constexpr int kHalf = kBN / 2; // token rows staged per CTA
    static constexpr uint32_t kABytes = kUmmaM * kUmmaKBytes;
    static constexpr uint32_t kBBytes = kHalf * kUmmaKBytes;
    static constexpr uint32_t kStageBytes = kABytes + kTerms * kBBytes;
    static constexpr int kStages = kTerms == 2 ? (kBN == 256 ? 3 : 4) : (kBN == 256 ? 5 : 6);
    static constexpr int kChunk = 32; // tokens per epilogue chunk
    static constexpr uint32_t kChunkBytes = kChunk * kUmmaM * 4;
    // two epilogue groups of four warps (warps 2-5 and 6-9) drain alternate
    // chunks, each through its own chunk tile and scratch
    static constexpr int kEpiGroups = 2;
    static constexpr int kThreads = 64 + 128 * kEpiGroups;
    // two accumulator buffers 256 columns apart
    static constexpr uint32_t kBufCols = 256;
    static constexpr uint32_t kTmemCols = 2 * kBufCols;
    static_assert(kBN % 32 == 0 && kBN <= 256 && kHalf % 8 == 0, "pair tile width");
    static constexpr size_t kEpiScratchBytes = 16u * BN; // per group
    static constexpr size_t kSmemBytes = 1024 + static_cast<size_t>(kStages) * kStageBytes +
                                         kEpiGroups * kChunkBytes + 256 + kEpiGroups * kEpiScratchBytes;
    static_assert(kSmemBytes <= 227u * 1024u, "shared memory per CTA");
    static_assert(kBN >= kEpiGroups * kChunk, "every epilogue group drains a chunk of every tile");
};

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// mbar_wait with cluster-scope acquire (arrivals come from both CTAs).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity) {
    const uint64_t start = global_timer_ns();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i) {
            uint32_t done;
            asm volatile("{\n\t.reg .pred p;\n\t"
                         "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
                         "selp.u32 %0, 1, 0, p;\n\t}"
                         : "=r"(done)
                         : "r"(smem_u32(bar)), "r"(parity)
                         : "memory");
            if (done)
                return true;
        }
        if (global_timer_ns() - start > kWaitTimeoutNs)
            return false;
    }
}

template <typename Epi, int kTerms, int kBN>
__global__ void __launch_bounds__(PairPShape<kTerms, kBN>::kThreads, 1)
    umma_gemm_pair_persistent_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                     const __grid_constant__ CUtensorMap tmB_lo, GemmParams p, int ntt, int ntiles,
                                     Epi epi) {
    using S = PairPShape<kTerms, kBN>;
    constexpr int kStages = S::kStages;
    static_assert(is_tile_epilogue<Epi>::value, "the pair GEMM runs tile epilogues");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // [stages][chunk tile per epilogue group][barriers][scratch per group]
    float *ctile_all = reinterpret_cast<float *>(smem + kStages * S::kStageBytes);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * S::kStageBytes + S::kEpiGroups * S::kChunkBytes);
    uint64_t *empty = full + kStages;
    uint64_t *accum = empty + kStages;    // [2]
    uint64_t *tmem_empty = accum + 2;     // [2], the leader's are used
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tmem_empty + 2);
    uint8_t *scratch_all = smem + kStages * S::kStageBytes + S::kEpiGroups * S::kChunkBytes + 256;

    const int warp = threadIdx.x / kWarpSize;
    const int lane = threadIdx.x % kWarpSize;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int cid = static_cast<int>(blockIdx.x) / 2, ncl = static_cast<int>(gridDim.x) / 2;

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&accum[b], 1);
            mbar_init(&tmem_empty[b], 8 * S::kEpiGroups); // every epilogue warp of both CTAs
        }
        fence_mbarrier_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        if constexpr (kTerms == 2)
            prefetch_tmap(&tmB_lo);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, S::kTmemCols);
        tmem_relinquish_pair();
    }
    pdl_trigger();
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_d = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t full0 = map_to_rank(smem_u32(full), 0);
            auto bar = [&](int s) { return full0 + static_cast<uint32_t>(s) * 8u; };
            int it = 0, armed = 0;
            bool first = true;
            for (int w = cid; w < ntiles && ok; w += ncl) {
                const int f0 = (2 * (w / ntt) + static_cast<int>(rank)) * kUmmaM;
                const int tb = (w % ntt) * S::BN + static_cast<int>(rank) * S::kHalf;
                auto load_a = [&](int kb, int s) {
                    tma_load_2d_pair(smem + s * S::kStageBytes, &tmA, bar(s), kb * 64, f0);
                };
                auto load_b = [&](int kb, int s) {
                    uint8_t *st = smem + s * S::kStageBytes;
                    tma_load_2d_pair(st + S::kABytes, &tmB, bar(s), kb * 64, tb);
                    if constexpr (kTerms == 2)
                        tma_load_2d_pair(st + S::kABytes + S::kBBytes, &tmB_lo, bar(s), kb * 64, tb);
                };
                int kb = 0;
                if (first) {
                    // weights of the first stages stream before the
                    // programmatic-launch wait; activations after it
                    const int pre = min(kStages, p.num_kb);
                    for (; kb < pre; ++kb, ++it) {
                        if (leader)
                            mbar_arrive_expect_tx(&full[it % kStages], 2u * S::kStageBytes);
                        load_a(kb, it % kStages);
                        ++armed;
                    }
                    pdl_wait();
                    for (int j = 0; j < pre; ++j)
                        load_b(j, j % kStages);
                    first = false;
                }
                for (; kb < p.num_kb; ++kb, ++it) {
                    const int s = it % kStages;
                    if (!mbar_wait(&empty[s], (static_cast<uint32_t>(it / kStages) & 1u) ^ 1u)) {
                        ok = false;
                        break;
                    }
                    if (leader)
                        mbar_arrive_expect_tx(&full[s], 2u * S::kStageBytes);
                    load_a(kb, s);
                    load_b(kb, s);
                    ++armed;
                }
            }
            // no copy in flight at exit, on the error path too: the leader's
            // full barriers count both CTAs' copies, so the leader waits
            // (bounded) for the last block armed in every slot, and the
            // final cluster barrier holds the peer until then
            if (leader)
                for (int j = (armed > kStages ? armed - kStages : 0); j < armed; ++j)
                    if (!mbar_wait(&full[j % kStages], static_cast<uint32_t>(j / kStages) & 1u)) {
                        ok = false;
                        break;
                    }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            const uint32_t idesc = idesc_make(p.ab_fmt, 2 * kUmmaM, S::BN);
            int it = 0, lt = 0;
            for (int w = cid; w < ntiles && ok; w += ncl, ++lt) {
                const int buf = lt & 1;
                if (lt >= 2) { // both CTAs' epilogues drained this buffer's previous tile
                    if (!mbar_wait_cluster(&tmem_empty[buf], (static_cast<uint32_t>(lt >> 1) - 1u) & 1u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                }
                const uint32_t dst = tmem_d + static_cast<uint32_t>(buf) * S::kBufCols;
                for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
                    const int s = it % kStages;
                    if (!mbar_wait(&full[s], static_cast<uint32_t>(it / kStages) & 1u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a = smem_u32(smem + s * S::kStageBytes);
                    const uint32_t b = a + S::kABytes;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint64_t ad = sdesc_k128(a + 32 * k);
                        const uint64_t bd = sdesc_k128(b + 32 * k);
                        const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
                        if constexpr (kTerms == 2) {
                            const uint64_t bd_lo = sdesc_k128(b + S::kBBytes + 32 * k);
                            umma_bf16_pair(dst, ad, bd_lo, idesc, acc);
                            umma_bf16_pair(dst, ad, bd, idesc, 1u);
                        } else {
                            umma_bf16_pair(dst, ad, bd, idesc, acc);
                        }
                    }
                    umma_commit_pair(&empty[s], 0x3);
                }
                // also on the error path: the epilogues of both CTAs wait on it
                umma_commit_pair(&accum[buf], 0x3);
            }
            // every MMA issued has completed before tensor memory is freed
            if (lt > 0 && !mbar_wait(&accum[(lt - 1) & 1], static_cast<uint32_t>((lt - 1) >> 1) & 1u))
                ok = false;
        }
    } else {
        pdl_wait(); // the outputs may still be read by an earlier kernel
        // epilogue group g (warps 2-5: 0, 6-9: 1) drains chunks g, g + 2, ...
        // of every tile through its own chunk tile and scratch; its named
        // barrier (epilogue_bar) is 1 + g
        const int eg = (warp - 2) >> 2;
        const int et = (static_cast<int>(threadIdx.x) - 64) & 127; // thread of the group
        float *ctile = ctile_all + eg * (S::kChunk * kUmmaM);
        void *epi_scratch = scratch_all + eg * S::kEpiScratchBytes;
        const int q = warp & 3;
        const int col = q * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        const uint32_t tmem_empty0 = map_to_rank(smem_u32(tmem_empty), 0);
        int lt = 0;
        for (int w = cid; w < ntiles; w += ncl, ++lt) {
            const int buf = lt & 1;
            const int f0 = (2 * (w / ntt) + static_cast<int>(rank)) * kUmmaM;
            const int t0 = (w % ntt) * S::BN;
            const int nfeat = min(kUmmaM, p.n_feat - f0);
            if (!ok || !mbar_wait_warp(&accum[buf], static_cast<uint32_t>(lt >> 1) & 1u))
                ok = false; // after a failed wait, no further wait (warp-uniform)
            tc_fence_after();
#pragma unroll 1
            for (int c = eg * S::kChunk; c < S::BN; c += S::kEpiGroups * S::kChunk) {
                uint32_t r[2][16];
                tmem_ld_32x16(tmem_d + lane_base + static_cast<uint32_t>(buf) * S::kBufCols + static_cast<uint32_t>(c),
                              r[0]);
                tmem_ld_32x16(tmem_d + lane_base + static_cast<uint32_t>(buf) * S::kBufCols +
                                  static_cast<uint32_t>(c + 16),
                              r[1]);
                tmem_wait_ld();
                tmem_reg_fence(r[0]);
                tmem_reg_fence(r[1]);
                if (c + S::kEpiGroups * S::kChunk >= S::BN) { // this warp's last read of the buffer
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive_cluster(tmem_empty0 + static_cast<uint32_t>(buf) * 8u);
                }
#pragma unroll
                for (int i = 0; i < S::kChunk; ++i)
                    ctile[i * kUmmaM + col] = __uint_as_float(r[i >> 4][i & 15]);
                const int ntok = max(0, min(S::kChunk, p.m_tok - (t0 + c)));
                const bool run = nfeat > 0 && ntok > 0; // uniform over the group
                if (run) {
                    if constexpr (has_prepare<Epi>::value)
                        epi.prepare(t0 + c, ntok, f0, nfeat, et, epi_scratch);
                }
                epilogue_bar(); // the chunk (and the scratch) are written
                if (run)
                    epi(ctile, t0 + c, ntok, f0, nfeat, et, epi_scratch);
                epilogue_bar(); // the chunk and the scratch are free again
            }
        }
    }
    if (!ok)
        atomicExch(p.err, 1);
    tc_fence_before();
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_d, S::kTmemCols);
    }
}

template <typename Epi, int kTerms, int kBN> inline int gemm_pair_persistent_prepare() {
    struct Slot {
        int device = -1, clusters = 0;
    };
    static thread_local Slot slot[16];
    int dev = 0;
    OPWORKS_CUDA_CHECK(cudaGetDevice(&dev));
    Slot &sl = slot[dev % 16];
    if (sl.device != dev) {
        auto kernel = umma_gemm_pair_persistent_kernel<Epi, kTerms, kBN>;
        const int smem = static_cast<int>(PairPShape<kTerms, kBN>::kSmemBytes);
        OPWORKS_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(2 * detail::device_facts().sm_count);
        cfg.blockDim = dim3(PairPShape<kTerms, kBN>::kThreads);
        cfg.dynamicSmemBytes = static_cast<size_t>(smem);
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        OPWORKS_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, kernel, &cfg));
        sl.clusters = n > 0 ? n : detail::device_facts().sm_count / 2;
        sl.device = dev;
    }
    return sl.clusters;
}

template <typename Epi, int kTerms> inline void gemm_pair_prepare_kernel() {
    static thread_local int done_device = -1;
    int dev = 0;
    OPWORKS_CUDA_CHECK(cudaGetDevice(&dev));
    if (done_device != dev) {
        OPWORKS_CUDA_CHECK(cudaFuncSetAttribute(umma_gemm_pair_kernel<Epi, kTerms>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(PairShape<kTerms>::kSmemBytes)));
        done_device = dev;
    }
}

// The persistent form for every grid (OPWORKS_PAIR_PERSISTENT=0: the one-tile
// kernel instead).
inline bool gemm_pair_persistent_enabled() {
    static const bool on = [] {
        const char *e = std::getenv("OPWORKS_PAIR_PERSISTENT");
        return !(e && e[0] == '0');
    }();
    return on;
}

// out via `epi` (a tile epilogue): W [n_feat][k] 16-bit, X = Xhi + Xlo
// [m_tok][k] 16-bit (K-major, row strides 16-byte aligned; X.lo == nullptr:
// one activation term). One launch, no K split; grids are pairs of
// 128-feature tiles by 256-token tiles.
template <typename Epi>
inline void gemm_pair_bf16x2(const GemmOperand &W, const GemmOperand &X, int k, cudaStream_t stream, const Epi &epi) {
    static_assert(is_tile_epilogue<Epi>::value, "gemm_pair_bf16x2 runs tile epilogues");
    detail::require(k > 0 && W.rows > 0 && X.rows > 0, "gemm_pair_bf16x2: empty operand");
    GemmParams p{};
    p.out = nullptr;
    p.ldo = 0;
    p.split_stride = 0;
    p.n_feat = W.rows;
    p.m_tok = X.rows;
    p.num_kb = (k + 63) / 64;
    p.splits = 1;
    p.err = device_error_word();
    p.ab_fmt = gemm_ab_format(W, X);
    const CUtensorMap ta = make_tmap_2d(W.hi, true, static_cast<uint64_t>(k), W.rows, W.ld, 64, kUmmaM);
    const CUtensorMap tb = make_tmap_2d(X.hi, true, static_cast<uint64_t>(k), X.rows, X.ld, 64, 128);
    const CUtensorMap tb_lo = X.lo ? make_tmap_2d(X.lo, true, static_cast<uint64_t>(k), X.rows, X.ld, 64, 128) : tb;
    const int ftiles = (W.rows + kUmmaM - 1) / kUmmaM;
    const dim3 grid((ftiles + 1) / 2 * 2, (X.rows + PairShape<2>::BN - 1) / PairShape<2>::BN, 1);
    detail::require(grid.y <= 65535, "gemm_pair_bf16x2: grid exceeds the CUDA limits");
    const int ntiles = static_cast<int>(grid.x / 2 * grid.y);
    if (gemm_pair_persistent_enabled()) {
        // persistent grid (at most one cluster per tile; a grid of one
        // wave still drains with both epilogue groups), with the token tile
        // (256 or 192) that needs fewer token rows of rounds:
        // rounds x width, rounds = ceil(tiles / clusters). One-term tiles
        // of 192 must win by 10%: they move a third more weight bytes per
        // flop (measured at M = 8192: QKV 7% faster, O even, down 13%
        // slower); two-term tiles carry twice the MMA work per byte.
        const int clusters = X.lo ? gemm_pair_persistent_prepare<Epi, 2, 256>()
                                  : gemm_pair_persistent_prepare<Epi, 1, 256>();
        {
            const int pairs = static_cast<int>(grid.x / 2);
            auto cost = [&](int bn) {
                const int64_t tiles = static_cast<int64_t>(pairs) * ((X.rows + bn - 1) / bn);
                return ((tiles + clusters - 1) / clusters) * bn;
            };
            const int bn = (X.lo ? cost(192) < cost(256) : 10 * cost(192) < 9 * cost(256)) ? 192 : 256;
            const int ntt = (X.rows + bn - 1) / bn;
            const int nt = pairs * ntt;
            const CUtensorMap pb = make_tmap_2d(X.hi, true, static_cast<uint64_t>(k), X.rows, X.ld, 64, bn / 2);
            const CUtensorMap pb_lo = X.lo ? make_tmap_2d(X.lo, true, static_cast<uint64_t>(k), X.rows, X.ld, 64, bn / 2)
                                           : pb;
            auto go = [&](auto terms, auto width) {
                constexpr int kT = decltype(terms)::value, kW = decltype(width)::value;
                const int cl = std::min(gemm_pair_persistent_prepare<Epi, kT, kW>(), nt);
                launch_ex_cluster(umma_gemm_pair_persistent_kernel<Epi, kT, kW>, dim3(2 * cl), dim3(2, 1, 1),
                                  dim3(PairPShape<kT, kW>::kThreads), PairPShape<kT, kW>::kSmemBytes, stream, ta, pb,
                                  pb_lo, p, ntt, nt, epi);
            };
            using I1 = std::integral_constant<int, 1>;
            using I2 = std::integral_constant<int, 2>;
            using W192 = std::integral_constant<int, 192>;
            using W256 = std::integral_constant<int, 256>;
            if (X.lo)
                bn == 192 ? go(I2{}, W192{}) : go(I2{}, W256{});
            else
                bn == 192 ? go(I1{}, W192{}) : go(I1{}, W256{});
            return;
        }
    }
    if (X.lo) {
        gemm_pair_prepare_kernel<Epi, 2>();
        launch_ex_cluster(umma_gemm_pair_kernel<Epi, 2>, grid, dim3(2, 1, 1), dim3(192), PairShape<2>::kSmemBytes,
                          stream, ta, tb, tb_lo, p, epi);
    } else {
        gemm_pair_prepare_kernel<Epi, 1>();
        launch_ex_cluster(umma_gemm_pair_kernel<Epi, 1>, grid, dim3(2, 1, 1), dim3(192), PairShape<1>::kSmemBytes,
                          stream, ta, tb, tb_lo, p, epi);
    }
}

} // namespace opworks::sm100

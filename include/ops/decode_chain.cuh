#pragma once

// Persistent decode chain for sm_100a: the projections that follow one
// decode attention kernel (O, gate/up, down, and the next layer's fused QKV)
// as PHASES of one launch instead of four GEMM kernels.
//
// Why: in a decode step every projection is a short weight stream followed
// by a serial chain (the previous kernel's completion, the activation load,
// the MMAs, the split-K reduction, the fused epilogue) that leaves HBM idle
// for several microseconds per kernel. Here one CTA per SM stays resident for
// the whole chain; at the end of a phase each CTA issues the weight loads of
// its first blocks of the NEXT phase into free ring stages before it waits
// for the phase barrier, so the weights of a phase are already in shared
// memory when its activations become ready.
//
// Work split (stream-K): phase p's output is `tiles` 128-feature tiles of
// all (<= 32) tokens, each needing `num_kb` 64-element K blocks. The
// tiles x num_kb units are cut into `active` contiguous ranges, one per CTA
// (CTA c >= active has no work in the phase). A CTA's range covers one or
// more items (a tile's K sub-range). An item accumulates in one of two TMEM
// buffers (32 columns each), so the next item's MMAs overlap this item's
// drain. A tile with one contributor runs its epilogue directly; otherwise
// each contributor stores its partial tile [32][128] fp32 to L2 and the last
// to arrive (per-tile counter) sums the partials in contributor order (K
// order: deterministic) and runs the epilogue.
//
// Phase barrier: every CTA adds 1 to a global counter when its phase work
// (epilogues included) is done; a producer waits for G * (p + 1) before
// loading phase p + 1's activations (bounded wait, %globaltimer). The grid is
// one CTA per SM (the shared-memory footprint admits one), so all CTAs are
// resident; the kernel triggers its dependents only at its start, so no
// later kernel can take an SM from a CTA that has not started. The last CTA
// to exit resets the counters for the next launch.
//
// Roles (192 threads): warp 0 TMA producer, warp 1 TMEM allocator and
// single-thread MMA issuer (16-bit weights x two-term 16-bit activations,
// kind::f16), warps 2-5 the epilogue (the tile epilogues of
// include/ops/llama_kernels.cuh, unchanged).

#include "gemm_sm100.cuh"

namespace opworks::sm100 {

constexpr int kChainPhases = 4;
constexpr int kChainBN = 32; // decode tokens (one N tile)
constexpr int kChainStages = 8;
constexpr uint32_t kChainABytes = kUmmaM * kUmmaKBytes;   // 128 weight rows x 64 elements
constexpr uint32_t kChainBBytes = kChainBN * kUmmaKBytes; // 32 token rows x 64 elements (one term)
constexpr uint32_t kChainStageBytes = kChainABytes + 2 * kChainBBytes;
constexpr uint32_t kChainTileBytes = kChainBN * kUmmaM * 4;
constexpr size_t kChainSmemBytes =
    1024 + static_cast<size_t>(kChainStages) * kChainStageBytes + kChainTileBytes + 512 + kEpiScratchNarrow;
constexpr uint32_t kChainTmemCols = 2 * kChainBN;

// Tensor maps of every phase: weights (A), activations hi (B) and lo (B_lo).
struct ChainMaps {
    CUtensorMap a[kChainPhases];
    CUtensorMap b[kChainPhases];
    CUtensorMap b_lo[kChainPhases];
};

struct ChainPhase {
    int tiles = 0;           // 128-feature output tiles
    int num_kb = 0;          // 64-element K blocks per tile
    int n_feat = 0;          // output features
    int active = 0;          // CTAs sharing the phase's units
    int max_parts = 0;       // most contributors of any tile
    float *partial = nullptr; // [tiles][max_parts][kChainBN][128] fp32
    unsigned *counter = nullptr; // [tiles], zero between launches
};

struct ChainParams {
    ChainPhase ph[kChainPhases];
    int nphases = 0;
    int m_tok = 0;              // token rows (<= kChainBN)
    uint32_t ab_fmt = kFmtBF16; // A/B format of the 16-bit operands
    unsigned *sync = nullptr;   // [2]: phase arrivals, exits; zero between launches
    int *err = nullptr;
};

// The contiguous unit range [lo, hi) of CTA c (units in tile-major order).
__host__ __device__ inline void chain_range(int tiles, int num_kb, int active, int c, int &lo, int &hi) {
    const int64_t units = static_cast<int64_t>(tiles) * num_kb;
    if (c >= active) {
        lo = hi = 0;
        return;
    }
    lo = static_cast<int>(units * c / active);
    hi = static_cast<int>(units * (c + 1) / active);
}

// The CTA whose range holds unit u (the inverse of chain_range).
__host__ __device__ inline int chain_owner(int tiles, int num_kb, int active, int u) {
    const int64_t units = static_cast<int64_t>(tiles) * num_kb;
    return static_cast<int>((static_cast<int64_t>(u + 1) * active - 1) / units);
}

// Most contributors of any tile of a phase (host side, to size the partials).
inline int chain_max_parts(int tiles, int num_kb, int active) {
    int most = 1;
    for (int t = 0; t < tiles; ++t) {
        const int c0 = chain_owner(tiles, num_kb, active, t * num_kb);
        const int c1 = chain_owner(tiles, num_kb, active, (t + 1) * num_kb - 1);
        most = c1 - c0 + 1 > most ? c1 - c0 + 1 : most;
    }
    return most;
}

// A tile epilogue that does nothing (a chain with fewer than four phases).
struct NoTileEpi {
    static constexpr bool kTile = true;
    __device__ __forceinline__ void operator()(const float *, int, int, int, int, int, void *) const {}
};

__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Bounded wait until *cnt >= target (acquire, GPU scope). One thread per
// CTA polls, with a short sleep between reads: without it the idle CTAs'
// reads of the one counter queue up at its L2 slice and slow every access
// of the working CTAs that maps there.
__device__ __forceinline__ bool chain_grid_wait(const unsigned *cnt, unsigned target) {
    const uint64_t start = global_timer_ns();
    while (true) {
        unsigned v;
        asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
        if (v >= target) {
            asm volatile("fence.acq_rel.gpu;" ::: "memory");
            return true;
        }
        if (global_timer_ns() - start > kWaitTimeoutNs)
            return false;
        __nanosleep(128);
    }
}

template <typename Epi>
__device__ __forceinline__ void chain_run_epilogue(const Epi &epi, const float *tile, int ntok, int f0, int nfeat,
                                                   int et, void *scratch) {
    if constexpr (has_prepare<Epi>::value) {
        epi.prepare(0, ntok, f0, nfeat, et, scratch);
        epilogue_bar(); // scratch written by every epilogue thread
    }
    epi(tile, 0, ntok, f0, nfeat, et, scratch);
}

template <typename E0, typename E1, typename E2, typename E3>
__global__ void __launch_bounds__(192, 1)
    decode_chain_kernel(const __grid_constant__ ChainMaps maps, ChainParams p, E0 e0, E1 e1, E2 e2, E3 e3) {
    constexpr int S = kChainStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *tile = reinterpret_cast<float *>(smem + S * kChainStageBytes);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + S * kChainStageBytes + kChainTileBytes);
    uint64_t *empty = full + S;
    uint64_t *accum = empty + S;   // [2] TMEM buffer filled
    uint64_t *drained = accum + 2; // [2] TMEM buffer read out
    uint64_t *phase_go = drained + 2; // the producer passed a phase barrier
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(phase_go + 1);
    int *last_flag = reinterpret_cast<int *>(tmem_slot + 1);
    void *scratch = smem + S * kChainStageBytes + kChainTileBytes + 512;

    const int warp = threadIdx.x / kWarpSize, lane = threadIdx.x % kWarpSize;
    const int G = gridDim.x, c = blockIdx.x;
    if (warp == 0 && lane == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&accum[b], 1);
            mbar_init(&drained[b], 128);
        }
        mbar_init(phase_go, 1);
        fence_mbarrier_init();
        for (int ph = 0; ph < p.nphases; ++ph) {
            prefetch_tmap(&maps.a[ph]);
            prefetch_tmap(&maps.b[ph]);
            prefetch_tmap(&maps.b_lo[ph]);
        }
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kChainTmemCols);
        tmem_relinquish();
    }
    pdl_trigger();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = *tmem_slot;
    bool ok = true;

    if (warp == 0) {
        if (lane == 0) {
            int it = 0;    // ring position over every block this CTA streams
            int armed = 0; // blocks whose copies were issued (ring positions 0 .. armed-1)
            for (int ph = 0; ph < p.nphases && ok; ++ph) {
                const ChainPhase &P = p.ph[ph];
                int lo, hi;
                chain_range(P.tiles, P.num_kb, P.active, c, lo, hi);
                const int n = hi - lo;
                auto stage = [&](int j) { return smem + ((it + j) % S) * kChainStageBytes; };
                auto load_a = [&](int j) {
                    const int u = lo + j;
                    tma_load_2d(stage(j), &maps.a[ph], &full[(it + j) % S], (u % P.num_kb) * 64, (u / P.num_kb) * kUmmaM);
                };
                auto load_b = [&](int j) {
                    const int u = lo + j;
                    uint8_t *st = stage(j);
                    tma_load_2d(st + kChainABytes, &maps.b[ph], &full[(it + j) % S], (u % P.num_kb) * 64, 0);
                    tma_load_2d(st + kChainABytes + kChainBBytes, &maps.b_lo[ph], &full[(it + j) % S],
                                (u % P.num_kb) * 64, 0);
                };
                // weights of the first blocks: independent of earlier phases
                const int pre = n < S ? n : S;
                int issued = 0;
                for (; issued < pre; ++issued) {
                    const int s = (it + issued) % S;
                    if (!mbar_wait(&empty[s], ((static_cast<uint32_t>(it + issued) / S) & 1u) ^ 1u)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], kChainStageBytes);
                    load_a(issued);
                    ++armed;
                }
                // activations: the previous kernel (phase 0) or phase ph - 1 of every CTA
                if (ph == 0) {
                    pdl_wait();
                } else {
                    if (!chain_grid_wait(p.sync, static_cast<unsigned>(G) * ph))
                        ok = false;
                    mbar_arrive(phase_go); // the epilogue warps wait on it
                }
                fence_proxy_async_global();
                for (int j = 0; j < issued; ++j)
                    load_b(j);
                for (int j = pre; j < n && ok; ++j) {
                    const int s = (it + j) % S;
                    if (!mbar_wait(&empty[s], ((static_cast<uint32_t>(it + j) / S) & 1u) ^ 1u)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], kChainStageBytes);
                    load_a(j);
                    load_b(j);
                    ++armed;
                }
                it += n;
            }
            // leave no copy in flight, on the error path too: the last block
            // armed in every slot landed (each wait bounded; after one runs
            // out, no further wait)
            for (int j = (armed > S ? armed - S : 0); j < armed; ++j)
                if (!mbar_wait(&full[j % S], (static_cast<uint32_t>(j) / S) & 1u)) {
                    ok = false;
                    break;
                }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_make(p.ab_fmt, kUmmaM, kChainBN);
            int it = 0, ic = 0;
            for (int ph = 0; ph < p.nphases && ok; ++ph) {
                const ChainPhase &P = p.ph[ph];
                int lo, hi;
                chain_range(P.tiles, P.num_kb, P.active, c, lo, hi);
                for (int u = lo; u < hi && ok;) {
                    const int t = u / P.num_kb, u_end = min(hi, (t + 1) * P.num_kb), u0 = u;
                    const int buf = ic & 1;
                    if (ic >= 2) { // the epilogue read this buffer's previous item out
                        if (!mbar_wait(&drained[buf], (static_cast<uint32_t>(ic >> 1) - 1u) & 1u)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                    }
                    const uint32_t dst = tmem_d + static_cast<uint32_t>(buf * kChainBN);
                    for (; u < u_end; ++u, ++it) {
                        const int s = it % S;
                        if (!mbar_wait(&full[s], (static_cast<uint32_t>(it) / S) & 1u)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a = smem_u32(smem + s * kChainStageBytes);
                        const uint32_t b = a + kChainABytes;
#pragma unroll
                        for (int k = 0; k < 4; ++k) { // four 32-byte K steps per 128-byte block
                            const uint64_t ad = sdesc_k128(a + 32 * k);
                            const uint64_t bd = sdesc_k128(b + 32 * k);
                            const uint64_t bd_lo = sdesc_k128(b + kChainBBytes + 32 * k);
                            umma_bf16(dst, ad, bd_lo, idesc, (u > u0 || k > 0) ? 1u : 0u);
                            umma_bf16(dst, ad, bd, idesc, 1u);
                        }
                        umma_commit(&empty[s]);
                    }
                    umma_commit(&accum[buf]); // also on the error path: the epilogue waits on it
                    ++ic;
                }
            }
            // every MMA issued has completed before TMEM is released (the
            // epilogue skips its waits after a failure)
            if (ic > 0 && !mbar_wait(&accum[(ic - 1) & 1], static_cast<uint32_t>((ic - 1) >> 1) & 1u))
                ok = false;
        }
    } else {
        const int et = threadIdx.x - 64; // epilogue thread 0..127
        const int q = warp & 3;          // TMEM lane quarter of this warp
        const int col = q * 32 + lane;   // feature row of the tile
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        pdl_wait(); // residual rows and step inputs come from earlier kernels
        int ic = 0;
        for (int ph = 0; ph < p.nphases; ++ph) {
            const ChainPhase &P = p.ph[ph];
            if (ph > 0) { // the other CTAs' writes of the previous phase are visible
                // the producer passed the grid barrier of this phase (it
                // alone polls the counter)
                if (!ok || !mbar_wait_warp(phase_go, static_cast<uint32_t>(ph - 1) & 1u))
                    ok = false;
            }
            int lo, hi;
            chain_range(P.tiles, P.num_kb, P.active, c, lo, hi);
            for (int u = lo; u < hi;) {
                const int t = u / P.num_kb, u_end = min(hi, (t + 1) * P.num_kb);
                const int buf = ic & 1;
                if (!ok || !mbar_wait_warp(&accum[buf], static_cast<uint32_t>(ic >> 1) & 1u))
                    ok = false; // a failed wait skips the later ones (warp-uniform)
                tc_fence_after();
                uint32_t r[2][16];
                tmem_ld_32x16(tmem_d + lane_base + static_cast<uint32_t>(buf * kChainBN), r[0]);
                tmem_ld_32x16(tmem_d + lane_base + static_cast<uint32_t>(buf * kChainBN + 16), r[1]);
                tmem_wait_ld();
                tmem_reg_fence(r[0]);
                tmem_reg_fence(r[1]);
                tc_fence_before();
                mbar_arrive(&drained[buf]);
                const int c0 = chain_owner(P.tiles, P.num_kb, P.active, t * P.num_kb);
                const int c1 = chain_owner(P.tiles, P.num_kb, P.active, (t + 1) * P.num_kb - 1);
                const int parts = c1 - c0 + 1;
                bool run = true;
                if (parts == 1) {
#pragma unroll
                    for (int i = 0; i < kChainBN; ++i)
                        tile[i * kUmmaM + col] = __uint_as_float(r[i >> 4][i & 15]);
                    epilogue_bar();
                } else {
                    float *mine = P.partial + (static_cast<int64_t>(t) * P.max_parts + (c - c0)) * kChainBN * kUmmaM;
#pragma unroll
                    for (int i = 0; i < kChainBN; ++i)
                        __stcg(mine + i * kUmmaM + col, __uint_as_float(r[i >> 4][i & 15]));
                    __threadfence();
                    epilogue_bar();
                    if (et == 0)
                        *last_flag = atomicAdd(P.counter + t, 1u) == static_cast<unsigned>(parts - 1);
                    epilogue_bar();
                    run = *last_flag != 0;
                    if (run) {
                        __threadfence(); // every contributor's partial is visible
                        const float *base = P.partial + static_cast<int64_t>(t) * P.max_parts * kChainBN * kUmmaM;
                        float acc[kChainBN];
#pragma unroll
                        for (int i = 0; i < kChainBN; ++i)
                            acc[i] = __ldcg(base + i * kUmmaM + col);
                        for (int j = 1; j < parts; ++j) {
                            const float *pj = base + static_cast<int64_t>(j) * kChainBN * kUmmaM;
#pragma unroll
                            for (int i = 0; i < kChainBN; ++i)
                                acc[i] += __ldcg(pj + i * kUmmaM + col);
                        }
#pragma unroll
                        for (int i = 0; i < kChainBN; ++i)
                            tile[i * kUmmaM + col] = acc[i];
                        if (et == 0)
                            P.counter[t] = 0u; // ready for the next launch
                        epilogue_bar();
                    }
                }
                if (run) {
                    const int f0 = t * kUmmaM, nfeat = min(kUmmaM, P.n_feat - f0);
                    if (ph == 0)
                        chain_run_epilogue(e0, tile, p.m_tok, f0, nfeat, et, scratch);
                    else if (ph == 1)
                        chain_run_epilogue(e1, tile, p.m_tok, f0, nfeat, et, scratch);
                    else if (ph == 2)
                        chain_run_epilogue(e2, tile, p.m_tok, f0, nfeat, et, scratch);
                    else
                        chain_run_epilogue(e3, tile, p.m_tok, f0, nfeat, et, scratch);
                    epilogue_bar(); // the tile and scratch are free again
                }
                u = u_end;
                ++ic;
            }
            // this CTA's share of the phase is written
            epilogue_bar();
            if (et == 0) {
                __threadfence();
                atomicAdd(p.sync, 1u);
            }
        }
    }
    if (!ok)
        atomicExch(p.err, 1);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_d, kChainTmemCols);
    }
    if (threadIdx.x == 0) {
        // the last CTA out re-arms the phase counter (every CTA is past its
        // last wait on it)
        __threadfence();
        if (atomicAdd(p.sync + 1, 1u) == static_cast<unsigned>(G - 1)) {
            atomicExch(p.sync, 0u);
            atomicExch(p.sync + 1, 0u);
        }
    }
}

template <typename E0, typename E1, typename E2, typename E3> inline void decode_chain_prepare() {
    static thread_local int done_device = -1;
    int dev = 0;
    OPWORKS_CUDA_CHECK(cudaGetDevice(&dev));
    if (done_device != dev) {
        OPWORKS_CUDA_CHECK(cudaFuncSetAttribute(decode_chain_kernel<E0, E1, E2, E3>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(kChainSmemBytes)));
        done_device = dev;
    }
}

// One phase of a chain launch: the weight operand W [n_feat][k] and the
// activation operand X = hi + lo [m_tok][k] (16-bit words, both in the
// format of W.f16), with `active` CTAs streaming it.
struct ChainGemm {
    GemmOperand w, x;
    int k = 0;
    int active = 0;
    float *partial = nullptr;
    unsigned *counter = nullptr;
};

// Launches the chain: grid = one CTA per SM (`ctas`), phases in order.
template <typename E0, typename E1, typename E2, typename E3>
inline void decode_chain_launch(const ChainGemm *g, int nphases, int ctas, unsigned *sync, cudaStream_t stream,
                                const E0 &e0, const E1 &e1, const E2 &e2, const E3 &e3) {
    detail::require(nphases >= 1 && nphases <= kChainPhases, "decode chain: 1 to 4 phases");
    ChainMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    ChainParams p;
    p.nphases = nphases;
    p.sync = sync;
    p.err = device_error_word();
    p.m_tok = g[0].x.rows;
    p.ab_fmt = gemm_ab_format(g[0].w, g[0].x);
    detail::require(p.m_tok >= 1 && p.m_tok <= kChainBN, "decode chain: 1 to 32 token rows");
    for (int ph = 0; ph < nphases; ++ph) {
        const ChainGemm &G = g[ph];
        detail::require(G.x.rows == p.m_tok && G.x.lo != nullptr && G.k > 0 && G.k % 64 == 0,
                        "decode chain: two-term operands of the same rows and K a multiple of 64");
        detail::require(gemm_ab_format(G.w, G.x) == p.ab_fmt, "decode chain: one 16-bit format");
        ChainPhase &P = p.ph[ph];
        P.tiles = (G.w.rows + kUmmaM - 1) / kUmmaM;
        P.num_kb = G.k / 64;
        P.n_feat = G.w.rows;
        P.active = G.active > 0 && G.active < ctas ? G.active : ctas;
        P.max_parts = chain_max_parts(P.tiles, P.num_kb, P.active);
        P.partial = G.partial;
        P.counter = G.counter;
        detail::require(P.max_parts == 1 || (P.partial != nullptr && P.counter != nullptr),
                        "decode chain: split tiles need a partial buffer and counters");
        maps.a[ph] = make_tmap_2d(G.w.hi, true, static_cast<uint64_t>(G.k), G.w.rows, G.w.ld, 64, kUmmaM);
        maps.b[ph] = make_tmap_2d(G.x.hi, true, static_cast<uint64_t>(G.k), G.x.rows, G.x.ld, 64, kChainBN);
        maps.b_lo[ph] = make_tmap_2d(G.x.lo, true, static_cast<uint64_t>(G.k), G.x.rows, G.x.ld, 64, kChainBN);
    }
    decode_chain_prepare<E0, E1, E2, E3>();
    launch_ex(decode_chain_kernel<E0, E1, E2, E3>, dim3(ctas), dim3(192), kChainSmemBytes, stream, maps, p, e0, e1, e2,
              e3);
}

} // namespace opworks::sm100

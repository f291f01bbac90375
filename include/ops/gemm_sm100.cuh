#pragma once

// Warp-specialised tcgen05 GEMM for sm_100a ("TN": both operands K-major).
//
//   out[split][tok][feat] = epi( sum_{k in split} A[feat][k] * B[tok][k] )
//
// A is the "feature" operand (weights [out_features, in_features] in the HF
// layout, or B^T of ops::mat_mul) and fills the 128 TMEM lanes; B is the
// "token" operand (activations [tokens, in_features]) and fills BN TMEM
// columns. Putting features on lanes makes the epilogue store coalesced:
// for each token column the 32 lanes of a warp write 32 consecutive floats.
// Decode (few tokens) therefore runs the same kernel with a narrow N tile
// (BN = 32) and split-K across CTAs; prefill uses BN = 256.
//
// Roles (192 threads): warp 0 = TMA producer (one elected lane), warp 1 =
// TMEM allocator + single-thread MMA issuer, warps 2-5 = epilogue (warp w may
// only read TMEM lanes 32*(w%4)..+31). A STAGES-deep ring of smem stages is
// guarded by full/empty mbarriers; tcgen05.commit releases a stage when the
// MMAs reading it complete, and a final commit hands the accumulator to the
// epilogue.
//
// Precision kinds:
//   kBF16   one kind::f16 MMA per 16-wide K step (16-bit x 16-bit -> fp32)
//   kBF16x2 16-bit weights times a two-term 16-bit activation (x = hi + lo,
//           lo = r(x - hi)): two kind::f16 MMAs per K step, so activations
//           keep about twice the format's mantissa bits while the weight
//           stream stays 2 bytes/element
//   The 16-bit format of both kinds is bf16 or fp16 (GemmOperand::f16, the
//   instruction descriptor's A/B format at run time); the kind names keep
//   the bf16 spelling of their first format.
//   kTF32x3 split-precision fp32: operands pre-split into tf32 hi/lo parts,
//           three kind::tf32 MMAs per K step (hi*hi + hi*lo + lo*hi) give
//           ~fp32 accuracy on the tensor cores.

#include <type_traits>
#include <cooperative_groups.h>
#include <cuda_bf16.h>

#include "detail/operand_prep.cuh"
#include "detail/sm100.cuh"

namespace opworks::sm100 {

// kTF32x3S: the split-precision GEMM on raw fp32 operands — the A (feature)
// operand MN-major straight from a row-major [contraction][features] matrix,
// the B (token) operand K-major — split into tf32 hi / lo in shared memory by
// four converter warps (no pre-pass, no scratch).
enum class GemmKind { kBF16, kTF32x3, kBF16x2, kTF32x3S };

struct GemmParams {
    float *out;           // [splits][m_tok][ldo]
    int64_t ldo;          // row stride of out (elements)
    int64_t split_stride; // elements between split slices
    int n_feat;           // rows of A
    int m_tok;            // rows of B
    int num_kb;           // K blocks of 128 bytes
    int splits;
    int *err;             // error word (bounded wait ran out)
    // optional: bytes the next kernel will stream (its weights), pulled into
    // L2 while this GEMM runs; every CTA prefetches its share, either at its
    // start (l2_prefetch_tail false) or once its producer has issued its own
    // last load, so the prefetch fills the HBM time the MMA drain and the
    // epilogue leave idle instead of competing with this GEMM's stream
    const uint8_t *l2_prefetch = nullptr;
    uint64_t l2_prefetch_bytes = 0;
    bool l2_prefetch_tail = false;
    // tile epilogues: CTAs per cluster (0 = splits). With splits = G x
    // cluster, each of the G clusters of a tile reduces its partials through
    // distributed shared memory, stores its row slices to red_ws, and the
    // last cluster to arrive at red_cnt[tile][slice] sums the G slices in
    // group order and runs the epilogue (counters are zero between launches:
    // the last arrival resets its own)
    int cluster = 0;
    float *red_ws = nullptr;
    unsigned int *red_cnt = nullptr;
    // A/B format of the 16-bit kinds (kFmtBF16 or kFmtF16; both operands share it)
    uint32_t ab_fmt = kFmtBF16;
};

// Workspace of grouped split-K tile epilogues (GemmParams::red_ws / red_cnt).
struct SplitGroupWorkspace {
    float *partials = nullptr;        // [tiles][groups][BN][128] fp32
    size_t floats = 0;
    unsigned int *counters = nullptr; // [tiles][cluster], zero-initialised
    int max_counters = 0;
};

struct Identity {
    __device__ __forceinline__ float operator()(float x) const { return x; }
};

// Epilogues are unary `float(float)` functors (the ops::mat_mul contract),
// position-aware `float(float, int tok, int feat)` functors (bias), or tile
// epilogues (a `kTile` member), which see finished fp32 tiles in shared
// memory: the K splits of a tile then run as one thread-block cluster, each
// CTA keeps its partial tile in shared memory, and after a cluster barrier
// CTA r sums rows [r*ceil(BN/S), ...) of all S partials through distributed
// shared memory in rank order (a fixed order: deterministic) and hands them
// to the epilogue,
//   epi(tile [ntok][128], tok0, ntok, f0, nfeat, tid in [0, 128)),
// so split-K needs no global workspace and no separate reduction kernel.
//
// A tile epilogue may also define
//   prepare(tok0, ntok, f0, nfeat, tid, void *scratch)
// which runs on the epilogue threads while the main loop streams, before the
// accumulator is final (metadata loads such as token positions, residual rows),
// with shared scratch (kEpiScratchNarrow bytes for BN <= 64, else at least
// max(2 KB, 16 bytes per token row)) that stays valid for operator().
template <typename Epi, typename = void> struct is_tile_epilogue : std::false_type {};
template <typename Epi> struct is_tile_epilogue<Epi, std::void_t<decltype(Epi::kTile)>> : std::true_type {};
template <typename Epi, typename = void> struct has_prepare : std::false_type {};
template <typename Epi>
struct has_prepare<Epi, std::void_t<decltype(std::declval<const Epi &>().prepare(0, 0, 0, 0, 0, nullptr))>>
    : std::true_type {};
constexpr size_t kEpiScratchNarrow = 8192; // epilogue scratch bytes of BN <= 64 tiles
constexpr int kMaxClusterSplits = 8;           // portable cluster size
constexpr int kMaxClusterSplitsNonPortable = 16; // with the non-portable opt-in

// Named barrier of the 128 threads of one epilogue group: warps 2-5 are group
// 0 (barrier 1), warps 6-9 group 1 (barrier 2; the persistent two-SM GEMM
// runs two epilogue groups on alternating chunks). Constant barrier ids (a
// warp-uniform branch), so kernels reserve only the barriers they name.
__device__ __forceinline__ void epilogue_bar() {
    if (threadIdx.x < 192)
        asm volatile("bar.sync 1, 128;" ::: "memory");
    else
        asm volatile("bar.sync 2, 128;" ::: "memory");
}
// split cluster barrier: arrive (release this CTA's shared-memory writes) and
// wait (acquire the peers'); every thread of every CTA takes both
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
template <typename Epi>
__device__ __forceinline__ float apply_epilogue(const Epi &epi, float v, int tok, int feat) {
    if constexpr (std::is_invocable_v<const Epi &, float, int, int>)
        return epi(v, tok, feat);
    else
        return epi(v);
}

// Split-K reduction of a cluster's partial tiles [tokens][128] through
// distributed shared memory: this CTA's token slice [tl0, tl1) summed over
// the kN CTAs in rank order (0 + p0 + p1 + ..., the order of the generic
// loop) into rtile. Clusters of 2 and 4: several items per thread are
// loaded together so that eight remote loads are in flight (clusters of 8
// already have eight per item; the batched form measured slower there).
template <int kN, typename Cluster>
__device__ __forceinline__ void cluster_reduce_slice(Cluster &cluster, const float *ptile, float *rtile, int tl0,
                                                     int tl1, int et) {
    constexpr int kItems = kN >= 8 ? 1 : 8 / kN;
    constexpr int kF4 = kUmmaM / 4; // float4 per token row
    const int n = (tl1 - tl0) * kF4;
    const float4 *src[kN];
#pragma unroll
    for (int r = 0; r < kN; ++r)
        src[r] = reinterpret_cast<const float4 *>(cluster.map_shared_rank(ptile, r));
    for (int i0 = et; i0 < n; i0 += 128 * kItems) {
        float4 v[kItems][kN];
#pragma unroll
        for (int i = 0; i < kItems; ++i) {
            const int idx = i0 + i * 128;
            const int t = tl0 + idx / kF4, c4 = idx % kF4;
#pragma unroll
            for (int r = 0; r < kN; ++r)
                if (idx < n)
                    v[i][r] = src[r][t * kF4 + c4];
        }
#pragma unroll
        for (int i = 0; i < kItems; ++i) {
            const int idx = i0 + i * 128;
            if (idx < n) {
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int r = 0; r < kN; ++r) {
                    acc.x += v[i][r].x;
                    acc.y += v[i][r].y;
                    acc.z += v[i][r].z;
                    acc.w += v[i][r].w;
                }
                reinterpret_cast<float4 *>(rtile)[idx] = acc;
            }
        }
    }
}

template <GemmKind kKind, int BN> struct GemmShape {
    static constexpr bool kSplit3 = kKind == GemmKind::kTF32x3 || kKind == GemmKind::kTF32x3S;
    // hi / lo halves made in shared memory by warps 6-9 (kTF32x3S)
    static constexpr bool kConvert = kKind == GemmKind::kTF32x3S;
    static constexpr int kThreads = kConvert ? 320 : 192;
    static constexpr bool kSplitB = kKind == GemmKind::kBF16x2; // B_lo tile, A shared
    static constexpr uint32_t kABytes = kUmmaM * kUmmaKBytes;
    static constexpr uint32_t kBBytes = BN * kUmmaKBytes;
    static constexpr uint32_t kStageBytes =
        kSplit3 ? 2u * (kABytes + kBBytes) : (kSplitB ? kABytes + 2u * kBBytes : kABytes + kBBytes);
    // bytes the TMA brings per stage (kConvert: the hi halves only)
    static constexpr uint32_t kLoadBytes = kConvert ? kABytes + kBBytes : kStageBytes;
    // narrow token tiles (decode) run two CTAs per SM: the hardware keeps two
    // tensor-memory CTAs of this size resident (the occupancy calculator
    // reports one for any kernel that allocates tensor memory), and a second
    // CTA overlaps one CTA's prologue / epilogue with the other's stream
    static constexpr int kCtasPerSm = BN <= 64 ? 2 : 1;
    static constexpr int kBudget = kCtasPerSm == 2 ? 98 * 1024 : 192 * 1024;
    static constexpr int kStagesRaw = kBudget / static_cast<int>(kStageBytes);
    static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
    static constexpr int kKElems = kSplit3 ? 32 : 64; // elements per 128-byte K block
    // split-precision path: two accumulators (double-buffered promotion)
    static constexpr uint32_t kTmemCols = (BN < 32 ? 32 : BN) * (kSplit3 ? 2u : 1u);
    // K blocks accumulated in TMEM before the epilogue promotes the partial
    // sum into fp32 registers (split-precision path only)
    static constexpr int kPromoteKb = 2;
    // tile epilogue scratch (prepare() metadata, per-token reductions, rows
    // preloaded during the main loop): 8 KB for narrow decode tiles (two
    // CTAs still fit an SM), else 16 bytes per token row, at least 2 KB
    static constexpr size_t kEpiScratchBytes = BN <= 64 ? kEpiScratchNarrow : (16u * BN > 2048u ? 16u * BN : 2048u);
    static constexpr size_t kSmemBytes = 1024 + static_cast<size_t>(kStages) * kStageBytes + 256 + kEpiScratchBytes;
    static_assert(kStages >= 2, "GEMM tile does not fit two pipeline stages");
    static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "token tiles are multiples of 32 in [32, 256] (UMMA N)");
};

template <GemmKind kKind, int BN, typename Epi>
__global__ void __launch_bounds__(GemmShape<kKind, BN>::kThreads, GemmShape<kKind, BN>::kCtasPerSm)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmA_lo, const __grid_constant__ CUtensorMap tmB_lo,
                     GemmParams p, Epi epi) {
    using S = GemmShape<kKind, BN>;
    constexpr int kStages = S::kStages;
    constexpr bool kTileEpi = is_tile_epilogue<Epi>::value;
    // the partial tile [BN][128] fp32 (and, for split K, the reduced slice)
    // reuse the pipeline stages
    static_assert(!kTileEpi || BN * kUmmaM * 4u <= kStages * S::kStageBytes,
                  "tile epilogue: the partial tile must fit in the pipeline stages");
    constexpr bool kFitsReduce = 2u * BN * kUmmaM * 4u <= kStages * S::kStageBytes;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * S::kStageBytes);
    uint64_t *empty = full + kStages;
    uint64_t *accum = empty + kStages;
    uint64_t *ready = accum + 1;   // [2] promotion buffers filled (split path)
    uint64_t *drained = ready + 2; // [2] promotion buffers read (split path)
    uint64_t *conv = drained + 2;  // [kStages] stage split into hi / lo (kConvert)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(conv + kStages);
    static_assert((3 * kStages + 5) * 8 + 4 <= 256, "barriers fit their 256-byte slot");
    void *epi_scratch = smem + kStages * S::kStageBytes + 256;

    const int warp = threadIdx.x / kWarpSize;
    const int lane = threadIdx.x % kWarpSize;
    const int f0 = blockIdx.x * kUmmaM;
    const int t0 = blockIdx.y * BN;
    const int split = blockIdx.z;
    const int kb_begin = static_cast<int>(static_cast<int64_t>(p.num_kb) * split / p.splits);
    const int kb_end = static_cast<int>(static_cast<int64_t>(p.num_kb) * (split + 1) / p.splits);

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        mbar_init(&ready[0], 1);
        mbar_init(&ready[1], 1);
        mbar_init(&drained[0], 128);
        mbar_init(&drained[1], 128);
        if constexpr (S::kConvert)
            for (int s = 0; s < kStages; ++s)
                mbar_init(&conv[s], 4); // one arrival per converter warp
        fence_mbarrier_init();
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        if constexpr (S::kSplit3) {
            prefetch_tmap(&tmA_lo);
            prefetch_tmap(&tmB_lo);
        }
        if constexpr (S::kSplitB)
            prefetch_tmap(&tmB_lo);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, S::kTmemCols);
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
            // A (weights) of the first stages does not depend on earlier
            // kernels: it streams in while the previous kernel drains; B
            // (activations) follows the programmatic-launch wait
            auto load_a = [&](int kb, int s) {
                uint8_t *st = smem + s * S::kStageBytes;
                const int kc = kb * S::kKElems;
                if constexpr (S::kConvert) {
                    // MN-major: four 32-feature x 32-contraction boxes
                    // ([32 contraction rows][32 features] each, 4 KB apart)
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        tma_load_2d(st + j * 4096, &tmA, &full[s], f0 + 32 * j, kc);
                } else {
                    tma_load_2d(st, &tmA, &full[s], kc, f0);
                    if constexpr (S::kSplit3)
                        tma_load_2d(st + S::kABytes + S::kBBytes, &tmA_lo, &full[s], kc, f0);
                }
            };
            auto load_b = [&](int kb, int s) {
                uint8_t *st = smem + s * S::kStageBytes;
                const int kc = kb * S::kKElems;
                tma_load_2d(st + S::kABytes, &tmB, &full[s], kc, t0);
                if constexpr (S::kSplit3 && !S::kConvert)
                    tma_load_2d(st + 2 * S::kABytes + S::kBBytes, &tmB_lo, &full[s], kc, t0);
                if constexpr (S::kSplitB)
                    tma_load_2d(st + S::kABytes + S::kBBytes, &tmB_lo, &full[s], kc, t0);
            };
            const int pre = min(kStages, kb_end - kb_begin);
            for (int j = 0; j < pre; ++j) {
                mbar_arrive_expect_tx(&full[j], S::kLoadBytes);
                load_a(kb_begin + j, j);
            }
            // this CTA's share of the next kernel's stream, in 16-byte
            // multiples and chunks of at most 64 KB
            auto prefetch_next = [&]() {
                const uint64_t ctas = static_cast<uint64_t>(gridDim.x) * gridDim.y * gridDim.z;
                const uint64_t cta = (static_cast<uint64_t>(blockIdx.z) * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
                const uint64_t share = ((p.l2_prefetch_bytes + ctas - 1) / ctas + 15) & ~uint64_t(15);
                const uint64_t lo = min(p.l2_prefetch_bytes, cta * share);
                const uint64_t hi = min(p.l2_prefetch_bytes, lo + share);
                for (uint64_t o = lo; o < hi; o += 65536)
                    bulk_prefetch_l2(p.l2_prefetch + o, static_cast<uint32_t>(hi - o < 65536 ? hi - o : 65536));
            };
            if (p.l2_prefetch_bytes > 0 && !p.l2_prefetch_tail)
                prefetch_next();
            pdl_wait();
            for (int j = 0; j < pre; ++j)
                load_b(kb_begin + j, j);
            int it = pre;
            for (int kb = kb_begin + pre; kb < kb_end; ++kb, ++it) {
                const int s = it % kStages;
                const uint32_t ph = static_cast<uint32_t>(it / kStages) & 1u;
                if (!mbar_wait(&empty[s], ph ^ 1u)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&full[s], S::kLoadBytes);
                load_a(kb, s);
                load_b(kb, s);
            }
            if (ok && p.l2_prefetch_bytes > 0 && p.l2_prefetch_tail)
                prefetch_next();
            // never leave the CTA with copies in flight: the last issued
            // phase of every slot must have landed (returns at once when the
            // MMA warp already consumed it)
            for (int j = (it > kStages ? it - kStages : 0); j < it; ++j)
                if (!mbar_wait(&full[j % kStages], static_cast<uint32_t>(j / kStages) & 1u))
                    ok = false;
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // kConvert: A (features) MN-major (instruction descriptor bit 15)
            const uint32_t idesc =
                idesc_make(S::kSplit3 ? kFmtTF32 : p.ab_fmt, kUmmaM, BN) | (S::kConvert ? (1u << 15) : 0u);
            int it = 0;
            for (int kb = kb_begin; kb < kb_end; ++kb, ++it) {
                const int s = it % kStages;
                const uint32_t ph = static_cast<uint32_t>(it / kStages) & 1u;
                // split path: group of kPromoteKb blocks into TMEM buffer group & 1
                const int group = it / S::kPromoteKb;
                const bool first_in_group = !S::kSplit3 || it % S::kPromoteKb == 0;
                const uint32_t dst = S::kSplit3 ? tmem_d + static_cast<uint32_t>((group & 1) * BN) : tmem_d;
                if (S::kSplit3 && first_in_group && group >= 2) {
                    if (!mbar_wait(&drained[group & 1], static_cast<uint32_t>((group - 2) >> 1) & 1u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                }
                // kConvert: the stage is also split into hi / lo
                if (!mbar_wait(S::kConvert ? &conv[s] : &full[s], ph)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a = smem_u32(smem + s * S::kStageBytes);
                const uint32_t b = a + S::kABytes;
                // MN-major A: a K step is 8 contraction rows (1 KB) of the four
                // 4 KB feature boxes; atoms 4 rows x 128 bytes
                auto a_desc = [&](uint32_t base, int k) {
                    return S::kConvert ? sdesc_mn128_32b(base + 1024u * static_cast<uint32_t>(k), 4096u, 512u)
                                       : sdesc_k128(base + 32u * static_cast<uint32_t>(k));
                };
#pragma unroll
                for (int k = 0; k < 4; ++k) { // four 32-byte K steps per 128-byte block
                    const uint64_t ad = a_desc(a, k);
                    const uint64_t bd = sdesc_k128(b + 32 * k);
                    if constexpr (S::kSplit3) {
                        const uint32_t acc = (first_in_group && k == 0) ? 0u : 1u;
                        const uint64_t ad_lo = a_desc(a + S::kABytes + S::kBBytes, k);
                        const uint64_t bd_lo = sdesc_k128(a + 2 * S::kABytes + S::kBBytes + 32 * k);
                        umma_tf32(dst, ad, bd_lo, idesc, acc);
                        umma_tf32(dst, ad_lo, bd, idesc, 1u);
                        umma_tf32(dst, ad, bd, idesc, 1u);
                    } else if constexpr (S::kSplitB) {
                        const uint32_t acc = (kb > kb_begin || k > 0) ? 1u : 0u;
                        const uint64_t bd_lo = sdesc_k128(b + S::kBBytes + 32 * k);
                        umma_bf16(dst, ad, bd_lo, idesc, acc);
                        umma_bf16(dst, ad, bd, idesc, 1u);
                    } else {
                        const uint32_t acc = (kb > kb_begin || k > 0) ? 1u : 0u;
                        umma_bf16(dst, ad, bd, idesc, acc);
                    }
                }
                umma_commit(&empty[s]);
                if (S::kSplit3 && (it % S::kPromoteKb == S::kPromoteKb - 1 || kb == kb_end - 1))
                    umma_commit(&ready[group & 1]);
            }
            if (!S::kSplit3)
                umma_commit(accum);
        }
    } else if (warp < 6) {
        pdl_wait(); // the output may still be read by an earlier kernel
        const int q = warp & 3; // TMEM lane quarter this warp may access
        const int feat = f0 + q * 32 + lane;
        float *out = p.out + static_cast<int64_t>(split) * p.split_stride;
        const bool feat_ok = feat < p.n_feat;
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        // tile epilogues: the partial tile goes to shared memory [BN][128]
        // (the pipeline stages are idle once the accumulator is final)
        float *ptile = reinterpret_cast<float *>(smem);
        const int col = q * 32 + lane;
        if constexpr (kTileEpi && has_prepare<Epi>::value) {
            const bool sliced = p.splits > 1; // this CTA's row slice of the cluster's tile
            const int csz = p.cluster > 0 ? p.cluster : p.splits;
            const int per = (BN + csz - 1) / csz;
            const int tb = sliced ? min(BN, (split % csz) * per) : 0;
            const int nt = sliced ? min(BN, tb + per) - tb : BN;
            epi.prepare(t0 + tb, max(0, min(nt, p.m_tok - (t0 + tb))), f0, min(kUmmaM, p.n_feat - f0),
                        static_cast<int>(threadIdx.x) - 64, epi_scratch);
        }
        if constexpr (S::kSplit3) {
            // promote each group's TMEM partial into fp32 registers: the
            // tensor core's accumulator only ever holds kPromoteKb blocks
            float acc[BN];
#pragma unroll
            for (int i = 0; i < BN; ++i)
                acc[i] = 0.f;
            const int ngroups = (kb_end - kb_begin + S::kPromoteKb - 1) / S::kPromoteKb;
            for (int g = 0; g < ngroups; ++g) {
                if (!mbar_wait_warp(&ready[g & 1], static_cast<uint32_t>(g >> 1) & 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < BN; c += 16) {
                    uint32_t r[16];
                    tmem_ld_32x16(tmem_d + lane_base + static_cast<uint32_t>((g & 1) * BN + c), r);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        acc[c + i] += __uint_as_float(r[i]);
                }
                tc_fence_before();
                mbar_arrive(&drained[g & 1]);
            }
#pragma unroll
            for (int i = 0; i < BN; ++i) {
                const int tok = t0 + i;
                if constexpr (kTileEpi)
                    ptile[i * kUmmaM + col] = acc[i];
                else if (feat_ok && tok < p.m_tok)
                    out[static_cast<int64_t>(tok) * p.ldo + feat] = apply_epilogue(epi, acc[i], tok, feat);
            }
        } else {
        if (!mbar_wait_warp(accum, 0)) {
            ok = false;
        }
        tc_fence_after();
        // two 16-column loads per wait (BN is a multiple of 32)
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
            uint32_t r[2][16];
            tmem_ld_32x16(tmem_d + lane_base + static_cast<uint32_t>(c), r[0]);
            tmem_ld_32x16(tmem_d + lane_base + static_cast<uint32_t>(c + 16), r[1]);
            tmem_wait_ld();
            tmem_reg_fence(r[0]);
            tmem_reg_fence(r[1]);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int tok = t0 + c + i;
                const float v = __uint_as_float(r[i >> 4][i & 15]);
                if constexpr (kTileEpi)
                    ptile[(c + i) * kUmmaM + col] = v;
                else if (feat_ok && tok < p.m_tok)
                    out[static_cast<int64_t>(tok) * p.ldo + feat] = apply_epilogue(epi, v, tok, feat);
            }
        }
        }
    } else if constexpr (S::kConvert) {
        // warps 6-9: each landed stage's fp32 values x stay in place as the
        // hi halves (the tensor cores read a 32-bit operand as tf32 by
        // dropping its 13 low mantissa bits) and lo = x - that truncation
        // (exact in fp32) goes to the lo half of the stage; the layout does
        // not matter (the same element-wise map over both swizzled tiles).
        // Infinities and NaNs give a NaN lo, as in the pre-pass split.
        const int ct = threadIdx.x - 192;
        int it = 0;
        for (int kb = kb_begin; kb < kb_end; ++kb, ++it) {
            const int s = it % kStages;
            if (!mbar_wait_warp(&full[s], static_cast<uint32_t>(it / kStages) & 1u)) {
                ok = false;
                break;
            }
            const float4 *hi = reinterpret_cast<const float4 *>(smem + s * S::kStageBytes);
            float4 *lo = reinterpret_cast<float4 *>(smem + s * S::kStageBytes + S::kABytes + S::kBBytes);
            constexpr int kVecs = static_cast<int>((S::kABytes + S::kBBytes) / 16);
            auto low = [](float x) { return x - __uint_as_float(__float_as_uint(x) & 0xffffe000u); };
#pragma unroll 4
            for (int i = ct; i < kVecs; i += 128) {
                const float4 x = hi[i];
                lo[i] = make_float4(low(x.x), low(x.y), low(x.z), low(x.w));
            }
            fence_proxy_async_smem(); // generic writes, read next by the tensor cores
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&conv[s]);
        }
    }
    if constexpr (kTileEpi) {
        // every thread of every CTA of the cluster takes both barriers, on
        // the error path too
        namespace cg = cooperative_groups;
        // nsplit = CTAs of this tile's cluster (the host splits only shapes
        // that fit); groups = clusters per tile
        const int nsplit = kFitsReduce ? (p.splits > 1 && p.cluster > 0 ? p.cluster : p.splits) : 1;
        const int groups = kFitsReduce ? p.splits / nsplit : 1;
        const int rank = split % nsplit, group = split / nsplit;
        float *ptile = reinterpret_cast<float *>(smem);
        float *rtile = ptile + BN * kUmmaM;
        const int per = (BN + nsplit - 1) / nsplit;
        const int tl0 = min(BN, rank * per), tl1 = min(BN, tl0 + per);
        __shared__ int run_epilogue;
        if (nsplit > 1) {
            cluster_arrive(); // this CTA's partial tile is published
            cluster_wait();   // and every peer's
        } else {
            __syncthreads();
        }
        const float *src = ptile;
        if (nsplit > 1) {
            if (warp >= 2 && warp < 6) {
                const int et = threadIdx.x - 64;
                cg::cluster_group cluster = cg::this_cluster();
                switch (nsplit) {
                case 2: cluster_reduce_slice<2>(cluster, ptile, rtile, tl0, tl1, et); break;
                case 4: cluster_reduce_slice<4>(cluster, ptile, rtile, tl0, tl1, et); break;
                default:
                    // other cluster sizes: one item at a time, eight remote
                    // loads in flight, summed in rank order
                    for (int idx = et; idx < (tl1 - tl0) * (kUmmaM / 4); idx += 128) {
                        const int t = tl0 + idx / (kUmmaM / 4), c4 = idx % (kUmmaM / 4);
                        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                        for (int r0 = 0; r0 < nsplit; r0 += 8) {
                            float4 v[8];
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                if (r0 + j < nsplit)
                                    v[j] = reinterpret_cast<const float4 *>(
                                        cluster.map_shared_rank(ptile, r0 + j))[t * (kUmmaM / 4) + c4];
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                if (r0 + j < nsplit) {
                                    acc.x += v[j].x;
                                    acc.y += v[j].y;
                                    acc.z += v[j].z;
                                    acc.w += v[j].w;
                                }
                        }
                        reinterpret_cast<float4 *>(rtile)[idx] = acc;
                    }
                    break;
                }
                epilogue_bar();
                if (groups > 1) {
                    // across the tile's clusters: publish this slice, count
                    // arrivals; the last group's CTA sums the slices in group
                    // order (deterministic) and runs the epilogue
                    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
                    const int nf4 = (tl1 - tl0) * (kUmmaM / 4);
                    float4 *ws = reinterpret_cast<float4 *>(p.red_ws) +
                                 (static_cast<int64_t>(tile) * groups * BN + tl0) * (kUmmaM / 4);
                    const int64_t gstride = static_cast<int64_t>(BN) * (kUmmaM / 4);
                    for (int i = et; i < nf4; i += 128)
                        __stcg(ws + group * gstride + i, reinterpret_cast<const float4 *>(rtile)[i]);
                    __threadfence();
                    epilogue_bar();
                    if (et == 0) {
                        unsigned int *cnt = p.red_cnt + tile * nsplit + rank;
                        const bool last = atomicAdd(cnt, 1u) == static_cast<unsigned>(groups - 1);
                        if (last)
                            *cnt = 0u; // ready for the next launch
                        run_epilogue = last;
                    }
                    epilogue_bar();
                    if (run_epilogue) {
                        __threadfence(); // the other groups' slices are visible
                        for (int i = et; i < nf4; i += 128) {
                            float4 acc = __ldcg(ws + i);
                            for (int g = 1; g < groups; ++g) {
                                const float4 v = __ldcg(ws + g * gstride + i);
                                acc.x += v.x;
                                acc.y += v.y;
                                acc.z += v.z;
                                acc.w += v.w;
                            }
                            reinterpret_cast<float4 *>(rtile)[i] = acc;
                        }
                        epilogue_bar();
                    }
                }
            }
            src = rtile;
            cluster_arrive(); // done reading the peers' tiles; the epilogue runs under the barrier
        }
        if (warp >= 2 && warp < 6 && (groups == 1 || run_epilogue)) {
            const int tb = nsplit > 1 ? tl0 : 0;
            const int ntok = max(0, min(nsplit > 1 ? tl1 - tl0 : BN, p.m_tok - (t0 + tb)));
            epi(src, t0 + tb, ntok, f0, min(kUmmaM, p.n_feat - f0), static_cast<int>(threadIdx.x) - 64, epi_scratch);
        }
        if (nsplit > 1)
            cluster_wait(); // peers are done reading this CTA's tile
    }
    if (!ok)
        atomicExch(p.err, 1);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_d, S::kTmemCols);
    }
}

template <GemmKind kKind, int BN, typename Epi> inline void gemm_prepare_kernel() {
    using S = GemmShape<kKind, BN>;
    static thread_local int done_device = -1;
    int dev = 0;
    OPWORKS_CUDA_CHECK(cudaGetDevice(&dev));
    if (done_device != dev) {
        OPWORKS_CUDA_CHECK(cudaFuncSetAttribute(umma_gemm_kernel<kKind, BN, Epi>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(S::kSmemBytes)));
        if constexpr (is_tile_epilogue<Epi>::value)
            OPWORKS_CUDA_CHECK(cudaFuncSetAttribute(umma_gemm_kernel<kKind, BN, Epi>,
                                                    cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        done_device = dev;
    }
}

template <GemmKind kKind, int BN, typename Epi>
inline void gemm_launch(const CUtensorMap &a, const CUtensorMap &b, const CUtensorMap &a_lo,
                        const CUtensorMap &b_lo, const GemmParams &p, const Epi &epi, cudaStream_t stream) {
    using S = GemmShape<kKind, BN>;
    gemm_prepare_kernel<kKind, BN, Epi>();
    const dim3 grid((p.n_feat + kUmmaM - 1) / kUmmaM, (p.m_tok + BN - 1) / BN, p.splits);
    detail::require(grid.y <= 65535 && grid.z <= 65535, "GEMM grid exceeds the CUDA limits");
    if constexpr (is_tile_epilogue<Epi>::value) {
        const int csz = p.splits > 1 && p.cluster > 0 ? p.cluster : p.splits;
        detail::require(csz >= 1 && csz <= kMaxClusterSplitsNonPortable && p.splits % csz == 0,
                        "tile epilogue: at most 16 K splits per cluster, splits a multiple of the cluster");
        detail::require(p.splits == csz || (p.red_ws != nullptr && p.red_cnt != nullptr),
                        "tile epilogue: grouped split K needs a workspace");
        launch_ex_cluster(umma_gemm_kernel<kKind, BN, Epi>, grid, dim3(1, 1, csz), dim3(S::kThreads),
                          S::kSmemBytes, stream, a, b, a_lo, b_lo, p, epi);
    } else {
        launch_ex(umma_gemm_kernel<kKind, BN, Epi>, grid, dim3(S::kThreads), S::kSmemBytes, stream, a, b, a_lo, b_lo,
                  p, epi);
    }
}

// Operand description for the host launcher.
struct GemmOperand {
    const void *hi;     // 16-bit words (bf16, or fp16 with f16) or fp32 (tf32 hi part)
    const void *lo;     // tf32 lo part (kTF32x3), remainder term (token operand of kBF16x2)
    int rows;
    int64_t ld;         // row stride in elements; K extent is the GEMM's k
    bool f16 = false;   // 16-bit words are fp16 (both operands of a GEMM agree)
};

// A/B format code of a 16-bit GEMM from its operands.
inline uint32_t gemm_ab_format(const GemmOperand &A, const GemmOperand &B) {
    detail::require(A.f16 == B.f16, "GEMM operands must share one 16-bit format");
    return A.f16 ? kFmtF16 : kFmtBF16;
}

inline int gemm_pick_bn(GemmKind kind, int m_tok) {
    if (m_tok <= 32)
        return 32;
    if (m_tok <= 64)
        return 64;
    if (m_tok <= 128 || kind != GemmKind::kBF16)
        return 128;
    return 256;
}

// CTAs of one tile shape resident per SM.
inline int gemm_ctas_per_sm(int bn) { return bn <= 64 ? 2 : 1; }

// Number of K splits: the most that keep tiles x splits CTAs resident in one
// wave (`slots` = SMs x CTAs per SM) without making a split shorter than
// `min_kb` blocks. A grid of at least one wave of tiles is not split.
inline int gemm_pick_splits(int tiles, int num_kb, int slots, int min_kb = 2, int max_splits = 64) {
    if (tiles >= slots / 2)
        return 1;
    int s = slots / tiles;
    if (s > max_splits)
        s = max_splits;
    const int cap = num_kb / (min_kb > 0 ? min_kb : 1);
    if (s > cap)
        s = cap;
    return s > 1 ? s : 1;
}

// out[split][tok][feat] = epi(sum_k A[feat][k] B[tok][k]); `k` is the logical
// K extent. A K tail shorter than one 128-byte block is zero-filled by TMA,
// so only the row strides need 16-byte alignment.
template <GemmKind kKind, typename Epi = Identity>
inline void gemm_tn(const GemmOperand &A, const GemmOperand &B, int k, float *out, int64_t ldo, int splits,
                    int64_t split_stride, cudaStream_t stream, const Epi &epi = {}, int force_bn = 0,
                    const void *l2_prefetch = nullptr, uint64_t l2_prefetch_bytes = 0,
                    const SplitGroupWorkspace *groups_ws = nullptr, int cluster = 0, bool l2_prefetch_tail = false) {
    constexpr bool kBf16 = kKind != GemmKind::kTF32x3;
    constexpr int kKElems = kBf16 ? 64 : 32;
    detail::require(k > 0, "gemm_tn: K must be positive");
    detail::require(A.rows > 0 && B.rows > 0, "gemm_tn: empty operand");
    GemmParams p;
    p.out = out;
    p.ldo = ldo;
    p.split_stride = split_stride;
    p.n_feat = A.rows;
    p.m_tok = B.rows;
    p.num_kb = (k + kKElems - 1) / kKElems;
    p.splits = splits < 1 ? 1 : (splits > p.num_kb ? p.num_kb : splits);
    p.err = device_error_word();
    if constexpr (kBf16)
        p.ab_fmt = gemm_ab_format(A, B);
    detail::require(l2_prefetch_bytes == 0 || (reinterpret_cast<uintptr_t>(l2_prefetch) % 16 == 0),
                    "gemm_tn: L2 prefetch range must be 16-byte aligned");
    p.l2_prefetch = static_cast<const uint8_t *>(l2_prefetch);
    p.l2_prefetch_bytes = l2_prefetch_bytes & ~uint64_t(15);
    p.l2_prefetch_tail = l2_prefetch_tail;
    int bn = force_bn ? force_bn : gemm_pick_bn(kKind, B.rows);
    if (is_tile_epilogue<Epi>::value && cluster > 0 && p.splits > cluster) {
        // grouped split K: the tile grid's partial slices must fit the workspace
        const int tiles = ((A.rows + kUmmaM - 1) / kUmmaM) * ((B.rows + bn - 1) / bn);
        detail::require(groups_ws != nullptr && force_bn != 0 && p.splits % cluster == 0,
                        "gemm_tn: grouped split K needs a workspace, an explicit token tile and whole clusters");
        detail::require(static_cast<size_t>(tiles) * (p.splits / cluster) * bn * kUmmaM <= groups_ws->floats &&
                            tiles * cluster <= groups_ws->max_counters,
                        "gemm_tn: grouped split-K workspace too small");
        p.cluster = cluster;
        p.red_ws = groups_ws->partials;
        p.red_cnt = groups_ws->counters;
    }
    if (!force_bn && p.splits == 1) {
        // narrow the token tile while the grid is under one wave
        const int sms = detail::device_facts().sm_count;
        const int ftiles = (A.rows + kUmmaM - 1) / kUmmaM;
        while (bn > 32 && ftiles * ((B.rows + bn - 1) / bn) < sms)
            bn /= 2;
    }
    const CUtensorMap ta = make_tmap_2d(A.hi, kBf16, static_cast<uint64_t>(k), A.rows, A.ld, kKElems, kUmmaM);
    const CUtensorMap tb = make_tmap_2d(B.hi, kBf16, static_cast<uint64_t>(k), B.rows, B.ld, kKElems, bn);
    CUtensorMap ta_lo = ta, tb_lo = tb;
    if constexpr (!kBf16) {
        ta_lo = make_tmap_2d(A.lo, false, static_cast<uint64_t>(k), A.rows, A.ld, kKElems, kUmmaM);
        tb_lo = make_tmap_2d(B.lo, false, static_cast<uint64_t>(k), B.rows, B.ld, kKElems, bn);
    }
    if constexpr (kKind == GemmKind::kBF16x2)
        tb_lo = make_tmap_2d(B.lo, true, static_cast<uint64_t>(k), B.rows, B.ld, kKElems, bn);
    switch (bn) {
    case 32: gemm_launch<kKind, 32, Epi>(ta, tb, ta_lo, tb_lo, p, epi, stream); break;
    case 64: gemm_launch<kKind, 64, Epi>(ta, tb, ta_lo, tb_lo, p, epi, stream); break;
    case 128: gemm_launch<kKind, 128, Epi>(ta, tb, ta_lo, tb_lo, p, epi, stream); break;
    default:
        // BN = 256 for single-term bf16 (tile epilogues: unsplit only)
        if constexpr (kKind != GemmKind::kBF16)
            gemm_launch<kKind, 128, Epi>(ta, tb, ta_lo, tb_lo, p, epi, stream);
        else if (is_tile_epilogue<Epi>::value && p.splits > 1)
            gemm_launch<kKind, 128, Epi>(ta, tb, ta_lo, tb_lo, p, epi, stream);
        else
            gemm_launch<kKind, 256, Epi>(ta, tb, ta_lo, tb_lo, p, epi, stream);
        break;
    }
}

// Tile epilogue that writes C[tok][feat] = epi(sum) from the reduced tile:
// lets a plain element epilogue (which may be non-linear, e.g. ReLU) run
// behind cluster split-K, where it sees the full sum.
template <typename Epi> struct StoreTileEpi {
    static constexpr bool kTile = true;
    float *c;
    int64_t ldc;
    Epi epi;
    __device__ void operator()(const float *tile, int tok0, int ntok, int f0, int nfeat, int tid, void *) const {
        for (int i = tid; i < ntok * kUmmaM; i += 128) {
            const int t = i / kUmmaM, f = i % kUmmaM;
            if (f < nfeat)
                c[static_cast<int64_t>(tok0 + t) * ldc + f0 + f] = apply_epilogue(epi, tile[i], tok0 + t, f0 + f);
        }
    }
};

// Split-precision (3xTF32) C[tok][feat] = epi(A . B^T) with the tile plan for
// fp32 operator GEMMs: when 128 x 128 tiles leave most SMs idle and K is
// long, the K range of each tile is split across a cluster of up to 8 CTAs
// (reduced through distributed shared memory, epilogue on the full sum);
// otherwise one unsplit launch with the token tile narrowed to fill a wave.
template <typename Epi = Identity>
inline void gemm_tf32x3(const GemmOperand &A, const GemmOperand &B, int k, float *C, int64_t ldc,
                        cudaStream_t stream, const Epi &epi = {}) {
    const int sms = detail::device_facts().sm_count;
    const int tiles = ((A.rows + kUmmaM - 1) / kUmmaM) * ((B.rows + 127) / 128);
    const int num_kb = (k + 31) / 32;
    if (B.rows > 64 && tiles < sms / 2) {
        int splits = sms / tiles;
        splits = splits > kMaxClusterSplits ? kMaxClusterSplits : splits;
        splits = splits > num_kb / 8 ? num_kb / 8 : splits;
        if (splits >= 2) {
            gemm_tn<GemmKind::kTF32x3, StoreTileEpi<Epi>>(A, B, k, nullptr, ldc, splits, 0, stream,
                                                           StoreTileEpi<Epi>{C, ldc, epi}, 128);
            return;
        }
    }
    gemm_tn<GemmKind::kTF32x3, Epi>(A, B, k, C, ldc, 1, 0, stream, epi);
}

// C[m][k] = epi(sum_n A[m][n] * B[n][k]) on raw row-major fp32 matrices
// (A [M][N] row stride lda, B [N][K] row stride ldb): kTF32x3S, the
// split-precision GEMM that splits both operands into tf32 hi / lo in shared
// memory, with B's rows read as the MN-major feature operand (no transpose,
// no scratch). A, B 16-byte aligned and lda, ldb multiples of 4; grids of
// fewer tiles than half the SMs split K over a cluster as gemm_tf32x3 does.
template <typename Epi>
inline void gemm_tf32x3s(const float *A, int64_t lda, const float *B, int64_t ldb, int M, int N, int K, float *C,
                         int64_t ldc, cudaStream_t stream, const Epi &epi = {}) {
    detail::require(M > 0 && N > 0 && K > 0, "gemm_tf32x3s: empty operand");
    GemmParams p;
    p.out = C;
    p.ldo = ldc;
    p.split_stride = 0;
    p.n_feat = K;
    p.m_tok = M;
    p.num_kb = (N + 31) / 32;
    p.splits = 1;
    p.err = device_error_word();
    const int sms = detail::device_facts().sm_count;
    const int ftiles = (K + kUmmaM - 1) / kUmmaM;
    int bn = gemm_pick_bn(GemmKind::kTF32x3S, M);
    int splits = 1;
    if (M > 64 && ftiles * ((M + 127) / 128) < sms / 2) {
        splits = sms / (ftiles * ((M + 127) / 128));
        splits = splits > kMaxClusterSplits ? kMaxClusterSplits : splits;
        splits = splits > p.num_kb / 8 ? p.num_kb / 8 : splits;
        splits = splits < 1 ? 1 : splits;
    }
    if (splits == 1)
        while (bn > 32 && ftiles * ((M + bn - 1) / bn) < sms)
            bn /= 2;
    else
        bn = 128;
    const CUtensorMap ta = make_tmap_2d(B, false, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                                        static_cast<uint64_t>(ldb), 32, 32, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    const CUtensorMap tb = make_tmap_2d(A, false, static_cast<uint64_t>(N), static_cast<uint64_t>(M),
                                        static_cast<uint64_t>(lda), 32, static_cast<uint32_t>(bn));
    if (splits > 1) {
        p.splits = splits;
        p.out = nullptr;
        gemm_launch<GemmKind::kTF32x3S, 128, StoreTileEpi<Epi>>(ta, tb, ta, tb, p, StoreTileEpi<Epi>{C, ldc, epi},
                                                                 stream);
        return;
    }
    switch (bn) {
    case 32: gemm_launch<GemmKind::kTF32x3S, 32, Epi>(ta, tb, ta, tb, p, epi, stream); break;
    case 64: gemm_launch<GemmKind::kTF32x3S, 64, Epi>(ta, tb, ta, tb, p, epi, stream); break;
    default: gemm_launch<GemmKind::kTF32x3S, 128, Epi>(ta, tb, ta, tb, p, epi, stream); break;
    }
}

} // namespace opworks::sm100

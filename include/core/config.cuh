#pragma once

// Compile-time knobs of the OpWorks-B200 operator layer.
//
// The OPWORKS_* macro names and the opworks::k* constants are the public
// surface of the OpWorks configuration header (reference: include/core/
// config.cuh:15-77) and keep their meaning, so code written against OpWorks
// (e.g. `nvcc -DOPWORKS_THREADS=512`) still builds. The kernels behind them
// are sm_100a-specific: the elementwise pack is 16 bytes per thread by
// default and the GEMM tile constants below describe the tcgen05 tiles, not
// the SIMT 64x64 tile of the original.

#include <cfloat>
#include <cmath>

#ifndef OPWORKS_THREADS
#define OPWORKS_THREADS 256
#endif

#ifndef OPWORKS_NUM_WAVES
#define OPWORKS_NUM_WAVES 32
#endif

#ifndef OPWORKS_PACK_SIZE
#define OPWORKS_PACK_SIZE 4
#endif

// Kept for source compatibility: kMatmulTile/kMatmulBlock/kMatmulSub are
// still validated, but the sm_100a GEMM uses the tcgen05 tile constants.
#ifndef OPWORKS_MATMUL_TILE
#define OPWORKS_MATMUL_TILE 64
#endif

#ifndef OPWORKS_MATMUL_BLOCK
#define OPWORKS_MATMUL_BLOCK 16
#endif

#ifndef OPWORKS_MATMUL_SUBTILE
#define OPWORKS_MATMUL_SUBTILE 4
#endif

#ifndef OPWORKS_LAYERNORM_EPS
#define OPWORKS_LAYERNORM_EPS 1e-5f
#endif

// Device-side spin-wait limit (nanoseconds) for mbarrier waits in the
// warp-specialised kernels. A wait that runs out records an error code and
// the kernel returns instead of hanging the GPU.
#ifndef OPWORKS_WAIT_TIMEOUT_NS
#define OPWORKS_WAIT_TIMEOUT_NS 2000000000ull
#endif

namespace opworks {

// Hardware facts (CUDA execution model; not tunable).
constexpr int kWarpSize = 32;
constexpr int kMaxThreadsPerBlock = 1024;
constexpr unsigned kFullWarpMask = 0xffffffffu;

constexpr float kInf = INFINITY;
constexpr float kNegInf = -INFINITY;
constexpr float kFloatMax = FLT_MAX;
constexpr float kFloatLowest = -FLT_MAX;

constexpr int kThreads = OPWORKS_THREADS;
constexpr int kNumWaves = OPWORKS_NUM_WAVES;
constexpr int kPackSize = OPWORKS_PACK_SIZE;

constexpr int kMatmulTile = OPWORKS_MATMUL_TILE;
constexpr int kMatmulBlock = OPWORKS_MATMUL_BLOCK;
constexpr int kMatmulSub = OPWORKS_MATMUL_SUBTILE;

constexpr float kLayerNormEps = OPWORKS_LAYERNORM_EPS;

constexpr unsigned long long kWaitTimeoutNs = OPWORKS_WAIT_TIMEOUT_NS;

// B200 (sm_100a) facts used to size grids and tiles.
constexpr int kB200SmCount = 148;           // 2 dies x 74 SMs
constexpr int kMaxSmemPerBlock = 227 * 1024; // opt-in dynamic shared memory
constexpr int kTmemColumns = 512;            // 32-bit columns per SM

// tcgen05 GEMM tile: 128 output features (TMEM lanes) x BN tokens (TMEM
// columns), 128-byte K slices so each smem row is one 128B swizzle atom.
constexpr int kUmmaM = 128;
constexpr int kUmmaKBytes = 128;

static_assert(kThreads > 0 && kThreads % kWarpSize == 0 && kThreads <= kMaxThreadsPerBlock,
              "kThreads must be a positive multiple of kWarpSize and fit in a block");
static_assert(kNumWaves > 0, "kNumWaves must be positive");
static_assert(kPackSize == 1 || kPackSize == 2 || kPackSize == 4,
              "kPackSize must be 1, 2 or 4 (alignment must be a power of two)");
static_assert(kMatmulTile == kMatmulBlock * kMatmulSub, "kMatmulTile must equal kMatmulBlock * kMatmulSub");
static_assert(kMatmulBlock > 0 && kMatmulSub > 0 && kMatmulTile > 0, "matmul dimensions must be positive");
static_assert(kMatmulBlock * kMatmulBlock <= kMaxThreadsPerBlock,
              "matmul thread block must fit in kMaxThreadsPerBlock threads");
static_assert(kLayerNormEps > 0 && kLayerNormEps <= FLT_MAX, "layer norm epsilon must be finite and positive");

} // namespace opworks

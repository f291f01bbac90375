#pragma once

// Tensor-parallel shard plan: which rows and columns of each fused projection
// rank `rank` of `world` owns (the engine's layout: QKV = [q; k; v] rows,
// gate/up rows interleaved 2j = gate_j, 2j + 1 = up_j, O = [H][q width],
// down = [H][I]). Rank r owns query heads [r qh / world, ...), the KV heads
// they read, [r kvh / world, ...), and MLP columns [r I / world, ...):
//   QKV   its q, k and v head rows (three row ranges)
//   O     the input columns of its query heads (a column slice; the partial
//         products of all ranks sum to the full projection)
//   gate/up  the interleaved rows of its MLP columns (one contiguous range)
//   down  the input columns of its MLP columns (a column slice)
// Embedding, norms and the LM head stay whole on every rank. Pure host
// arithmetic: the engine and the host-side tests share it.

#include <cstdint>

#include "../core/cuda_utils.cuh"
#include "../runtime/model_config.cuh"

namespace opworks {

struct TpShard {
    int q_heads = 0, kv_heads = 0, inter = 0; // this rank's counts
    int64_t q_row0 = 0, k_row0 = 0, v_row0 = 0; // first QKV rows of its q / k / v heads
    int64_t q_rows = 0, kv_rows = 0;             // rows per range (q, and k = v)
    int64_t o_col0 = 0;                          // O input columns [o_col0, o_col0 + q_rows)
    int64_t gu_row0 = 0, gu_rows = 0;            // interleaved gate/up rows
    int64_t down_col0 = 0;                       // down input columns [down_col0, down_col0 + inter)
};

inline TpShard tp_shard(const ModelConfig &cfg, int rank, int world) {
    detail::require(world >= 1 && rank >= 0 && rank < world, "bad tensor-parallel rank / world");
    detail::require(cfg.num_q_heads % world == 0 && cfg.num_kv_heads % world == 0 &&
                        cfg.intermediate_size % (128 * world) == 0 && cfg.hidden_size % 128 == 0,
                    "tensor parallelism needs KV heads and 128-column MLP tiles divisible by the world size");
    const int64_t D = cfg.head_dim;
    TpShard s;
    s.q_heads = cfg.num_q_heads / world;
    s.kv_heads = cfg.num_kv_heads / world;
    s.inter = cfg.intermediate_size / world;
    s.q_rows = s.q_heads * D;
    s.kv_rows = s.kv_heads * D;
    s.q_row0 = rank * s.q_rows;
    s.k_row0 = static_cast<int64_t>(cfg.num_q_heads) * D + rank * s.kv_rows;
    s.v_row0 = static_cast<int64_t>(cfg.num_q_heads + cfg.num_kv_heads) * D + rank * s.kv_rows;
    s.o_col0 = rank * s.q_rows;
    s.gu_rows = 2 * static_cast<int64_t>(s.inter);
    s.gu_row0 = rank * s.gu_rows;
    s.down_col0 = static_cast<int64_t>(rank) * s.inter;
    return s;
}

} // namespace opworks

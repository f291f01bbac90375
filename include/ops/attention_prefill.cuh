#pragma once

// ops::attention_prefill_chunked — causal GQA attention of T queries
// (absolute positions q_offset .. q_offset + T - 1, q_offset == S - T) over S
// cached keys, q/out in per-head slabs [qh, T, D], cache [kvh, cap, D]
// (OpWorks include/ops/attention_prefill.cuh:164-177; same checks). Online
// softmax over 64-key tiles staged by bulk async copies, the kRep heads of a
// GQA group sharing each tile. head_dim must be 64.

#include "attention_kernels.cuh"

namespace opworks::ops {

inline void attention_prefill_chunked(const float *q_heads, const float *kcache, const float *vcache, float *out,
                                      int T, int S, int q_offset, int num_q_heads, int kv_rep, int head_dim, int cap,
                                      cudaStream_t stream = nullptr) {
    detail::require(T > 0 && S >= T && q_offset == S - T, "attention_prefill_chunked: bad shape/offset");
    detail::require(num_q_heads > 0 && kv_rep > 0 && num_q_heads % kv_rep == 0,
                    "attention_prefill_chunked: bad head shape");
    detail::require(head_dim == detail::kAttnD, "attention_prefill_chunked supports head_dim == 64");
    detail::require(cap >= S, "attention_prefill_chunked: length exceeds cache capacity");
    detail::require(q_heads && kcache && vcache && out, "attention_prefill_chunked requires non-null pointers");
    const int kvh = num_q_heads / kv_rep;
    const float scale = 1.f / sqrtf(static_cast<float>(head_dim));
    const detail::ContigKV kv{kcache, vcache, cap};
    const int64_t tok = detail::kAttnD, head = static_cast<int64_t>(T) * detail::kAttnD;
    const detail::StridedOut<float> o{out, tok, head};
    switch (kv_rep) {
    case 1: detail::attn_prefill_launch<detail::ContigKV, 1>(q_heads, tok, head, o, kv, 0, T, q_offset, kvh, scale, stream); break;
    case 2: detail::attn_prefill_launch<detail::ContigKV, 2>(q_heads, tok, head, o, kv, 0, T, q_offset, kvh, scale, stream); break;
    case 4: detail::attn_prefill_launch<detail::ContigKV, 4>(q_heads, tok, head, o, kv, 0, T, q_offset, kvh, scale, stream); break;
    case 8: detail::attn_prefill_launch<detail::ContigKV, 8>(q_heads, tok, head, o, kv, 0, T, q_offset, kvh, scale, stream); break;
    default: detail::require(false, "attention_prefill_chunked supports kv_rep in {1, 2, 4, 8}");
    }
}

} // namespace opworks::ops

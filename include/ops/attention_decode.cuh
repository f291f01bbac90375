#pragma once

// ops::attention_decode — one query per q head against the first `len`
// entries of a [kvh, max_seq, D] cache, GQA kv head = q_head / kv_rep
// (OpWorks include/ops/attention_decode.cuh:99-109). Same arguments and the
// same contract: asynchronous on `stream`, no allocation, no host copy, so it
// can be captured in a CUDA graph. The 8192-token shared-memory limit of the
// original is gone (K/V stream through a staged ring); head_dim must be 64
// with kv_rep in {1, 2, 4, 8}. One CTA per KV head runs all of its query
// heads, so every K/V row is read once (the original reads it once per query
// head); the batched engine uses the split-KV form of the same kernel.

#include "attention_kernels.cuh"

namespace opworks::ops {

inline void attention_decode(const float *q, const float *kcache, const float *vcache, float *out, int num_q_heads,
                             int kv_rep, int head_dim, int len, int max_seq, cudaStream_t stream = nullptr) {
    detail::require(num_q_heads > 0 && kv_rep > 0 && head_dim > 0, "attention_decode requires positive head shape");
    detail::require(head_dim == detail::kAttnD, "attention_decode supports head_dim == 64");
    detail::require(num_q_heads % kv_rep == 0, "attention_decode: q heads must be a multiple of kv_rep");
    detail::require(len > 0 && len <= max_seq, "attention_decode length outside the cache capacity");
    detail::require(q && kcache && vcache && out, "attention_decode requires non-null pointers");
    const int kvh = num_q_heads / kv_rep;
    const float scale = 1.f / sqrtf(static_cast<float>(head_dim));
    // one split covering every token: the result is normalised in place of
    // split partials, so nothing but q, the caches and out is touched
    const int tps = (len + detail::kDecodeTile - 1) / detail::kDecodeTile * detail::kDecodeTile;
    const detail::ContigKV kv{kcache, vcache, max_seq};
    const detail::StridedOut<float> o{out, 0, detail::kAttnD};
    switch (kv_rep) {
    case 1: detail::attn_decode_launch<detail::ContigKV, 1>(q, 0, kv, nullptr, 1, kvh, tps, 1, scale, nullptr, nullptr, o, stream, len); break;
    case 2: detail::attn_decode_launch<detail::ContigKV, 2>(q, 0, kv, nullptr, 1, kvh, tps, 1, scale, nullptr, nullptr, o, stream, len); break;
    case 4: detail::attn_decode_launch<detail::ContigKV, 4>(q, 0, kv, nullptr, 1, kvh, tps, 1, scale, nullptr, nullptr, o, stream, len); break;
    case 8: detail::attn_decode_launch<detail::ContigKV, 8>(q, 0, kv, nullptr, 1, kvh, tps, 1, scale, nullptr, nullptr, o, stream, len); break;
    default: detail::require(false, "attention_decode supports kv_rep in {1, 2, 4, 8}");
    }
}

} // namespace opworks::ops

#pragma once

// ops::attention_decode — one query per q head against the first `len`
// entries of a [kvh, max_seq, D] cache, GQA kv head = q_head / kv_rep
// (OpWorks include/ops/attention_decode.cuh:99-109). Same arguments; the
// 8192-token shared-memory limit of the original is gone (split-KV), and
// head_dim must be 64 with kv_rep in {1, 2, 4, 8}.

#include "attention_kernels.cuh"
#include "detail/operand_prep.cuh"

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
    const int tps = detail::decode_tokens_per_split(kvh, len, detail::device_facts().sm_count);
    const int splits = (len + tps - 1) / tps;
    const size_t po = sizeof(float) * static_cast<size_t>(num_q_heads) * splits * detail::kAttnD;
    const size_t pml = sizeof(float) * static_cast<size_t>(num_q_heads) * splits * 2;
    detail::StreamScratch scratch(po + pml + 256, stream);
    float *part_o = scratch.as<float>(0);
    float *part_ml = scratch.as<float>(po);
    int *lens = scratch.as<int>(po + pml);
    OPWORKS_CUDA_CHECK(cudaMemcpyAsync(lens, &len, sizeof(int), cudaMemcpyHostToDevice, stream));
    const detail::ContigKV kv{kcache, vcache, max_seq};
    const detail::StridedOut<float> o{out, 0, detail::kAttnD};
    switch (kv_rep) {
    case 1: detail::attn_decode_launch<detail::ContigKV, 1>(q, 0, kv, lens, 1, kvh, tps, splits, scale, part_o, part_ml, o, stream); break;
    case 2: detail::attn_decode_launch<detail::ContigKV, 2>(q, 0, kv, lens, 1, kvh, tps, splits, scale, part_o, part_ml, o, stream); break;
    case 4: detail::attn_decode_launch<detail::ContigKV, 4>(q, 0, kv, lens, 1, kvh, tps, splits, scale, part_o, part_ml, o, stream); break;
    case 8: detail::attn_decode_launch<detail::ContigKV, 8>(q, 0, kv, lens, 1, kvh, tps, splits, scale, part_o, part_ml, o, stream); break;
    default: detail::require(false, "attention_decode supports kv_rep in {1, 2, 4, 8}");
    }
    // the host value `len` must outlive the async copy
    OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream));
}

} // namespace opworks::ops

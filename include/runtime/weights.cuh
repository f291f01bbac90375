#pragma once

// Device-resident Llama weights, laid out for the B200 kernels at load time.
//
// The pack stores HF tensors [out, in] (OpWorks include/runtime/weights.cuh:
// same tensor names and element-count checks, norms always fp32, the tied
// lm_head alias required). Here each layer's projections are fused and
// converted once on the device:
//   qkv  = [q; k; v] rows           [(qh + 2 kvh) * D, H]
//   gu   = interleaved gate/up rows  [2 I, H]   (row 2j = gate_j, 2j+1 = up_j)
//   o    = [H, qh * D], down = [H, I]
// in up to three precisions:
//   16-bit (fast path: tcgen05 kind::f16 GEMMs) — fp16 for float32 packs
//          (11 significant bits at 2 bytes per weight), the pack's own bf16
//          values for bfloat16 packs; OPWORKS_FAST_WEIGHTS=bf16 makes
//          float32 packs round to bf16 instead
//   f32    (accurate path, few rows: shared-weight GEMV)
//   hi/lo  (accurate path, many rows: split-precision tf32 GEMM)
// bf16 packs load the 16-bit set only.

#include <cuda_bf16.h>

#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../core/typed_device_buffer.cuh"
#include "../ops/llama_kernels.cuh"
#include "model_config.cuh"
#include "pack_reader.cuh"

namespace opworks {

enum WeightSets : unsigned { kWeights16 = 1u, kWeightsF32 = 2u, kWeightsSplit = 4u };

// One fused projection in every precision that was loaded.
struct Projection {
    int out = 0, in = 0;
    TypedDeviceBuffer<uint16_t> w16; // format: ModelWeights::f16
    TypedDeviceBuffer<float> f32, hi, lo;
};

template <typename WT> struct LayerWeights {
    TypedDeviceBuffer<float> input_norm; // [H]
    TypedDeviceBuffer<float> post_norm;  // [H]
    Projection qkv, o, gu, down;
};

template <typename WT> struct ModelWeights {
    TypedDeviceBuffer<float> embed_f32;           // [V, H] fp32 packs
    TypedDeviceBuffer<uint16_t> embed_w16;        // [V, H] (tied LM head, fast path)
    TypedDeviceBuffer<float> final_norm;          // [H]
    std::vector<LayerWeights<WT>> layers;
    TypedDeviceBuffer<float> rope_inv_freq;       // [D / 2]
    TypedDeviceBuffer<float> rope_table;          // [max_pos][D / 2][2] (cos, sin)
    int rope_max_pos = 0;
    unsigned sets = 0;
    bool f16 = false; // the 16-bit set holds fp16 words (else bf16)

    static ModelWeights load(const PackReader &pack, const ModelConfig &cfg, unsigned sets,
                             int rope_max_pos = 8192, cudaStream_t stream = nullptr) {
        const bool f32_pack = pack.dtype() == "float32";
        if constexpr (std::is_same_v<WT, float>) {
            if (!f32_pack)
                throw std::runtime_error("fp32 model requires a float32 pack");
        } else {
            if (f32_pack)
                throw std::runtime_error("bf16 model requires a bfloat16 pack");
            sets = kWeights16;
        }
        if (sets == 0)
            sets = kWeights16;
        ModelWeights w;
        w.sets = sets;
        const char *fmt = std::getenv("OPWORKS_FAST_WEIGHTS");
        w.f16 = f32_pack && !(fmt && std::strcmp(fmt, "bf16") == 0);
        const int64_t H = cfg.hidden_size, I = cfg.intermediate_size;
        const int64_t qw = cfg.q_width(), kw = cfg.kv_width();
        const int64_t V = cfg.vocab_size;
        auto check = [&](const std::string &name, int64_t numel) {
            if (pack.meta(name).numel != numel)
                throw std::runtime_error(name + ": element count mismatch");
        };
        // staging of raw pack bytes on the device (largest tensor: embedding)
        const size_t esz = pack.elem_size();
        TypedDeviceBuffer<uint8_t> stage(static_cast<int64_t>(V * H * esz));
        TypedDeviceBuffer<uint8_t> stage2(static_cast<int64_t>(I * H * esz));
        auto upload = [&](const std::string &name, void *dst, int64_t numel) {
            check(name, numel);
            OPWORKS_CUDA_CHECK(cudaMemcpyAsync(dst, pack.data(name), static_cast<size_t>(numel) * esz,
                                               cudaMemcpyHostToDevice, stream));
        };
        auto norm = [&](const std::string &name) {
            check(name, H);
            if (f32_pack)
                return TypedDeviceBuffer<float>::from_host(pack.read(name), stream);
            return TypedDeviceBuffer<float>::from_host(pack.read_bf16_as_float(name), stream);
        };
        const int grid = 4 * detail::device_facts().sm_count;

        // embedding / tied LM head
        check("model.embed_tokens.weight", V * H);
        if (!pack.has("lm_head.weight"))
            throw std::runtime_error("pack has neither lm_head.weight nor a tying alias");
        if (f32_pack) {
            w.embed_f32 = TypedDeviceBuffer<float>(V * H);
            upload("model.embed_tokens.weight", w.embed_f32.data(), V * H);
            if (sets & kWeights16) {
                w.embed_w16 = TypedDeviceBuffer<uint16_t>(V * H);
                detail::weights_to_16_kernel<<<grid, 256, 0, stream>>>(w.embed_f32.data(), nullptr,
                                                                       static_cast<int>(V), static_cast<int>(H),
                                                                       w.embed_w16.data(), w.f16);
                OPWORKS_CUDA_CHECK(cudaGetLastError());
            }
        } else {
            w.embed_w16 = TypedDeviceBuffer<uint16_t>(V * H);
            upload("model.embed_tokens.weight", w.embed_w16.data(), V * H);
        }
        w.final_norm = norm("model.norm.weight");

        // fp32 source matrix (already on the device) -> the loaded precisions
        auto finish_f32 = [&](Projection &p, float *src_f32, const float *interleave_b) {
            const int rows = interleave_b ? p.out / 2 : p.out;
            if (sets & kWeights16) {
                p.w16 = TypedDeviceBuffer<uint16_t>(static_cast<int64_t>(p.out) * p.in);
                detail::weights_to_16_kernel<<<grid, 256, 0, stream>>>(src_f32, interleave_b, rows, p.in,
                                                                       p.w16.data(), w.f16);
                OPWORKS_CUDA_CHECK(cudaGetLastError());
            }
            if (sets & kWeightsSplit) {
                p.hi = TypedDeviceBuffer<float>(static_cast<int64_t>(p.out) * p.in);
                p.lo = TypedDeviceBuffer<float>(static_cast<int64_t>(p.out) * p.in);
                detail::weights_to_split_kernel<<<grid, 256, 0, stream>>>(src_f32, interleave_b, rows, p.in,
                                                                          p.hi.data(), p.lo.data());
                OPWORKS_CUDA_CHECK(cudaGetLastError());
            }
        };

        w.layers.resize(cfg.num_layers);
        for (int i = 0; i < cfg.num_layers; ++i) {
            const std::string pre = "model.layers." + std::to_string(i) + ".";
            LayerWeights<WT> &lw = w.layers[i];
            lw.input_norm = norm(pre + "input_layernorm.weight");
            lw.post_norm = norm(pre + "post_attention_layernorm.weight");
            lw.qkv.out = static_cast<int>(qw + 2 * kw);
            lw.qkv.in = static_cast<int>(H);
            lw.o.out = static_cast<int>(H);
            lw.o.in = static_cast<int>(qw);
            lw.gu.out = static_cast<int>(2 * I);
            lw.gu.in = static_cast<int>(H);
            lw.down.out = static_cast<int>(H);
            lw.down.in = static_cast<int>(I);
            if (f32_pack) {
                // q|k|v concatenated in the fp32 buffer (kept only if the f32 set is loaded)
                TypedDeviceBuffer<float> qkv(static_cast<int64_t>(lw.qkv.out) * H);
                upload(pre + "self_attn.q_proj.weight", qkv.data(), qw * H);
                upload(pre + "self_attn.k_proj.weight", qkv.data() + qw * H, kw * H);
                upload(pre + "self_attn.v_proj.weight", qkv.data() + (qw + kw) * H, kw * H);
                finish_f32(lw.qkv, qkv.data(), nullptr);
                TypedDeviceBuffer<float> o(H * qw);
                upload(pre + "self_attn.o_proj.weight", o.data(), H * qw);
                finish_f32(lw.o, o.data(), nullptr);
                // gate in `stage`, up in `stage2`, interleaved into gu
                float *gate = reinterpret_cast<float *>(stage.data());
                float *up = reinterpret_cast<float *>(stage2.data());
                upload(pre + "mlp.gate_proj.weight", gate, I * H);
                upload(pre + "mlp.up_proj.weight", up, I * H);
                finish_f32(lw.gu, gate, up);
                TypedDeviceBuffer<float> gu;
                if (sets & kWeightsF32) {
                    gu = TypedDeviceBuffer<float>(2 * I * H);
                    detail::weights_interleave_kernel<<<grid, 256, 0, stream>>>(gate, up, static_cast<int>(I),
                                                                                static_cast<int>(H), gu.data());
                    OPWORKS_CUDA_CHECK(cudaGetLastError());
                }
                TypedDeviceBuffer<float> down(H * I);
                upload(pre + "mlp.down_proj.weight", down.data(), H * I);
                finish_f32(lw.down, down.data(), nullptr);
                if (sets & kWeightsF32) {
                    lw.qkv.f32 = std::move(qkv);
                    lw.o.f32 = std::move(o);
                    lw.gu.f32 = std::move(gu);
                    lw.down.f32 = std::move(down);
                }
                // the temporaries are released here; the stream must finish
                // using them first
                OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream));
            } else {
                auto alloc16 = [&](Projection &p) {
                    p.w16 = TypedDeviceBuffer<uint16_t>(static_cast<int64_t>(p.out) * p.in);
                };
                alloc16(lw.qkv);
                upload(pre + "self_attn.q_proj.weight", lw.qkv.w16.data(), qw * H);
                upload(pre + "self_attn.k_proj.weight", lw.qkv.w16.data() + qw * H, kw * H);
                upload(pre + "self_attn.v_proj.weight", lw.qkv.w16.data() + (qw + kw) * H, kw * H);
                alloc16(lw.o);
                upload(pre + "self_attn.o_proj.weight", lw.o.w16.data(), H * qw);
                alloc16(lw.gu);
                uint16_t *gate = reinterpret_cast<uint16_t *>(stage.data());
                uint16_t *up = reinterpret_cast<uint16_t *>(stage2.data());
                upload(pre + "mlp.gate_proj.weight", gate, I * H);
                upload(pre + "mlp.up_proj.weight", up, I * H);
                detail::interleave16_kernel<<<grid, 256, 0, stream>>>(gate, up, static_cast<int>(I),
                                                                      static_cast<int>(H), lw.gu.w16.data());
                OPWORKS_CUDA_CHECK(cudaGetLastError());
                alloc16(lw.down);
                upload(pre + "mlp.down_proj.weight", lw.down.w16.data(), H * I);
                OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream));
            }
        }
        const std::vector<float> inv = cfg.rope_inv_freq();
        w.rope_inv_freq = TypedDeviceBuffer<float>::from_host(inv, stream);
        w.rope_max_pos = rope_max_pos;
        const int half = cfg.head_dim / 2;
        w.rope_table = TypedDeviceBuffer<float>(static_cast<int64_t>(rope_max_pos) * half * 2);
        detail::rope_table_kernel<<<grid, 256, 0, stream>>>(w.rope_inv_freq.data(), rope_max_pos, half,
                                                            reinterpret_cast<float2 *>(w.rope_table.data()));
        OPWORKS_CUDA_CHECK(cudaGetLastError());
        OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream));
        return w;
    }
};

} // namespace opworks

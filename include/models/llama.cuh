#pragma once

// Llama-3.2 decoder on sm_100a kernels: LlamaModelT<WT> + LlamaSession keep
// the API of OpWorks include/models/llama.cuh:47-291 (load, create_session,
// prefill, decode_step, is_eos, last_logits, copy_last_logits, hidden_state,
// debug_prefill; LlamaModel = fp32 pack, LlamaModelBF16 = bf16 pack), and
// LlamaEngineT runs B sequences per forward over a paged KV cache.
//
// One forward step (rows = prefill tokens of one sequence, or one decode
// token for each of B sequences):
//   embed_rmsnorm                      hidden = E[ids], x = rms(hidden) w_in0
//   per layer:
//     QKV GEMM (split-K)  -> qkv_finalize: RoPE, K/V into paged cache, q
//     attention: decode = split-KV flash decoding (+ combine),
//                prefill = causal GQA flash attention from the cache
//     O GEMM -> add_rmsnorm (residual + post-attention norm, fused)
//     gate/up GEMM (interleaved rows) -> silu_mul
//     down GEMM -> add_rmsnorm (residual + next layer's input norm)
//   LM head (tied embedding) -> sample (greedy argmax or exact top-p)
// 9 launches per layer instead of the reference's 17, and the decode step is
// captured once per batch size as a CUDA graph (input H2D, forward, sampler,
// token D2H), so a step costs one graph launch and one stream sync.
//
// Precision: kFast = 16-bit weights and two-term 16-bit GEMM activations
// (fp16 for float32 packs, bf16 for bfloat16 packs), fp32 residual stream,
// fp32 KV cache, fp32 attention and softmax; kAccurate = fp32 end to end
// (shared-weight fp32 GEMV for <= 4 rows, split-precision TF32 tensor-core
// GEMM otherwise) — the fp32 model's default, for parity with the reference.

#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <tuple>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "../core/cuda_utils.cuh"
#include "../ops/attention_kernels.cuh"
#include "../ops/attention_prefill_tc.cuh"
#include "../ops/gemm_sm100.cuh"
#include "../ops/decode_chain.cuh"
#include "../ops/gemm_sm100_pair.cuh"
#include "../ops/linear.cuh"
#include "../ops/llama_kernels.cuh"
#include "../runtime/kv_cache.cuh"
#include "../runtime/model_config.cuh"
#include "../runtime/nccl_lite.cuh"
#include "../runtime/pack_reader.cuh"
#include "../runtime/weights.cuh"
#include "tp_plan.cuh"

namespace opworks {

enum class Precision : int { kAccurate = 0, kFast = 1 };

// Sampling controls of one sequence for one step. temperature <= 0: greedy.
struct SampleArgs {
    float temperature = 0.f;
    float top_p = 1.f;
    double uniform = -1.0; // >= 0: use this uniform (parity tests); < 0: counter RNG (seed, step)
    uint64_t seed = 0;
    int step = 0;
};

// Tensor parallelism of a fast-path engine (one process per GPU): rank `rank`
// of `world` owns query heads [rank * qh / world, ...), the matching KV heads,
// and MLP columns [rank * I / world, ...); after the o and down projections
// the ranks sum their partial outputs with one NCCL all-reduce each.
// nccl_id: the 128-byte communicator id from opw_llama_nccl_unique_id on one
// rank, shared with the others.
struct TensorParallel {
    int rank = 0, world = 1;
    const char *nccl_id = nullptr;
};

namespace detail {

// Inputs of one step, host-staged (pinned) and device-mirrored, one copy.
struct StepLayout {
    int64_t ids, seq, pos, lens, step, temp, top_p, uniform, seed, bytes;
    static int64_t align8(int64_t x) { return (x + 7) & ~int64_t(7); }
    static StepLayout make(int rows, int batch) {
        StepLayout L;
        int64_t o = 0;
        L.ids = o;
        o = align8(o + 4 * int64_t(rows));
        L.seq = o;
        o = align8(o + 4 * int64_t(rows));
        L.pos = o;
        o = align8(o + 4 * int64_t(rows));
        L.lens = o;
        o = align8(o + 4 * int64_t(batch));
        L.step = o;
        o = align8(o + 4 * int64_t(batch));
        L.temp = o;
        o = align8(o + 4 * int64_t(batch));
        L.top_p = o;
        o = align8(o + 4 * int64_t(batch));
        L.uniform = o;
        o = align8(o + 8 * int64_t(batch));
        L.seed = o;
        o = align8(o + 8 * int64_t(batch));
        L.bytes = o;
        return L;
    }
};

} // namespace detail

template <typename WT> class LlamaEngineT {
  public:
    // max_batch sequences of up to max_seq_len tokens; prefill runs in chunks
    // of at most prefill_rows tokens (0: max_seq_len).
    LlamaEngineT(const ModelConfig &cfg, const ModelWeights<WT> &w, int max_batch, int max_seq_len, Precision prec,
                 int prefill_rows = 0, const TensorParallel &tp = {})
        : cfg_(cfg), w_(w), prec_(prec), max_batch_(max_batch), max_seq_len_(max_seq_len) {
        detail::require(max_batch > 0, "batch capacity must be positive");
        detail::require(max_seq_len > 0, "max_seq_len must be positive");
        detail::require(max_seq_len <= w.rope_max_pos, "max_seq_len exceeds the model's RoPE table");
        detail::require(cfg.head_dim == detail::kAttnD, "this runtime supports head_dim 64");
        detail::require(cfg.hidden_size % detail::kRowThreads == 0 && cfg.hidden_size / detail::kRowThreads <= 16,
                        "hidden size must be a multiple of 256 (<= 4096)");
        const int rep = cfg.kv_rep();
        detail::require(rep == 1 || rep == 2 || rep == 4 || rep == 8, "GQA ratio must be 1, 2, 4 or 8");
        if (prec == Precision::kFast)
            detail::require(w.sets & kWeights16, "16-bit (fast path) weights were not loaded");
        else
            detail::require((w.sets & kWeightsF32) && (w.sets & kWeightsSplit),
                            "fp32 weights (accurate path) were not loaded");
        if (prefill_single_rows_ < 0)
            prefill_single_rows_ = w.f16 && pair_min_rows_ < (1 << 30) ? pair_min_rows_ - 1 : (1 << 30);
        prefill_rows_ = prefill_rows > 0 ? std::min(prefill_rows, max_seq_len) : max_seq_len;
        rows_max_ = std::max(prefill_rows_, max_batch);
        blocks_per_seq_ = (max_seq_len + kKvBlockTokens - 1) / kKvBlockTokens;
        OPWORKS_CUDA_CHECK(cudaGetDevice(&device_));
        OPWORKS_CUDA_CHECK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
        sm_count_ = detail::device_facts().sm_count;
        err_word_ = sm100::device_error_word();

        tp_rank_ = tp.rank;
        tp_world_ = tp.world;
        detail::require(tp_world_ >= 1 && tp_rank_ >= 0 && tp_rank_ < tp_world_, "bad tensor-parallel rank / world");
        if (tp_world_ > 1) {
            detail::require(prec == Precision::kFast, "tensor parallelism runs the fast (16-bit) path");
            detail::require(tp.nccl_id != nullptr, "tensor parallelism needs an NCCL id");
        }
        shard_ = tp_shard(cfg, tp_rank_, tp_world_);
        qh_l_ = shard_.q_heads;
        kvh_l_ = shard_.kv_heads;
        inter_l_ = shard_.inter;
        ModelConfig kv_cfg = cfg;
        kv_cfg.num_kv_heads = kvh_l_;
        kv_ = KvCache(kv_cfg, max_seq_len, max_batch * blocks_per_seq_);
        alloc_ = BlockAllocator(kv_.num_blocks);
        slots_.resize(max_batch);
        table_host_.assign(static_cast<size_t>(max_batch) * blocks_per_seq_, 0);
        table_dev_ = TypedDeviceBuffer<int32_t>(static_cast<int64_t>(max_batch) * blocks_per_seq_);

        const int64_t H = cfg.hidden_size, I = cfg.intermediate_size, QW = cfg.q_width();
        const bool fast = prec == Precision::kFast;
        hidden_ = TypedDeviceBuffer<float>(rows_max_ * H);
        // per-tile partial sums of squares of the residual stream (deferred norm)
        ss_ = TypedDeviceBuffer<float>(rows_max_ * ((H + kUmmaM - 1) / kUmmaM));
        q_ = TypedDeviceBuffer<float>(rows_max_ * QW);
        if (fast) {
            normed_h_ = TypedDeviceBuffer<uint16_t>(rows_max_ * H);
            attn_h_ = TypedDeviceBuffer<uint16_t>(rows_max_ * QW);
            act_h_ = TypedDeviceBuffer<uint16_t>(rows_max_ * I);
            normed_hlo_ = TypedDeviceBuffer<uint16_t>(rows_max_ * H);
            attn_hlo_ = TypedDeviceBuffer<uint16_t>(rows_max_ * QW);
            act_hlo_ = TypedDeviceBuffer<uint16_t>(rows_max_ * I);
        } else {
            normed_f_ = TypedDeviceBuffer<float>(rows_max_ * H);
            normed_lo_ = TypedDeviceBuffer<float>(rows_max_ * H);
            attn_f_ = TypedDeviceBuffer<float>(rows_max_ * QW);
            attn_lo_ = TypedDeviceBuffer<float>(rows_max_ * QW);
            act_f_ = TypedDeviceBuffer<float>(rows_max_ * I);
            act_lo_ = TypedDeviceBuffer<float>(rows_max_ * I);
        }
        // split-K partial buffer: the largest plan over every row count
        int64_t part = 0;
        const Projection *projs[4] = {&w.layers[0].qkv, &w.layers[0].o, &w.layers[0].gu, &w.layers[0].down};
        for (int r = 1; r <= rows_max_; r = (r < 64 ? r + 1 : r + 64)) {
            for (const Projection *p : projs)
                part = std::max(part, static_cast<int64_t>(plan_splits(*p, r)) * r * p->out);
        }
        for (const Projection *p : projs)
            part = std::max(part, static_cast<int64_t>(plan_splits(*p, rows_max_)) * rows_max_ * p->out);
        part_ = TypedDeviceBuffer<float>(part);
        make_views();
        if (fast && tp_world_ == 1 && chain_)
            alloc_chain();
        if (tp_world_ > 1) {
            tp_y_ = TypedDeviceBuffer<float>(rows_max_ * H);
            tp_comm_ = NcclLite::get().init(tp.nccl_id, tp_world_, tp_rank_);
            // receive slots and counters of the fused peer-to-peer reduction
            // (used once every rank has opened the others' with tp_open_peers)
            tp_recv_ = TypedDeviceBuffer<float>(2 * tp_world_ * rows_max_ * H);
            tp_cnt_ = TypedDeviceBuffer<int32_t>(4);
            OPWORKS_CUDA_CHECK(cudaMemset(tp_cnt_.data(), 0, 4 * sizeof(int32_t)));
        }
        if (fast) {
            // grouped split-K workspace: slices of up to kGroupTiles 32-token
            // tiles x 2 groups; counters zero-initialised
            groups_part_ = TypedDeviceBuffer<float>(static_cast<int64_t>(kGroupTiles) * 2 * 32 * kUmmaM);
            groups_cnt_ = TypedDeviceBuffer<int32_t>(kGroupTiles * sm100::kMaxClusterSplits);
            OPWORKS_CUDA_CHECK(cudaMemset(groups_cnt_.data(), 0, sizeof(int32_t) * kGroupTiles * sm100::kMaxClusterSplits));
            groups_ws_.partials = groups_part_.data();
            groups_ws_.floats = static_cast<size_t>(kGroupTiles) * 2 * 32 * kUmmaM;
            groups_ws_.counters = reinterpret_cast<unsigned int *>(groups_cnt_.data());
            groups_ws_.max_counters = kGroupTiles * sm100::kMaxClusterSplits;
        }
        // split-KV partials of decode attention, for every batch size
        int64_t attn_rows = 0;
        for (int n = 1; n <= max_batch; ++n) {
            const int tps = detail::decode_tokens_per_split(n * cfg.num_kv_heads, max_seq_len, sm_count_);
            attn_rows = std::max(attn_rows, static_cast<int64_t>(n) * ((max_seq_len + tps - 1) / tps));
        }
        attn_po_ = TypedDeviceBuffer<float>(attn_rows * cfg.num_q_heads * detail::kAttnD);
        attn_pml_ = TypedDeviceBuffer<float>(attn_rows * cfg.num_q_heads * 2);
        logits_ = TypedDeviceBuffer<float>(static_cast<int64_t>(max_batch) * cfg.vocab_size);
        tokens_ = TypedDeviceBuffer<int32_t>(max_batch);

        // decode and prefill stage their inputs in separate regions so a decode
        // step copies only decode-sized arrays
        dec_ = detail::StepLayout::make(max_batch, max_batch);
        pre_ = detail::StepLayout::make(prefill_rows_, 1);
        in_dev_ = TypedDeviceBuffer<uint8_t>(dec_.bytes + pre_.bytes);
        OPWORKS_CUDA_CHECK(cudaMallocHost(&in_host_, dec_.bytes + pre_.bytes));
        std::memset(in_host_, 0, dec_.bytes + pre_.bytes);
        OPWORKS_CUDA_CHECK(cudaMallocHost(reinterpret_cast<void **>(&out_host_), sizeof(int32_t) * (max_batch + 1)));
    }

    ~LlamaEngineT() {
        cudaSetDevice(device_);
        for (auto &g : graphs_)
            cudaGraphExecDestroy(g.second);
        for (auto &g : multi_graphs_)
            cudaGraphExecDestroy(g.second);
        if (tp_comm_) {
            if (stream_)
                cudaStreamSynchronize(stream_);
            NcclLite::get().destroy(tp_comm_);
        }
        for (void *p : peer_maps_)
            cudaIpcCloseMemHandle(p);
        if (stream_)
            cudaStreamSynchronize(stream_);
        if (in_host_)
            cudaFreeHost(in_host_);
        if (out_host_)
            cudaFreeHost(out_host_);
        if (stream_)
            cudaStreamDestroy(stream_);
    }
    LlamaEngineT(const LlamaEngineT &) = delete;
    LlamaEngineT &operator=(const LlamaEngineT &) = delete;

    int max_batch() const { return max_batch_; }
    int max_seq_len() const { return max_seq_len_; }
    int length(int slot) const { return slots_.at(slot).length; }
    Precision precision() const { return prec_; }
    cudaStream_t stream() const { return stream_; }
    KvCache &cache() { return kv_; }

    void reset(int slot) {
        check_slot(slot);
        Slot &s = slots_[slot];
        for (int b : s.blocks)
            alloc_.release(b);
        s.blocks.clear();
        s.length = 0;
    }

    // Runs `n` tokens of `slot` (appended after its current length) and
    // returns the next token sampled from the last position. hook(-1) after
    // the embedding and hook(l) after each layer (debugging; ids stay put).
    int32_t prefill(int slot, const int32_t *ids, int n, const SampleArgs &sa,
                    const std::function<void(int)> &hook = nullptr) {
        check_slot(slot);
        check_usable();
        detail::require(n > 0, "prefill requires at least one token");
        detail::require(ids != nullptr, "null token buffer");
        validate_ids(ids, n);
        Slot &s = slots_[slot];
        detail::require(s.length + n <= max_seq_len_, "prompt exceeds the session capacity");
        OPWORKS_CUDA_CHECK(cudaSetDevice(device_));
        ensure_blocks(slot, s.length + n);
        flush_table();
        int done = 0;
        use_layout(pre_, dec_.bytes);
        while (done < n) {
            const int rows = std::min(prefill_rows_, n - done);
            int32_t *h_ids = host_i32(layout_.ids), *h_seq = host_i32(layout_.seq), *h_pos = host_i32(layout_.pos);
            for (int r = 0; r < rows; ++r) {
                h_ids[r] = ids[done + r];
                h_seq[r] = slot;
                h_pos[r] = s.length + done + r;
            }
            const bool last = done + rows == n;
            if (last)
                stage_sampling(0, sa);
            OPWORKS_CUDA_CHECK(cudaMemcpyAsync(in_dev_.data() + base_, static_cast<char *>(in_host_) + base_,
                                               layout_.bytes, cudaMemcpyHostToDevice, stream_));
            forward(rows, /*decode=*/false, slot, s.length + done, hook);
            if (last) {
                sample(1);
                fetch_tokens(1);
            } else {
                OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream_)); // staging is reused
            }
            done += rows;
        }
        s.length += n;
        check_device_error();
        return out_host_[0];
    }

    // One decode token for each of n slots (n <= max_batch); prev[i] is the
    // token appended to slots[i]; out[i] receives the next token.
    void decode(int n, const int32_t *slots, const int32_t *prev, const SampleArgs *sa, int32_t *out) {
        detail::require(n > 0 && n <= max_batch_, "decode batch size outside the engine capacity");
        check_usable();
        OPWORKS_CUDA_CHECK(cudaSetDevice(device_));
        validate_ids(prev, n);
        use_layout(dec_, 0);
        int32_t *h_ids = host_i32(layout_.ids), *h_seq = host_i32(layout_.seq), *h_pos = host_i32(layout_.pos);
        int32_t *h_lens = host_i32(layout_.lens);
        for (int i = 0; i < n; ++i) {
            check_slot(slots[i]);
            for (int j = 0; j < i; ++j)
                detail::require(slots[j] != slots[i], "a slot appears twice in one decode step");
            const Slot &s = slots_[slots[i]];
            detail::require(s.length < max_seq_len_, "session capacity exhausted");
        }
        for (int i = 0; i < n; ++i) {
            Slot &s = slots_[slots[i]];
            ensure_blocks(slots[i], s.length + 1);
            h_ids[i] = prev[i];
            h_seq[i] = slots[i];
            h_pos[i] = s.length;
            h_lens[i] = s.length + 1;
            stage_sampling(i, sa ? sa[i] : SampleArgs{});
        }
        flush_table();
        auto it = graphs_.find(n);
        if (it == graphs_.end()) {
            // first step at this batch size runs eagerly (loads modules, sets
            // kernel attributes), then the step is captured for reuse
            decode_body(n);
            OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream_));
            cudaGraph_t graph = nullptr;
            OPWORKS_CUDA_CHECK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
            decode_body(n);
            OPWORKS_CUDA_CHECK(cudaStreamEndCapture(stream_, &graph));
            cudaGraphExec_t exec = nullptr;
            OPWORKS_CUDA_CHECK(cudaGraphInstantiate(&exec, graph, 0));
            OPWORKS_CUDA_CHECK(cudaGraphDestroy(graph));
            graphs_[n] = exec;
        } else {
            OPWORKS_CUDA_CHECK(cudaGraphLaunch(it->second, stream_));
        }
        OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream_));
        check_device_error();
        for (int i = 0; i < n; ++i) {
            slots_[slots[i]].length += 1;
            out[i] = out_host_[i];
        }
    }

    // `steps` decode tokens for each of n slots without a host round trip per
    // step: the step's CUDA graph is replayed `steps` times with the sampled
    // tokens fed back on the device (by the sampler, SampleAdvance); KV blocks for all
    // steps are reserved up front. out[k * n + i] is row i's token of step k,
    // or -1 after the row emitted `eos` (eos < 0: none); count[i] is the
    // number of tokens row i produced up to and including its eos. uniforms
    // (optional, [steps][n]) replace sa[i].uniform from the second step on.
    void decode_multi(int n, const int32_t *slots, const int32_t *prev, const SampleArgs *sa, int steps,
                      const double *uniforms, int eos, int32_t *out, int32_t *count) {
        detail::require(n > 0 && n <= max_batch_ && n <= 1024, "decode batch size outside the engine capacity");
        detail::require(steps > 0, "multi-step decode needs steps > 0");
        check_usable();
        OPWORKS_CUDA_CHECK(cudaSetDevice(device_));
        validate_ids(prev, n);
        use_layout(dec_, 0);
        int32_t *h_ids = host_i32(layout_.ids), *h_seq = host_i32(layout_.seq), *h_pos = host_i32(layout_.pos);
        int32_t *h_lens = host_i32(layout_.lens);
        for (int i = 0; i < n; ++i) {
            check_slot(slots[i]);
            for (int j = 0; j < i; ++j)
                detail::require(slots[j] != slots[i], "a slot appears twice in one decode step");
            detail::require(slots_[slots[i]].length + steps <= max_seq_len_, "session capacity exhausted");
        }
        for (int i = 0; i < n; ++i) {
            Slot &s = slots_[slots[i]];
            ensure_blocks(slots[i], s.length + steps);
            h_ids[i] = prev[i];
            h_seq[i] = slots[i];
            h_pos[i] = s.length;
            h_lens[i] = s.length + 1;
            stage_sampling(i, sa ? sa[i] : SampleArgs{});
        }
        flush_table();
        // step rows of the token and uniform buffers: steps + 1 (each step
        // reads the next row's uniforms; after the last step that value is
        // never used), at least 257 so that calls of up to 256 steps share
        // one captured graph. The graphs hold these pointers: a regrowth
        // recaptures them.
        if (multi_rows_ < steps + 1) {
            OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream_));
            for (auto &g : multi_graphs_)
                cudaGraphExecDestroy(g.second);
            multi_graphs_.clear();
            multi_rows_ = std::max(steps + 1, 257);
            multi_out_ = TypedDeviceBuffer<int32_t>(static_cast<int64_t>(multi_rows_) * max_batch_);
            multi_uni_ = TypedDeviceBuffer<uint8_t>(8 * static_cast<int64_t>(multi_rows_) * max_batch_);
        }
        if (multi_state_.size() == 0)
            multi_state_ = TypedDeviceBuffer<int32_t>(3 * static_cast<int64_t>(max_batch_));
        multi_eos_ = eos;
        multi_has_uni_ = uniforms != nullptr;
        OPWORKS_CUDA_CHECK(cudaMemcpyAsync(in_dev_.data(), in_host_, dec_.bytes, cudaMemcpyHostToDevice, stream_));
        if (uniforms)
            OPWORKS_CUDA_CHECK(cudaMemcpyAsync(multi_uni_.data(), uniforms, sizeof(double) * steps * n,
                                               cudaMemcpyHostToDevice, stream_));
        OPWORKS_CUDA_CHECK(cudaMemsetAsync(multi_state_.data(), 0, sizeof(int32_t) * 3 * max_batch_, stream_));
        // the step graph bakes in the rows, eos and whether uniforms are given
        const MultiKey key{n, eos, multi_has_uni_};
        auto it = multi_graphs_.find(key);
        if (it == multi_graphs_.end()) {
            if (graphs_.count(n) == 0) {
                // modules and kernel attributes load outside any capture
                multi_body(n);
                OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream_));
                // undo that eager step: same inputs again, counter to 0
                OPWORKS_CUDA_CHECK(cudaMemcpyAsync(in_dev_.data(), in_host_, dec_.bytes, cudaMemcpyHostToDevice,
                                                   stream_));
                OPWORKS_CUDA_CHECK(cudaMemsetAsync(multi_state_.data(), 0, sizeof(int32_t) * 3 * max_batch_,
                                                   stream_));
            }
            cudaGraph_t graph = nullptr;
            OPWORKS_CUDA_CHECK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
            multi_body(n);
            OPWORKS_CUDA_CHECK(cudaStreamEndCapture(stream_, &graph));
            cudaGraphExec_t exec = nullptr;
            OPWORKS_CUDA_CHECK(cudaGraphInstantiate(&exec, graph, 0));
            OPWORKS_CUDA_CHECK(cudaGraphDestroy(graph));
            it = multi_graphs_.emplace(key, exec).first;
        }
        for (int k = 0; k < steps; ++k)
            OPWORKS_CUDA_CHECK(cudaGraphLaunch(it->second, stream_));
        OPWORKS_CUDA_CHECK(cudaMemcpyAsync(out, multi_out_.data(), sizeof(int32_t) * steps * n,
                                           cudaMemcpyDeviceToHost, stream_));
        OPWORKS_CUDA_CHECK(cudaMemcpyAsync(count, multi_state_.data() + max_batch_, sizeof(int32_t) * n,
                                           cudaMemcpyDeviceToHost, stream_));
        OPWORKS_CUDA_CHECK(cudaMemcpyAsync(out_host_ + max_batch_, err_word_, sizeof(int32_t), cudaMemcpyDeviceToHost,
                                           stream_));
        OPWORKS_CUDA_CHECK(cudaMemsetAsync(err_word_, 0, sizeof(int32_t), stream_));
        OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream_));
        check_device_error();
        for (int i = 0; i < n; ++i)
            slots_[slots[i]].length += steps;
    }

    // Logits of row `row` of the last step (prefill: row 0 = last position).
    void copy_logits(int row, float *out, int n) {
        detail::require(n == cfg_.vocab_size, "logits buffer must hold vocab_size floats");
        detail::require(row >= 0 && row < max_batch_, "logits row outside the batch");
        OPWORKS_CUDA_CHECK(cudaSetDevice(device_));
        OPWORKS_CUDA_CHECK(cudaMemcpyAsync(out, logits_.data() + static_cast<int64_t>(row) * cfg_.vocab_size,
                                           sizeof(float) * static_cast<size_t>(n), cudaMemcpyDeviceToHost, stream_));
        OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream_));
    }

    // Bytes the host copies in / out around one decode step of n rows.
    int64_t decode_h2d_bytes() const { return dec_.bytes; }
    int64_t decode_d2h_bytes(int n) const { return static_cast<int64_t>(sizeof(int32_t)) * (n + 1); }

    // Device time of every kernel group of one decode step, measured with CUDA
    // events on the engine stream while re-running the last decode step of n
    // rows eagerly `iters` times (same inputs; rewrites the same KV entries;
    // lengths are not advanced). Returns (label, ms per step, launches per
    // step) in launch order of first appearance.
    struct KernelTime {
        std::string label;
        double ms_per_step = 0.0;
        int launches_per_step = 0;
    };
    std::vector<KernelTime> profile_decode(int n, int iters) {
        detail::require(graphs_.count(n) != 0, "profile a batch size after one decode step at that size");
        detail::require(iters > 0, "iters must be positive");
        OPWORKS_CUDA_CHECK(cudaSetDevice(device_));
        use_layout(dec_, 0);
        // the step is captured with event-record nodes between kernel groups,
        // so the measured intervals contain no host launch latency
        marks_.clear();
        marks_enabled_ = true;
        cudaGraph_t graph = nullptr;
        OPWORKS_CUDA_CHECK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
        mark("");
        forward(n, /*decode=*/true, 0, 0, nullptr);
        sample(n);
        mark("sample");
        OPWORKS_CUDA_CHECK(cudaStreamEndCapture(stream_, &graph));
        marks_enabled_ = false;
        cudaGraphExec_t exec = nullptr;
        OPWORKS_CUDA_CHECK(cudaGraphInstantiate(&exec, graph, 0));
        OPWORKS_CUDA_CHECK(cudaGraphDestroy(graph));
        std::vector<KernelTime> out;
        OPWORKS_CUDA_CHECK(cudaGraphLaunch(exec, stream_)); // warm
        for (int it = 0; it < iters; ++it) {
            OPWORKS_CUDA_CHECK(cudaGraphLaunch(exec, stream_));
            OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream_));
            for (size_t i = 1; i < marks_.size(); ++i) {
                float ms = 0.f;
                OPWORKS_CUDA_CHECK(cudaEventElapsedTime(&ms, marks_[i - 1].second, marks_[i].second));
                auto f = std::find_if(out.begin(), out.end(),
                                      [&](const KernelTime &k) { return k.label == marks_[i].first; });
                if (f == out.end()) {
                    out.push_back({marks_[i].first, 0.0, 0});
                    f = out.end() - 1;
                }
                f->ms_per_step += ms / iters;
                if (it == 0)
                    f->launches_per_step += 1;
            }
        }
        OPWORKS_CUDA_CHECK(cudaGraphExecDestroy(exec));
        for (auto &m : marks_)
            cudaEventDestroy(m.second);
        marks_.clear();
        return out;
    }

    // Residual stream of the last forward, `rows` x hidden.
    void copy_hidden(float *out, int rows) {
        OPWORKS_CUDA_CHECK(cudaSetDevice(device_));
        OPWORKS_CUDA_CHECK(cudaMemcpyAsync(out, hidden_.data(), sizeof(float) * static_cast<size_t>(rows) *
                                                                    cfg_.hidden_size,
                                           cudaMemcpyDeviceToHost, stream_));
        OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream_));
    }

    // KV inspection. Physical block ids of `slot`, as the kernels see them
    // (the device copy of the block table); writes min(count, cap) ids and
    // returns the slot's mapped block count.
    int kv_blocks(int slot, int32_t *out, int cap) {
        check_slot(slot);
        const int count = static_cast<int>(slots_[slot].blocks.size());
        const std::vector<int32_t> table = device_table_row(slot);
        for (int i = 0; i < std::min(count, cap); ++i)
            out[i] = table[i];
        return count;
    }

    // K and V of positions [pos0, pos0 + n) of `slot` in `layer`, gathered
    // through the device block table, as [n][kv_heads][head_dim] floats each
    // (post-RoPE K, as attention reads it). Positions may run past the slot's
    // length up to the end of its last mapped block.
    void read_kv(int slot, int layer, int pos0, int n, float *k_out, float *v_out) {
        check_slot(slot);
        detail::require(layer >= 0 && layer < kv_.num_layers, "layer index out of range");
        detail::require(pos0 >= 0 && n >= 0, "negative position or count");
        detail::require(static_cast<int64_t>(pos0) + n <=
                            static_cast<int64_t>(slots_[slot].blocks.size()) * kKvBlockTokens,
                        "positions past the slot's mapped KV blocks");
        const std::vector<int32_t> table = device_table_row(slot);
        const int64_t bf = kv_.block_floats(), D = kv_.head_dim, kvh = kv_.kv_heads;
        std::vector<float> kb(static_cast<size_t>(bf)), vb(static_cast<size_t>(bf));
        for (int lb = pos0 / kKvBlockTokens; lb * kKvBlockTokens < pos0 + n; ++lb) {
            const int phys = table[lb];
            detail::require(phys >= 0 && phys < kv_.num_blocks, "block table holds an invalid block id");
            copy_pool_block(layer, phys, kb.data(), vb.data());
            const int p_lo = std::max(pos0, lb * kKvBlockTokens), p_hi = std::min(pos0 + n, (lb + 1) * kKvBlockTokens);
            for (int p = p_lo; p < p_hi; ++p)
                for (int64_t h = 0; h < kvh; ++h) {
                    const int64_t src = (h * kKvBlockTokens + p % kKvBlockTokens) * D;
                    const int64_t dst = ((static_cast<int64_t>(p) - pos0) * kvh + h) * D;
                    std::memcpy(k_out + dst, kb.data() + src, sizeof(float) * D);
                    std::memcpy(v_out + dst, vb.data() + src, sizeof(float) * D);
                }
        }
    }

    // Raw pool blocks [block0, block0 + nblocks) of `layer` in pool order
    // ([block][kv_heads][16][head_dim] floats each for K and V). Returns the
    // pool's block count (nblocks = 0 only asks for it).
    int read_kv_pool(int layer, int block0, int nblocks, float *k_out, float *v_out) {
        detail::require(layer >= 0 && layer < kv_.num_layers, "layer index out of range");
        detail::require(block0 >= 0 && nblocks >= 0 && static_cast<int64_t>(block0) + nblocks <= kv_.num_blocks,
                        "block range outside the KV pool");
        const int64_t bf = kv_.block_floats();
        for (int b = 0; b < nblocks; ++b)
            copy_pool_block(layer, block0 + b, k_out + b * bf, v_out + b * bf);
        return kv_.num_blocks;
    }

  private:
    std::vector<int32_t> device_table_row(int slot) {
        std::vector<int32_t> row(static_cast<size_t>(blocks_per_seq_));
        OPWORKS_CUDA_CHECK(cudaSetDevice(device_));
        OPWORKS_CUDA_CHECK(cudaMemcpyAsync(row.data(), table_dev_.data() + static_cast<int64_t>(slot) * blocks_per_seq_,
                                           sizeof(int32_t) * row.size(), cudaMemcpyDeviceToHost, stream_));
        OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream_));
        return row;
    }
    void copy_pool_block(int layer, int block, float *k_host, float *v_host) {
        const int64_t bf = kv_.block_floats();
        OPWORKS_CUDA_CHECK(cudaSetDevice(device_));
        OPWORKS_CUDA_CHECK(cudaMemcpyAsync(k_host, kv_.k(layer) + block * bf, sizeof(float) * bf,
                                           cudaMemcpyDeviceToHost, stream_));
        OPWORKS_CUDA_CHECK(cudaMemcpyAsync(v_host, kv_.v(layer) + block * bf, sizeof(float) * bf,
                                           cudaMemcpyDeviceToHost, stream_));
        OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream_));
    }

    struct Slot {
        int length = 0;
        std::vector<int> blocks;
    };
    struct Act {
        const uint16_t *h16;    // 16-bit operand (format: w_.f16), hi term
        const uint16_t *h16_lo; // remainder term
        const float *f32;
        const float *lo;
    };

    void mark(const char *label) {
        if (!marks_enabled_)
            return;
        cudaEvent_t e;
        OPWORKS_CUDA_CHECK(cudaEventCreate(&e));
        OPWORKS_CUDA_CHECK(cudaEventRecordWithFlags(e, stream_, cudaEventRecordExternal));
        marks_.emplace_back(label, e);
    }

    void check_usable() const {
        if (!failed_.empty())
            throw std::runtime_error(failed_);
    }
    void check_slot(int slot) const {
        detail::require(slot >= 0 && slot < max_batch_, "slot outside the engine capacity");
    }
    void validate_ids(const int32_t *ids, int n) const {
        for (int i = 0; i < n; ++i)
            if (ids[i] < 0 || ids[i] >= cfg_.vocab_size)
                throw std::invalid_argument("token id outside the vocabulary");
    }
    void use_layout(const detail::StepLayout &L, int64_t base) {
        layout_ = L;
        base_ = base;
    }
    int32_t *host_i32(int64_t off) {
        return reinterpret_cast<int32_t *>(static_cast<char *>(in_host_) + base_ + off);
    }
    template <typename T> T *dev_at(int64_t off) { return reinterpret_cast<T *>(in_dev_.data() + base_ + off); }

    void stage_sampling(int row, const SampleArgs &sa) {
        char *h = static_cast<char *>(in_host_) + base_;
        reinterpret_cast<float *>(h + layout_.temp)[row] = sa.temperature;
        reinterpret_cast<float *>(h + layout_.top_p)[row] = sa.top_p;
        reinterpret_cast<double *>(h + layout_.uniform)[row] = sa.uniform;
        reinterpret_cast<uint64_t *>(h + layout_.seed)[row] = sa.seed;
        reinterpret_cast<int32_t *>(h + layout_.step)[row] = sa.step;
    }

    void ensure_blocks(int slot, int tokens) {
        Slot &s = slots_[slot];
        const int need = (tokens + kKvBlockTokens - 1) / kKvBlockTokens;
        while (static_cast<int>(s.blocks.size()) < need) {
            const int b = alloc_.alloc();
            table_host_[static_cast<size_t>(slot) * blocks_per_seq_ + s.blocks.size()] = b;
            s.blocks.push_back(b);
            table_dirty_ = true;
        }
    }
    void flush_table() {
        if (!table_dirty_)
            return;
        OPWORKS_CUDA_CHECK(cudaMemcpyAsync(table_dev_.data(), table_host_.data(),
                                           sizeof(int32_t) * table_host_.size(), cudaMemcpyHostToDevice, stream_));
        OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream_)); // host table may change next step
        table_dirty_ = false;
    }

    void decode_body(int n) {
        OPWORKS_CUDA_CHECK(cudaMemcpyAsync(in_dev_.data(), in_host_, dec_.bytes, cudaMemcpyHostToDevice, stream_));
        forward(n, /*decode=*/true, 0, 0, nullptr);
        sample(n);
        OPWORKS_CUDA_CHECK(cudaMemcpyAsync(out_host_, tokens_.data(), sizeof(int32_t) * n, cudaMemcpyDeviceToHost,
                                           stream_));
        OPWORKS_CUDA_CHECK(cudaMemcpyAsync(out_host_ + max_batch_, err_word_, sizeof(int32_t),
                                           cudaMemcpyDeviceToHost, stream_));
        OPWORKS_CUDA_CHECK(cudaMemsetAsync(err_word_, 0, sizeof(int32_t), stream_));
    }

    // one step of a multi-step decode: forward, sample, feed the tokens back
    void multi_body(int n) {
        forward(n, /*decode=*/true, 0, 0, nullptr);
        int32_t *st = multi_state_.data(); // done[max_batch] | count[max_batch] | steps taken[max_batch]
        detail::SampleAdvance adv;
        adv.ids = dev_at<int32_t>(layout_.ids);
        adv.pos = dev_at<int32_t>(layout_.pos);
        adv.lens = dev_at<int32_t>(layout_.lens);
        adv.step = dev_at<int32_t>(layout_.step);
        adv.uniform = dev_at<double>(layout_.uniform);
        adv.uniforms = multi_has_uni_ ? reinterpret_cast<const double *>(multi_uni_.data()) : nullptr;
        adv.done = st;
        adv.count = st + max_batch_;
        adv.taken = st + 2 * max_batch_;
        adv.out = multi_out_.data();
        adv.n = n;
        adv.eos = multi_eos_;
        sample(n, adv);
    }

    void fetch_tokens(int n) {
        OPWORKS_CUDA_CHECK(cudaMemcpyAsync(out_host_, tokens_.data(), sizeof(int32_t) * n, cudaMemcpyDeviceToHost,
                                           stream_));
        OPWORKS_CUDA_CHECK(cudaMemcpyAsync(out_host_ + max_batch_, err_word_, sizeof(int32_t),
                                           cudaMemcpyDeviceToHost, stream_));
        OPWORKS_CUDA_CHECK(cudaMemsetAsync(err_word_, 0, sizeof(int32_t), stream_));
        OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream_));
    }

    void check_device_error() {
        if (out_host_[max_batch_] != 0) {
            const int code = out_host_[max_batch_];
            out_host_[max_batch_] = 0;
            if (code == detail::kErrTpPeerTimeout)
                failed_ = "a tensor-parallel peer exchange timed out; recreate the batch on every rank";
            throw std::runtime_error("a device-side wait timed out in the forward pass (code " +
                                     std::to_string(code) + ")");
        }
    }

    // ------------------------------------------------------------ forward

    bool fast() const { return prec_ == Precision::kFast; }

    int plan_bn(int rows) const { return sm100::gemm_pick_bn(sm100::GemmKind::kBF16x2, rows); }
    // the fused GEMM of `rows` token rows runs narrow (BN <= 64) tiles, whose
    // epilogue scratch can hold rows preloaded during the main loop
    bool narrow_tile(int rows) const { return rows <= prefill_single_rows_ && plan_bn(rows) <= 64; }

    // A 16-bit weight operand: `out` rows of `in` elements, row stride ld
    // (a column slice of a wider matrix keeps the matrix's stride).
    struct WView {
        const uint16_t *w = nullptr;
        int out = 0, in = 0;
        int64_t ld = 0;
    };
    static WView view(const Projection &p) { return {p.w16.data(), p.out, p.in, p.in}; }
    // GEMM operands in the model's 16-bit format
    sm100::GemmOperand wop(const WView &p) const { return {p.w, nullptr, p.out, p.ld, w_.f16}; }
    sm100::GemmOperand xop(const Act &x, int rows, int64_t ld, bool two_term = true) const {
        return {x.h16, two_term ? x.h16_lo : nullptr, rows, ld, w_.f16};
    }

    // this rank's slices of the fast path's projections: QKV rows of its q,
    // k and v heads (a compact copy), O and down input-column slices (views),
    // gate/up rows of its interleaved MLP pairs (a view)
    void make_views() {
        if (!fast())
            return;
        const int H = cfg_.hidden_size, I = cfg_.intermediate_size;
        for (int l = 0; l < cfg_.num_layers; ++l) {
            const LayerWeights<WT> &L = w_.layers[l];
            if (tp_world_ == 1) {
                qkv_v_.push_back(view(L.qkv));
                o_v_.push_back(view(L.o));
                gu_v_.push_back(view(L.gu));
                down_v_.push_back(view(L.down));
                continue;
            }
            const TpShard &sh = shard_;
            const int qrows = static_cast<int>(sh.q_rows), kvrows = static_cast<int>(sh.kv_rows);
            tp_qkv_.emplace_back(static_cast<int64_t>(qrows + 2 * kvrows) * H);
            uint16_t *dst = tp_qkv_.back().data();
            const uint16_t *src = L.qkv.w16.data();
            const int64_t from[3] = {sh.q_row0, sh.k_row0, sh.v_row0};
            const int64_t count[3] = {qrows, kvrows, kvrows};
            int64_t at = 0;
            for (int i = 0; i < 3; ++i) {
                OPWORKS_CUDA_CHECK(cudaMemcpy(dst + at * H, src + from[i] * H,
                                              sizeof(uint16_t) * static_cast<size_t>(count[i] * H),
                                              cudaMemcpyDeviceToDevice));
                at += count[i];
            }
            qkv_v_.push_back({dst, qrows + 2 * kvrows, H, H});
            o_v_.push_back({L.o.w16.data() + sh.o_col0, H, qrows, cfg_.q_width()});
            gu_v_.push_back({L.gu.w16.data() + sh.gu_row0 * H, static_cast<int>(sh.gu_rows), H, H});
            down_v_.push_back({L.down.w16.data() + sh.down_col0, H, sh.inter, I});
        }
    }

    // ---- persistent decode chain (O, gate/up, down, next QKV in one launch)
    // phase p's (tiles, K blocks) for this model
    void chain_shape(int ph, int &tiles, int &nk) const {
        const int H = cfg_.hidden_size, I = cfg_.intermediate_size;
        const int rows_out[4] = {H, 2 * I, H, cfg_.qkv_width()};
        const int k[4] = {cfg_.q_width(), H, I, H};
        tiles = (rows_out[ph] + kUmmaM - 1) / kUmmaM;
        nk = (k[ph] + 63) / 64;
    }
    void alloc_chain() {
        // CTAs streaming each phase: O and QKV fewer (their weights fit the
        // rings of the active CTAs; the idle CTAs load the next phase's
        // weights early), gate/up and down all
        int want[4] = {64, sm_count_, 128, 96};
        if (const char *e = std::getenv("OPWORKS_CHAIN_ACTIVE"))
            std::sscanf(e, "%d,%d,%d,%d", &want[0], &want[1], &want[2], &want[3]);
        for (int ph = 0; ph < 4; ++ph) {
            int tiles = 0, nk = 0;
            chain_shape(ph, tiles, nk);
            chain_active_[ph] = std::max(1, std::min(want[ph], sm_count_));
            const int parts = sm100::chain_max_parts(tiles, nk, chain_active_[ph]);
            if (parts > 1) {
                chain_part_[ph] = TypedDeviceBuffer<float>(static_cast<int64_t>(tiles) * parts * sm100::kChainBN * kUmmaM);
                chain_cnt_[ph] = TypedDeviceBuffer<int32_t>(tiles);
                OPWORKS_CUDA_CHECK(cudaMemset(chain_cnt_[ph].data(), 0, sizeof(int32_t) * tiles));
            }
        }
        chain_sync_ = TypedDeviceBuffer<int32_t>(2);
        OPWORKS_CUDA_CHECK(cudaMemset(chain_sync_.data(), 0, 2 * sizeof(int32_t)));
    }
    bool use_chain(int rows, bool decode) const {
        return chain_ && fast() && tp_world_ == 1 && decode && rows <= sm100::kChainBN;
    }
    template <typename E3>
    void chain_launch(int l, int rows, const Act &attn, const Act &normed, const Act &act, const detail::ActOut &normed_o,
                      const detail::ActOut &act_o, const detail::RowSumSq &rs, const float *next_gain, int nphases,
                      const E3 &e3) {
        const int H = cfg_.hidden_size, I = cfg_.intermediate_size;
        auto part = [&](int ph) { return chain_part_[ph].size() ? chain_part_[ph].data() : nullptr; };
        auto cnt = [&](int ph) {
            return chain_cnt_[ph].size() ? reinterpret_cast<unsigned *>(chain_cnt_[ph].data()) : nullptr;
        };
        sm100::ChainGemm g[4];
        g[0] = {wop(o_v_[l]), xop(attn, rows, cfg_.q_width()), cfg_.q_width(), chain_active_[0], part(0), cnt(0)};
        g[1] = {wop(gu_v_[l]), xop(normed, rows, H), H, chain_active_[1], part(1), cnt(1)};
        g[2] = {wop(down_v_[l]), xop(act, rows, I), I, chain_active_[2], part(2), cnt(2)};
        if (nphases == 4)
            g[3] = {wop(qkv_v_[l + 1]), xop(normed, rows, H), H, chain_active_[3], part(3), cnt(3)};
        const LayerWeights<WT> &L = w_.layers[l];
        sm100::decode_chain_launch(g, nphases, sm_count_, reinterpret_cast<unsigned *>(chain_sync_.data()), stream_,
                                   detail::ResidualTileEpi{hidden_.data(), H, L.post_norm.data(), normed_o, rs, false},
                                   detail::SiluMulTileEpi{act_o, rs},
                                   detail::ResidualTileEpi{hidden_.data(), H, next_gain, normed_o, rs, false}, e3);
    }

    int plan_splits(const WView &p, int rows, int max_splits = 64) const {
        if (!fast() && rows <= 4)
            return 1;
        const int bn = fast() ? plan_bn(rows) : sm100::gemm_pick_bn(sm100::GemmKind::kTF32x3, rows);
        const int tiles = ((p.out + kUmmaM - 1) / kUmmaM) * ((rows + bn - 1) / bn);
        const int kb = fast() ? (p.in + 63) / 64 : (p.in + 31) / 32;
        return sm100::gemm_pick_splits(tiles, kb, sm_count_ * sm100::gemm_ctas_per_sm(bn), fast() ? 2 : 8,
                                       max_splits);
    }

    int plan_splits(const Projection &p, int rows, int max_splits = 64) const {
        if (!fast() && rows <= 4)
            return 1;
        const int bn = fast() ? plan_bn(rows) : sm100::gemm_pick_bn(sm100::GemmKind::kTF32x3, rows);
        const int tiles = ((p.out + kUmmaM - 1) / kUmmaM) * ((rows + bn - 1) / bn);
        const int kb = fast() ? (p.in + 63) / 64 : (p.in + 31) / 32;
        return sm100::gemm_pick_splits(tiles, kb, sm_count_ * sm100::gemm_ctas_per_sm(bn), fast() ? 2 : 8,
                                       max_splits);
    }

    // fast path: x . W^T with the split-K reduction and `epi` fused into the
    // GEMM (K splits of a tile form one cluster)
    // `next` (optional): the projection that streams after this one; its
    // weights are pulled into L2 while this GEMM runs (latency-bound decode
    // GEMMs leave HBM bandwidth idle)
    // `which` (0 QKV, 1 O, 2 gate/up, 3 down) selects a per-projection cap
    // on the K splits (OPWORKS_SPLITS_QKV / _O / _GU / _DOWN; default: the
    // cluster bound)
    template <typename Epi>
    void linear_tile(const WView &p, const Act &x, int rows, const Epi &epi, const WView *next = nullptr,
                     int which = -1) {
        const bool single = rows > prefill_single_rows_;
        if (rows >= pair_min_rows_) {
            // prefill-sized GEMMs: two-SM 256 x 256 tiles (cta_group::2);
            // one activation term (one MMA per K step) above the threshold
            sm100::gemm_pair_bf16x2<Epi>(wop(p), xop(x, rows, p.in, !single), p.in, stream_, epi);
            return;
        }
        if (single) {
            // single-term 16-bit activations (one MMA per K step, 256-token
            // tiles), compute-bound shapes
            sm100::gemm_tn<sm100::GemmKind::kBF16, Epi>(wop(p), xop(x, rows, p.in, false), p.in, part_.data(), p.out, 1,
                                                        static_cast<int64_t>(rows) * p.out, stream_, epi,
                                                        sm100::gemm_pick_bn(sm100::GemmKind::kBF16, rows));
            return;
        }
        const int cap = which >= 0 && split_cap_[which] > 0 ? std::min(split_cap_[which], max_cluster_splits_)
                                                            : max_cluster_splits_;
        int splits = plan_splits(p, rows, cap);
        const bool pf = next != nullptr && l2_prefetch_ && rows <= 64;
        const uint64_t pf_bytes = pf ? sizeof(uint16_t) * static_cast<uint64_t>(next->out) * next->ld : 0;
        // grids of at most one CTA per SM (16 tiles x 8 splits at C3) double
        // their splits as two clusters per tile, reduced across clusters
        // through L2, so twice the weight bytes are in flight
        int cluster = 0;
        if (split_groups_ > 0 && plan_bn(rows) == 32 && splits == sm100::kMaxClusterSplits) {
            const int tiles = (p.out + kUmmaM - 1) / kUmmaM;
            const int kb = (p.in + 63) / 64;
            if (tiles * 2 * splits <= 2 * sm_count_ && tiles * splits <= sm_count_ &&
                kb >= (split_groups_ >= 2 ? 32 : 64) && tiles * 2 <= kGroupTiles) {
                cluster = splits;
                splits *= 2;
            }
        }
        if (cluster > 0) {
            sm100::gemm_tn<sm100::GemmKind::kBF16x2, Epi>(
                wop(p), xop(x, rows, p.in), p.in, part_.data(), p.out, splits,
                static_cast<int64_t>(rows) * p.out, stream_, epi, 32, pf ? next->w : nullptr, pf_bytes, &groups_ws_,
                cluster, l2_prefetch_tail_);
            return;
        }
        sm100::gemm_tn<sm100::GemmKind::kBF16x2, Epi>(
            wop(p), xop(x, rows, p.in), p.in, part_.data(), p.out, splits,
            static_cast<int64_t>(rows) * p.out, stream_, epi, plan_bn(rows), pf ? next->w : nullptr, pf_bytes, nullptr,
            0, l2_prefetch_tail_);
    }

    // part[s][rows][p.out] = x[rows][p.in] . W^T (partial over split s)
    int linear(const Projection &p, const Act &x, int rows) {
        const int splits = plan_splits(p, rows);
        if (fast()) {
            sm100::gemm_tn<sm100::GemmKind::kBF16x2>(wop(view(p)), xop(x, rows, p.in), p.in, part_.data(), p.out,
                                                     splits, static_cast<int64_t>(rows) * p.out, stream_,
                                                     sm100::Identity{}, plan_bn(rows));
        } else if (rows <= 4) {
            detail::gemv_rows_launch<float>(x.f32, p.in, p.f32.data(), part_.data(), p.out, rows, p.in, p.out,
                                            stream_);
        } else {
            sm100::gemm_tn<sm100::GemmKind::kTF32x3>(
                {p.hi.data(), p.lo.data(), p.out, p.in}, {x.f32, x.lo, rows, p.in}, p.in, part_.data(), p.out, splits,
                static_cast<int64_t>(rows) * p.out, stream_, sm100::Identity{},
                sm100::gemm_pick_bn(sm100::GemmKind::kTF32x3, rows));
        }
        return splits;
    }

    detail::ActOut act_out(uint16_t *h, uint16_t *hlo, float *f, float *lo, int64_t ld, int rows) const {
        detail::ActOut o;
        o.ld = ld;
        if (fast()) {
            o.h16 = h;
            o.h16_lo = hlo;
            o.f16 = w_.f16;
        } else {
            o.f32 = f;
            o.lo = rows > 4 ? lo : nullptr;
        }
        return o;
    }

    template <int kPer>
    void launch_add_rmsnorm(int rows, int splits, const float *w, const detail::ActOut &o) {
        launch_ex(detail::add_rmsnorm_kernel<kPer>, dim3(rows), dim3(detail::kRowThreads), 0, stream_, hidden_.data(),
                  static_cast<const float *>(part_.data()), splits, static_cast<int64_t>(rows) * cfg_.hidden_size, w,
                  cfg_.rms_norm_eps, o, cfg_.hidden_size);
    }
    void add_rmsnorm(int rows, int splits, const float *w, const detail::ActOut &o) {
        switch (cfg_.hidden_size / detail::kRowThreads) {
        case 1: launch_add_rmsnorm<1>(rows, splits, w, o); break;
        case 2: launch_add_rmsnorm<2>(rows, splits, w, o); break;
        case 4: launch_add_rmsnorm<4>(rows, splits, w, o); break;
        case 8: launch_add_rmsnorm<8>(rows, splits, w, o); break;
        case 16: launch_add_rmsnorm<16>(rows, splits, w, o); break;
        default: throw std::invalid_argument("unsupported hidden size");
        }
        OPWORKS_CUDA_CHECK(cudaGetLastError());
    }
    template <int kPer, typename T> void launch_embed(int rows, const T *table, const detail::ActOut &o) {
        detail::embed_rmsnorm_kernel<kPer, T><<<rows, detail::kRowThreads, 0, stream_>>>(
            table, dev_at<int32_t>(layout_.ids), hidden_.data(), w_.layers[0].input_norm.data(), cfg_.rms_norm_eps, o,
            cfg_.hidden_size, fast() ? row_sumsq() : detail::RowSumSq{});
    }
    // deferred RMSNorm bookkeeping of the fast path (see detail::RowSumSq)
    detail::RowSumSq row_sumsq() {
        detail::RowSumSq rs;
        rs.part = ss_.data();
        rs.ld = rows_max_;
        rs.tiles = (cfg_.hidden_size + kUmmaM - 1) / kUmmaM;
        rs.cols = cfg_.hidden_size;
        rs.eps = cfg_.rms_norm_eps;
        return rs;
    }
    template <typename T> void embed(int rows, const T *table, const detail::ActOut &o) {
        switch (cfg_.hidden_size / detail::kRowThreads) {
        case 1: launch_embed<1>(rows, table, o); break;
        case 2: launch_embed<2>(rows, table, o); break;
        case 4: launch_embed<4>(rows, table, o); break;
        case 8: launch_embed<8>(rows, table, o); break;
        case 16: launch_embed<16>(rows, table, o); break;
        default: throw std::invalid_argument("unsupported hidden size");
        }
        OPWORKS_CUDA_CHECK(cudaGetLastError());
    }

    template <int kRep>
    void attention(int layer, int rows, bool decode, int slot, int pos0, const detail::PagedKV &kv,
                   const detail::ActOut &out) {
        const float scale = 1.f / std::sqrt(static_cast<float>(cfg_.head_dim));
        const int kvh = kvh_l_, qw = qh_l_ * cfg_.head_dim; // this rank's heads
        if (decode) {
            const int tps = detail::decode_tokens_per_split(rows * kvh, max_seq_len_, sm_count_);
            const int splits = (max_seq_len_ + tps - 1) / tps;
            detail::attn_decode_launch<detail::PagedKV, kRep, detail::ActOut>(
                q_.data(), qw, kv, dev_at<int32_t>(layout_.lens), rows, kvh, tps, splits, scale, attn_po_.data(),
                attn_pml_.data(), out, stream_);
        } else if (fast() && tc_prefill_) {
            // tensor-core (TF32) flash attention over the paged cache
            if (kv_maps_.empty()) {
                for (int l = 0; l < cfg_.num_layers; ++l)
                    kv_maps_.push_back(detail::make_kv_pool_maps(kv_.k(l), kv_.v(l), kv_.num_blocks, kvh));
            }
            detail::attn_prefill_tc_launch<kRep, detail::ActOut>(q_.data(), qw, qh_l_, kv_maps_[layer], kv.table,
                                                                 kv.table_stride, kvh, slot, rows, pos0, scale, out,
                                                                 stream_);
        } else {
            detail::attn_prefill_launch<detail::PagedKV, kRep, detail::ActOut>(q_.data(), qw, detail::kAttnD, out, kv,
                                                                               slot, rows, pos0, kvh, scale, stream_);
        }
    }

  public:
    // CUDA IPC handles of this rank's receive buffer and counters (2 x 64
    // bytes) for the fused peer-to-peer reduction of a tensor-parallel engine
    void tp_ipc_handles(char *out) const {
        detail::require(tp_world_ > 1, "not a tensor-parallel engine");
        cudaIpcMemHandle_t h[2];
        OPWORKS_CUDA_CHECK(cudaIpcGetMemHandle(&h[0], const_cast<float *>(tp_recv_.data())));
        OPWORKS_CUDA_CHECK(cudaIpcGetMemHandle(&h[1], const_cast<int32_t *>(tp_cnt_.data())));
        std::memcpy(out, h, sizeof(h));
    }
    // handles of every rank (world x 128 bytes, in rank order): maps the
    // peers' buffers; the projections then reduce through peer stores
    // instead of NCCL (OPWORKS_TP_P2P=0 keeps NCCL)
    void tp_open_peers(const char *all) {
        detail::require(tp_world_ > 1 && tp_world_ <= detail::kTpMaxWorld, "not a tensor-parallel engine");
        OPWORKS_CUDA_CHECK(cudaSetDevice(device_));
        OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream_)); // no captured step in flight
        // steps captured so far (NCCL, or earlier mappings) are captured again
        for (auto &g : graphs_)
            cudaGraphExecDestroy(g.second);
        graphs_.clear();
        for (auto &g : multi_graphs_)
            cudaGraphExecDestroy(g.second);
        multi_graphs_.clear();
        tp_p2p_ = false;
        for (void *p : peer_maps_) // a second call maps the handles afresh
            OPWORKS_CUDA_CHECK(cudaIpcCloseMemHandle(p));
        peer_maps_.clear();
        detail::TpPeers pe;
        pe.world = tp_world_;
        pe.rank = tp_rank_;
        pe.slot_floats = static_cast<int64_t>(rows_max_) * cfg_.hidden_size;
        for (int r = 0; r < tp_world_; ++r) {
            if (r == tp_rank_) {
                pe.recv[r] = tp_recv_.data();
                pe.cnt[r] = reinterpret_cast<unsigned int *>(tp_cnt_.data());
                continue;
            }
            cudaIpcMemHandle_t h[2];
            std::memcpy(h, all + 128 * r, sizeof(h));
            void *recv = nullptr, *cnt = nullptr;
            OPWORKS_CUDA_CHECK(cudaIpcOpenMemHandle(&recv, h[0], cudaIpcMemLazyEnablePeerAccess));
            peer_maps_.push_back(recv);
            OPWORKS_CUDA_CHECK(cudaIpcOpenMemHandle(&cnt, h[1], cudaIpcMemLazyEnablePeerAccess));
            peer_maps_.push_back(cnt);
            pe.recv[r] = static_cast<float *>(recv);
            pe.cnt[r] = static_cast<unsigned int *>(cnt);
        }
        tp_peers_ = pe;
        const char *e = std::getenv("OPWORKS_TP_P2P");
        tp_p2p_ = !(e && e[0] == '0');
    }

  private:
    // sum tp_y_ over the ranks, then hidden += y, the next operand and the
    // tiles' sums of squares (tp_residual_kernel)
    void tp_residual(int rows, const float *gain, const detail::ActOut &normed_o, const detail::RowSumSq &rs) {
        NcclLite::get().allreduce_sum(tp_y_.data(), static_cast<size_t>(rows) * cfg_.hidden_size, tp_comm_, stream_);
        launch_ex(detail::tp_residual_kernel, dim3(rows), dim3(128), 0, stream_, hidden_.data(),
                  static_cast<const float *>(tp_y_.data()), cfg_.hidden_size, gain, normed_o, rs);
    }

    void tp_p2p_residual(int rows, int parity, const float *gain, const detail::ActOut &normed_o,
                         const detail::RowSumSq &rs) {
        unsigned int *cnt = reinterpret_cast<unsigned int *>(tp_cnt_.data());
        launch_ex(detail::tp_p2p_residual_kernel, dim3(rows), dim3(128), 0, stream_, hidden_.data(),
                  static_cast<const float *>(tp_recv_.data()), cnt, cnt + 2, parity, tp_world_,
                  tp_peers_.slot_floats, rows, cfg_.hidden_size, gain, normed_o, rs, err_word_, tp_wait_ns_);
    }

    void forward(int rows, bool decode, int slot, int pos0, const std::function<void(int)> &hook) {
        const PdlScope pdl(pdl_);
        const int H = cfg_.hidden_size, I = inter_l_, QW = qh_l_ * cfg_.head_dim; // this rank's widths
        const int qh = qh_l_, kvh = kvh_l_;
        const detail::ActOut normed_o =
            act_out(normed_h_.data(), normed_hlo_.data(), normed_f_.data(), normed_lo_.data(), H, rows);
        const detail::ActOut attn_o = act_out(attn_h_.data(), attn_hlo_.data(), attn_f_.data(), attn_lo_.data(), QW, rows);
        const detail::ActOut act_o = act_out(act_h_.data(), act_hlo_.data(), act_f_.data(), act_lo_.data(), I, rows);
        const Act normed{normed_o.h16, normed_o.h16_lo, normed_o.f32, normed_o.lo};
        const Act attn{attn_o.h16, attn_o.h16_lo, attn_o.f32, attn_o.lo};
        const Act act{act_o.h16, act_o.h16_lo, act_o.f32, act_o.lo};

        if (w_.embed_f32.size() > 0)
            embed(rows, w_.embed_f32.data(), normed_o);
        else // bfloat16 packs: the table's words are bf16
            embed(rows, reinterpret_cast<const __nv_bfloat16 *>(w_.embed_w16.data()), normed_o);
        mark("embed_rmsnorm");
        if (hook) {
            OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream_));
            hook(-1);
        }
        const detail::TokenMap tm{dev_at<int32_t>(layout_.seq), dev_at<int32_t>(layout_.pos)};
        for (int l = 0; l < cfg_.num_layers; ++l) {
            const LayerWeights<WT> &L = w_.layers[l];
            const detail::PagedKV kv{kv_.k(l), kv_.v(l), table_dev_.data(), blocks_per_seq_, kvh};
            const float2 *rope = reinterpret_cast<const float2 *>(w_.rope_table.data());
            int s = 0;
            const detail::RowSumSq rs = row_sumsq();
            const bool chain = use_chain(rows, decode);
            if (fast() && chain && l > 0) {
                // this layer's QKV ran as the last phase of the previous chain
            } else if (fast()) {
                linear_tile(qkv_v_[l], normed, rows,
                            detail::QkvTileEpi{q_.data(), qh, kvh, rope, tm, kv, kv_.k(l), kv_.v(l), rs, narrow_tile(rows)},
                            l2_prefetch_qkv_o_ ? &o_v_[l] : nullptr, 0);
                mark("gemm_qkv_rope_kv_write");
            } else {
                s = linear(L.qkv, normed, rows);
                mark("gemm_qkv");
                launch_ex(detail::qkv_finalize_kernel, dim3(rows), dim3(256), 0, stream_,
                          static_cast<const float *>(part_.data()), s, static_cast<int64_t>(rows) * L.qkv.out, qh,
                          kvh, rope, tm, kv, kv_.k(l), kv_.v(l), q_.data());
                mark("qkv_rope_kv_write");
            }
            switch (cfg_.kv_rep()) {
            case 1: attention<1>(l, rows, decode, slot, pos0, kv, attn_o); break;
            case 2: attention<2>(l, rows, decode, slot, pos0, kv, attn_o); break;
            case 4: attention<4>(l, rows, decode, slot, pos0, kv, attn_o); break;
            default: attention<8>(l, rows, decode, slot, pos0, kv, attn_o); break;
            }
            mark("attention");
            if (fast()) {
                // the residual epilogues also emit the next projection's
                // operand h * gain and the tiles' sums of squares; the
                // consuming epilogues apply the norm's per-token scale
                const float *next_gain =
                    l + 1 < cfg_.num_layers ? w_.layers[l + 1].input_norm.data() : w_.final_norm.data();
                if (tp_world_ > 1 && tp_p2p_) {
                    // partial projection outputs stored into every rank's
                    // receive slot by the GEMM epilogue (peer memory), then
                    // the rank-order sum and the residual step
                    linear_tile(o_v_[l], attn, rows, detail::PeerStoreTileEpi{tp_peers_, 0, H});
                    tp_p2p_residual(rows, 0, L.post_norm.data(), normed_o, rs);
                    mark("gemm_o_p2p_reduce_residual");
                    linear_tile(gu_v_[l], normed, rows, detail::SiluMulTileEpi{act_o, rs});
                    mark("gemm_gate_up_silu");
                    linear_tile(down_v_[l], act, rows, detail::PeerStoreTileEpi{tp_peers_, 1, H});
                    tp_p2p_residual(rows, 1, next_gain, normed_o, rs);
                    mark("gemm_down_p2p_reduce_residual");
                } else if (tp_world_ > 1) {
                    // partial projection outputs, summed over the ranks,
                    // then the residual step of the fused epilogue
                    linear_tile(o_v_[l], attn, rows, sm100::StoreTileEpi<sm100::Identity>{tp_y_.data(), H, {}});
                    tp_residual(rows, L.post_norm.data(), normed_o, rs);
                    mark("gemm_o_allreduce_residual");
                    linear_tile(gu_v_[l], normed, rows, detail::SiluMulTileEpi{act_o, rs});
                    mark("gemm_gate_up_silu");
                    linear_tile(down_v_[l], act, rows, sm100::StoreTileEpi<sm100::Identity>{tp_y_.data(), H, {}});
                    tp_residual(rows, next_gain, normed_o, rs);
                    mark("gemm_down_allreduce_residual");
                } else if (chain) {
                    if (l + 1 < cfg_.num_layers) {
                        const detail::PagedKV kv1{kv_.k(l + 1), kv_.v(l + 1), table_dev_.data(), blocks_per_seq_, kvh};
                        chain_launch(l, rows, attn, normed, act, normed_o, act_o, rs, next_gain, 4,
                                     detail::QkvTileEpi{q_.data(), qh, kvh, rope, tm, kv1, kv_.k(l + 1), kv_.v(l + 1),
                                                        rs, false});
                    } else {
                        chain_launch(l, rows, attn, normed, act, normed_o, act_o, rs, next_gain, 3,
                                     sm100::NoTileEpi{});
                    }
                    mark("decode_chain");
                } else {
                    linear_tile(o_v_[l], attn, rows,
                                detail::ResidualTileEpi{hidden_.data(), H, L.post_norm.data(), normed_o, rs,
                                                        narrow_tile(rows)},
                                &gu_v_[l], 1);
                    mark("gemm_o_residual");
                    linear_tile(gu_v_[l], normed, rows, detail::SiluMulTileEpi{act_o, rs}, &down_v_[l], 2);
                    mark("gemm_gate_up_silu");
                    linear_tile(down_v_[l], act, rows,
                                detail::ResidualTileEpi{hidden_.data(), H, next_gain, normed_o, rs, narrow_tile(rows)},
                                l + 1 < cfg_.num_layers ? &qkv_v_[l + 1] : nullptr, 3);
                    mark("gemm_down_residual");
                }
            } else {
                s = linear(L.o, attn, rows);
                mark("gemm_o");
                add_rmsnorm(rows, s, L.post_norm.data(), normed_o);
                mark("residual_rmsnorm");
                s = linear(L.gu, normed, rows);
                mark("gemm_gate_up");
                launch_ex(detail::silu_mul_kernel, dim3(detail::grid_for(static_cast<int64_t>(rows) * I)),
                          dim3(kThreads), 0, stream_, static_cast<const float *>(part_.data()), s,
                          static_cast<int64_t>(rows) * L.gu.out, rows, I, act_o);
                mark("silu_mul");
                s = linear(L.down, act, rows);
                mark("gemm_down");
            }
            if (!fast()) {
                if (l + 1 < cfg_.num_layers) {
                    add_rmsnorm(rows, s, w_.layers[l + 1].input_norm.data(), normed_o);
                } else {
                    // the final norm feeds only the LM head, which reads full
                    // fp32 on the accurate path (never the tf32 hi/lo split)
                    detail::ActOut final_o = normed_o;
                    final_o.lo = nullptr;
                    add_rmsnorm(rows, s, w_.final_norm.data(), final_o);
                }
                mark("residual_rmsnorm");
            }
            if (hook) {
                OPWORKS_CUDA_CHECK(cudaStreamSynchronize(stream_));
                hook(l);
            }
        }
        // LM head: every row of a decode step, the last row of a prefill
        const int lrows = decode ? rows : 1;
        const int64_t first = decode ? 0 : rows - 1;
        const int V = cfg_.vocab_size;
        if (fast()) {
            // deferred final norm: the epilogue scales each row's logits
            sm100::gemm_tn<sm100::GemmKind::kBF16x2, detail::LogitsTileEpi>(
                {w_.embed_w16.data(), nullptr, V, H, w_.f16},
                {normed_h_.data() + first * H, normed_hlo_.data() + first * H, lrows, H, w_.f16}, H, logits_.data(), V,
                lm_head_splits_, 0, stream_, detail::LogitsTileEpi{logits_.data(), V, row_sumsq(), first},
                plan_bn(lrows));
        } else {
            for (int r0 = 0; r0 < lrows; r0 += 4) {
                const int r = std::min(4, lrows - r0);
                detail::gemv_rows_launch<float>(normed_f_.data() + (first + r0) * H, H, w_.embed_f32.data(),
                                                logits_.data() + static_cast<int64_t>(r0) * V, V, r, H, V, stream_);
            }
        }
        mark("lm_head");
    }

    void sample(int rows, const detail::SampleAdvance &adv = {}) {
        const PdlScope pdl(pdl_);
        detail::SampleParams sp;
        sp.temperature = dev_at<float>(layout_.temp);
        sp.top_p = dev_at<float>(layout_.top_p);
        sp.uniform = dev_at<double>(layout_.uniform);
        sp.seed = dev_at<uint64_t>(layout_.seed);
        sp.step = dev_at<int32_t>(layout_.step);
        detail::sample_launch(logits_.data(), cfg_.vocab_size, rows, cfg_.vocab_size, sp, tokens_.data(), stream_, adv);
    }

    ModelConfig cfg_;
    const ModelWeights<WT> &w_;
    Precision prec_;
    int max_batch_, max_seq_len_, prefill_rows_ = 0, rows_max_ = 0, blocks_per_seq_ = 0;
    int device_ = 0, sm_count_ = 0;
    cudaStream_t stream_ = nullptr;
    int *err_word_ = nullptr;
    KvCache kv_;
    BlockAllocator alloc_;
    std::vector<Slot> slots_;
    std::vector<int32_t> table_host_;
    TypedDeviceBuffer<int32_t> table_dev_;
    bool table_dirty_ = true;
    TypedDeviceBuffer<float> hidden_, ss_, q_, part_, attn_po_, attn_pml_, logits_;
    // tensor parallelism (tp_world_ == 1: the whole model on this GPU)
    int tp_rank_ = 0, tp_world_ = 1, qh_l_ = 0, kvh_l_ = 0, inter_l_ = 0;
    TpShard shard_;
    ncclComm_t tp_comm_ = nullptr;
    TypedDeviceBuffer<float> tp_y_, tp_recv_;
    TypedDeviceBuffer<int32_t> tp_cnt_; // arrival counters [2] | done counters [2]
    detail::TpPeers tp_peers_{};
    bool tp_p2p_ = false;
    std::string failed_; // set when the engine can take no further step
    // persistent decode chain (OPWORKS_CHAIN=1): CTAs per phase, split-K
    // partials and counters per phase, the phase barrier
    bool chain_ = [] {
        const char *e = std::getenv("OPWORKS_CHAIN");
        return e && e[0] == '1';
    }();
    int chain_active_[4] = {0, 0, 0, 0};
    TypedDeviceBuffer<float> chain_part_[4];
    TypedDeviceBuffer<int32_t> chain_cnt_[4];
    TypedDeviceBuffer<int32_t> chain_sync_;
    // limit of the cross-rank wait of the peer-store reduction
    unsigned long long tp_wait_ns_ = [] {
        const char *e = std::getenv("OPWORKS_TP_WAIT_MS");
        const long long ms = e ? std::atoll(e) : 0;
        return ms > 0 ? static_cast<unsigned long long>(ms) * 1000000ull : detail::kTpPeerWaitNs;
    }();
    std::vector<void *> peer_maps_;
    std::vector<TypedDeviceBuffer<uint16_t>> tp_qkv_;
    std::vector<WView> qkv_v_, o_v_, gu_v_, down_v_;
    static constexpr int kGroupTiles = 64;
    TypedDeviceBuffer<float> groups_part_;
    TypedDeviceBuffer<int32_t> groups_cnt_;
    sm100::SplitGroupWorkspace groups_ws_{};
    // grouped split K for narrow decode GEMMs whose 8-split grid leaves SMs
    // idle: 0 off, 1 long K only (>= 64 blocks: the down projection at C3),
    // 2 also K >= 32 blocks (O); OPWORKS_SPLIT_GROUPS overrides
    int split_groups_ = [] {
        const char *e = std::getenv("OPWORKS_SPLIT_GROUPS");
        return e ? std::atoi(e) : 1;
    }();
    // fast path: two-term 16-bit operands (format w_.f16)
    TypedDeviceBuffer<uint16_t> normed_h_, attn_h_, act_h_, normed_hlo_, attn_hlo_, act_hlo_;
    TypedDeviceBuffer<float> normed_f_, normed_lo_, attn_f_, attn_lo_, act_f_, act_lo_;
    TypedDeviceBuffer<int32_t> tokens_;
    detail::StepLayout layout_{}, dec_{}, pre_{};
    int64_t base_ = 0;
    TypedDeviceBuffer<uint8_t> in_dev_;
    void *in_host_ = nullptr;
    int32_t *out_host_ = nullptr;
    std::map<int, cudaGraphExec_t> graphs_;
    // multi-step decode: graphs keyed by (rows, eos, uniforms given); the
    // step count is the number of replays
    struct MultiKey {
        int n, eos;
        bool uni;
        bool operator<(const MultiKey &o) const { return std::tie(n, eos, uni) < std::tie(o.n, o.eos, o.uni); }
    };
    std::map<MultiKey, cudaGraphExec_t> multi_graphs_;
    TypedDeviceBuffer<int32_t> multi_out_, multi_state_;
    TypedDeviceBuffer<uint8_t> multi_uni_;
    int multi_rows_ = 0, multi_eos_ = -1;
    bool multi_has_uni_ = false;
    bool marks_enabled_ = false;
    // fast-path GEMMs with more token rows than this use single-term 16-bit
    // activations (one MMA per K step). Default: fp16 models from the
    // two-SM threshold on (every prefill GEMM of at least pair_min_rows_
    // rows), bf16 models never. Measured on the float32 pack: fp16 single
    // term keeps the logits within 1.65e-2 of the fp32 path at C3 and C4
    // (two terms: 1.23e-2) and makes the C4 prefill 19% faster; bf16 single
    // term moved them by 0.043 on a 1024-token prompt, over the 2e-2 GEMM
    // tolerance. OPWORKS_PREFILL_SINGLE_ROWS sets the threshold (resolved in
    // the constructor).
    int prefill_single_rows_ = [] {
        const char *e = std::getenv("OPWORKS_PREFILL_SINGLE_ROWS");
        return e ? std::atoi(e) : -1;
    }();
    // fast-path GEMMs of at least this many token rows (and not taken by
    // the single-term path) run the two-SM cta_group::2 kernel; 256 rows
    // measured 1.7% more C5 serving throughput than 512 with no change at
    // C3 or C4; OPWORKS_PAIR_GEMM_ROWS overrides the threshold (0: never)
    int pair_min_rows_ = [] {
        const char *e = std::getenv("OPWORKS_PAIR_GEMM_ROWS");
        const int v = e ? std::atoi(e) : 256;
        return v > 0 ? v : (1 << 30);
    }();
    // tensor-core prefill attention on the fast path (OPWORKS_TC_PREFILL=0:
    // the fp32 SIMT kernel instead); tensor maps of the layers' KV pools
    bool tc_prefill_ = [] {
        const char *e = std::getenv("OPWORKS_TC_PREFILL");
        return !(e && e[0] == '0');
    }();
    std::vector<detail::KvPoolMaps> kv_maps_;
    // upper bound on the K splits (one cluster) of the fused GEMMs: the
    // portable 8 measured fastest at C3 (4 and 16 were slower);
    // OPWORKS_CLUSTER_SPLITS overrides it (up to 16, non-portable clusters)
    int split_cap_[4] = {std::getenv("OPWORKS_SPLITS_QKV") ? std::atoi(std::getenv("OPWORKS_SPLITS_QKV")) : 0,
                         std::getenv("OPWORKS_SPLITS_O") ? std::atoi(std::getenv("OPWORKS_SPLITS_O")) : 0,
                         std::getenv("OPWORKS_SPLITS_GU") ? std::atoi(std::getenv("OPWORKS_SPLITS_GU")) : 0,
                         std::getenv("OPWORKS_SPLITS_DOWN") ? std::atoi(std::getenv("OPWORKS_SPLITS_DOWN")) : 0};
    int max_cluster_splits_ = [] {
        const char *e = std::getenv("OPWORKS_CLUSTER_SPLITS");
        const int want = e ? std::atoi(e) : sm100::kMaxClusterSplits;
        return std::max(1, std::min(want, sm100::kMaxClusterSplitsNonPortable));
    }();
    // L2 prefetch of the next projection's weights by each decode GEMM: off
    // by default (measured slower at C3: the prefetch competes with the
    // running GEMM's own weight stream); OPWORKS_L2_PREFETCH=1 turns it on,
    // =2 also lets the QKV GEMM pull the O weights across the attention kernel
    int l2_prefetch_ = [] {
        const char *e = std::getenv("OPWORKS_L2_PREFETCH");
        return e ? std::atoi(e) : 0;
    }();
    bool l2_prefetch_qkv_o_ = l2_prefetch_ >= 2;
    // K splits of the LM head GEMM (a cluster per vocabulary tile when > 1:
    // smaller CTAs, so the last wave of 1002 tiles leaves fewer SMs idle)
    int lm_head_splits_ = [] {
        const char *e = std::getenv("OPWORKS_LMHEAD_SPLITS");
        const int v = e ? std::atoi(e) : 1;
        return v >= 1 && v <= 8 ? v : 1;
    }();
    // where a GEMM issues that prefetch: after its own last load
    // (OPWORKS_L2_PREFETCH_AT=tail) or at its start
    bool l2_prefetch_tail_ = [] {
        const char *e = std::getenv("OPWORKS_L2_PREFETCH_AT");
        return e && std::strcmp(e, "tail") == 0;
    }();
    // programmatic dependent launch between the kernels of a step
    // (OPWORKS_PDL=0 turns it off)
    bool pdl_ = [] {
        const char *e = std::getenv("OPWORKS_PDL");
        return !(e && e[0] == '0');
    }();
    std::vector<std::pair<std::string, cudaEvent_t>> marks_;
};

template <typename WT> class LlamaModelT {
  public:
    using Engine = LlamaEngineT<WT>;

    // Session: KV cache + workspace + stream of one sequence. `cache.length`
    // and `cache.reset()` keep the reference's contract.
    struct Session {
        std::unique_ptr<Engine> engine;
        struct CacheView {
            Engine *e = nullptr;
            int max_seq_len = 0;
            int length_value() const { return e->length(0); }
            void reset() { e->reset(0); }
        } cache;
        cudaStream_t stream() const { return engine->stream(); }
    };

    // sets: which weight precisions to keep on the device (0 = default: all
    // for fp32 packs, the 16-bit set for bf16 packs).
    static LlamaModelT load(const std::string &pack_path, unsigned sets = 0, int max_positions = 8192) {
        PackReader pack(pack_path);
        LlamaModelT m;
        m.cfg_ = ModelConfig::from_manifest(pack.manifest());
        if (sets == 0)
            sets = std::is_same_v<WT, float> ? (kWeights16 | kWeightsF32 | kWeightsSplit) : kWeights16;
        OPWORKS_CUDA_CHECK(cudaGetDevice(&m.device_));
        m.weights_ = std::make_unique<ModelWeights<WT>>(ModelWeights<WT>::load(pack, m.cfg_, sets, max_positions));
        m.default_precision_ = std::is_same_v<WT, float> ? Precision::kAccurate : Precision::kFast;
        if (m.default_precision_ == Precision::kAccurate && !(sets & kWeightsSplit))
            m.default_precision_ = Precision::kFast;
        return m;
    }

    const ModelConfig &config() const { return cfg_; }
    const ModelWeights<WT> &weights() const { return *weights_; }
    int device() const { return device_; }
    Precision default_precision() const { return default_precision_; }

    Session create_session(int max_seq_len) const {
        if (max_seq_len <= 0 || max_seq_len > weights_->rope_max_pos)
            throw std::invalid_argument("max_seq_len must be in (0, 8192]");
        OPWORKS_CUDA_CHECK(cudaSetDevice(device_));
        Session s;
        s.engine = std::make_unique<Engine>(cfg_, *weights_, 1, max_seq_len, default_precision_);
        s.cache.e = s.engine.get();
        s.cache.max_seq_len = max_seq_len;
        return s;
    }

    std::unique_ptr<Engine> create_engine(int max_batch, int max_seq_len, Precision prec, int prefill_rows,
                                          const TensorParallel &tp = {}) const {
        OPWORKS_CUDA_CHECK(cudaSetDevice(device_));
        return std::make_unique<Engine>(cfg_, *weights_, max_batch, max_seq_len, prec, prefill_rows, tp);
    }

    int32_t prefill(Session &s, const std::vector<int32_t> &ids) {
        if (s.engine->length(0) != 0)
            throw std::invalid_argument("prefill requires a fresh session (reset first)");
        for (int32_t id : ids)
            if (id < 0 || id >= cfg_.vocab_size)
                throw std::invalid_argument("token id outside the vocabulary");
        if (ids.empty())
            throw std::invalid_argument("prefill requires at least one token");
        if (static_cast<int>(ids.size()) > s.cache.max_seq_len)
            throw std::invalid_argument("prompt exceeds the session capacity");
        return s.engine->prefill(0, ids.data(), static_cast<int>(ids.size()), SampleArgs{});
    }

    int32_t decode_step(Session &s, int32_t token) {
        if (token < 0 || token >= cfg_.vocab_size)
            throw std::invalid_argument("token id outside the vocabulary");
        if (s.engine->length(0) >= s.cache.max_seq_len)
            throw std::invalid_argument("session capacity exhausted");
        const int32_t slot = 0;
        int32_t out = 0;
        SampleArgs sa;
        s.engine->decode(1, &slot, &token, &sa, &out);
        return out;
    }

    bool is_eos(int32_t token) const {
        return std::find(cfg_.eos_token_ids.begin(), cfg_.eos_token_ids.end(), token) != cfg_.eos_token_ids.end();
    }

    std::vector<float> last_logits(Session &s) const {
        std::vector<float> out(cfg_.vocab_size);
        s.engine->copy_logits(0, out.data(), cfg_.vocab_size);
        return out;
    }

    void copy_last_logits(Session &s, float *out, int n) const {
        if (n != cfg_.vocab_size)
            throw std::invalid_argument("logits buffer must hold vocab_size floats");
        s.engine->copy_logits(0, out, n);
    }

    std::vector<float> hidden_state(Session &s, int rows) const {
        std::vector<float> out(static_cast<size_t>(rows) * cfg_.hidden_size);
        s.engine->copy_hidden(out.data(), rows);
        return out;
    }

    // Prefill that also returns the residual stream after the embedding and
    // after each layer (test/debug hook of the reference).
    std::vector<std::vector<float>> debug_prefill(Session &s, const std::vector<int32_t> &ids) {
        if (s.engine->length(0) != 0)
            throw std::invalid_argument("prefill requires a fresh session (reset first)");
        if (ids.empty())
            throw std::invalid_argument("prefill requires at least one token");
        if (static_cast<int>(ids.size()) > s.cache.max_seq_len)
            throw std::invalid_argument("prompt exceeds the session capacity");
        const int n = static_cast<int>(ids.size());
        std::vector<std::vector<float>> captures;
        s.engine->prefill(0, ids.data(), n, SampleArgs{}, [&](int) {
            std::vector<float> h(static_cast<size_t>(n) * cfg_.hidden_size);
            s.engine->copy_hidden(h.data(), n);
            captures.push_back(std::move(h));
        });
        return captures;
    }

  private:
    ModelConfig cfg_;
    std::unique_ptr<ModelWeights<WT>> weights_;
    int device_ = 0;
    Precision default_precision_ = Precision::kFast;
};

using LlamaModel = LlamaModelT<float>;
using LlamaModelBF16 = LlamaModelT<__nv_bfloat16>;

} // namespace opworks

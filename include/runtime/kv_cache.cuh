#pragma once

// Paged fp32 KV cache.
//
// OpWorks keeps one contiguous [kvh, max_seq_len, D] slab per layer and per
// session (include/runtime/kv_cache.cuh:11-35). Here K and V live in a pool of
// 16-token blocks shared by every sequence of an engine:
//   pool = [layers][K|V][num_blocks][kvh][16][D]  (fp32)
// and each sequence maps logical block i (tokens 16i..16i+15) to a physical
// block through a block table. A (sequence, kv head) block is 4 KB of
// contiguous floats, the unit the attention kernels stage with one bulk
// copy. `length` / `max_seq_len` / reset() keep the session-level contract of
// the original (reset only forgets the length; stale bytes are never read).

#include <stdexcept>
#include <vector>

#include "../core/typed_device_buffer.cuh"
#include "model_config.cuh"

namespace opworks {

constexpr int kKvBlockTokens = 16;

struct KvCache {
    int max_seq_len = 0;
    int length = 0; // valid entries of a single-sequence session
    int num_layers = 0, kv_heads = 0, head_dim = 0, num_blocks = 0;
    TypedDeviceBuffer<float> pool;

    KvCache() = default;
    KvCache(const ModelConfig &cfg, int max_seq_len_, int num_blocks_)
        : max_seq_len(max_seq_len_), num_layers(cfg.num_layers), kv_heads(cfg.num_kv_heads),
          head_dim(cfg.head_dim), num_blocks(num_blocks_) {
        pool = TypedDeviceBuffer<float>(static_cast<int64_t>(num_layers) * 2 * num_blocks * block_floats());
        // tensor-core prefill stages whole 16-token pages, including slots
        // past a sequence's end (masked, weight 0): they must hold finite values
        if (pool.size() > 0)
            OPWORKS_CUDA_CHECK(cudaMemset(pool.data(), 0, sizeof(float) * static_cast<size_t>(pool.size())));
    }
    KvCache(const KvCache &) = delete;
    KvCache &operator=(const KvCache &) = delete;
    KvCache(KvCache &&) = default;
    KvCache &operator=(KvCache &&) = default;

    int64_t block_floats() const { return static_cast<int64_t>(kv_heads) * kKvBlockTokens * head_dim; }
    float *k(int layer) { return pool.data() + (static_cast<int64_t>(layer) * 2) * num_blocks * block_floats(); }
    float *v(int layer) { return pool.data() + (static_cast<int64_t>(layer) * 2 + 1) * num_blocks * block_floats(); }
    void reset() { length = 0; }
};

// Free list of physical blocks.
class BlockAllocator {
  public:
    explicit BlockAllocator(int n = 0) {
        free_.reserve(n);
        for (int i = n - 1; i >= 0; --i)
            free_.push_back(i);
    }
    int alloc() {
        if (free_.empty())
            throw std::runtime_error("KV cache block pool exhausted");
        const int b = free_.back();
        free_.pop_back();
        return b;
    }
    void release(int b) { free_.push_back(b); }
    int available() const { return static_cast<int>(free_.size()); }

  private:
    std::vector<int> free_;
};

} // namespace opworks

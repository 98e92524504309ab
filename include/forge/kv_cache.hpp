// forge/kv_cache.hpp — the 3-tier int8 KV cache of the reference
// (include/forge/kv_cache.hpp:23-110 there) with its storage on the GPU.
//
// Per (layer, kv head): sink slots for positions < sink_size, a circular
// window of min(window_size, max_context) entries, and a pool of
// pool_block-entry means of evicted window entries (accumulated in double).
// store / attention_scores / attention_weighted_sum take HOST vectors and run
// one device kernel each (libpf_b200: pf_kvu_*), synchronously.  Scores and
// weighted sums keep the reference's summation order.
#ifndef FORGE_B200_KV_CACHE_HPP
#define FORGE_B200_KV_CACHE_HPP

#include <cstddef>
#include <cstdint>
#include <memory>
#include <vector>

#include "types.hpp"

namespace forge {

struct KVCacheConfig {
    uint32_t n_layers = 24;
    uint32_t n_kv_heads = 4;
    uint32_t head_dim = 64;
    uint32_t sink_size = 4;
    uint32_t window_size = 8192;
    uint32_t pool_block = 64;
    uint32_t max_context = 131072;
};

class FORGE_API KVCache {
public:
    explicit KVCache(const KVCacheConfig& cfg);
    ~KVCache();
    KVCache(const KVCache&) = delete;
    KVCache& operator=(const KVCache&) = delete;

    // Quantize and store the key / value of position `pos` (positions beyond
    // max_context, and layers / heads out of range, are ignored).
    void store(uint32_t layer, uint32_t head, uint32_t pos, const float* key, const float* value);
    // Scores q . (k * scale) of every stored entry, in the order sink, pool,
    // window oldest first; returns their number.
    uint32_t attention_scores(uint32_t layer, uint32_t head, const float* query, float* scores_out);
    // output = sum_e scores[e] * (v_e * scale_e) over the first `count` entries.
    void attention_weighted_sum(uint32_t layer, uint32_t head, const float* scores, float* output, uint32_t count);
    uint32_t size() const { return total_stored_; }
    void clear();
    // Device bytes held by the cache.
    size_t memory_usage() const;

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
    uint32_t total_stored_ = 0;
};

}  // namespace forge

#endif  // FORGE_B200_KV_CACHE_HPP

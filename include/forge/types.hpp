// forge/types.hpp — configuration and result types of the forge:: API
// (the reference's include/forge/types.hpp:32-268, kept field for field so
// code written against the reference compiles against this library).
#ifndef FORGE_B200_TYPES_HPP
#define FORGE_B200_TYPES_HPP

#include <cstddef>
#include <cstdint>
#include <functional>
#include <string>
#include <vector>

#if defined(__GNUC__)
#define FORGE_API __attribute__((visibility("default")))
#else
#define FORGE_API
#endif

namespace forge {

// Packed block layouts of the .squeeze format (types.hpp:14-31 of the reference).
struct Q8_0 {
    float d;
    int8_t q[32];
};
struct Q4_0 {
    float d;
    uint8_t q[16];
};
struct Q2_0 {
    float d;
    uint8_t q[8];
};
struct Q1_5 {
    uint8_t q[16];
};

struct SamplingConfig {
    float temperature = 0.8f;
    float top_p = 0.95f;
    uint32_t top_k = 40;
    bool greedy = false;
};

struct GenerationConfig {
    SamplingConfig sampling;
    uint32_t max_new_tokens = 256;
    uint32_t max_context = 131072;
    bool mtp_enabled = true;
    bool stream = false;
    float skip_threshold = 0.01f;
};

struct WeightBlock {
    uint32_t layer_id;
    uint32_t matrix_id;
    uint32_t n_rows;
    uint32_t n_cols;
    uint32_t compressed_size;
    uint32_t original_size;
    uint8_t quant_type;
    uint32_t offset;
};

struct FORGE_API ModelConfig {
    uint32_t n_layers = 24;
    uint32_t n_embd = 1536;
    uint32_t n_heads = 16;
    uint32_t n_kv_heads = 2;
    uint32_t n_ff = 4608;
    uint32_t n_vocab = 130560;
    uint32_t head_dim_ = 0;  // 0: n_embd / n_heads
    uint32_t max_seq_len = 131072;
    bool mtp_enabled = true;
    uint32_t mtp_heads = 4;
    float skip_threshold = 0.01f;
    uint32_t skip_interval = 4;
    uint32_t kv_cache_size = 8192;  // window
    size_t max_memory = 250 * 1024 * 1024;
    bool use_bpe = false;
    uint32_t head_dim() const { return head_dim_ ? head_dim_ : (n_embd / n_heads); }
    uint32_t kv_head_dim() const { return (head_dim_ && n_kv_heads) ? head_dim_ : (n_embd / n_kv_heads); }
    // Whether the model's weights (int8, 1 byte each) fit max_memory.
    bool check_memory_budget() const;
};

struct GenerationResult {
    std::vector<int32_t> tokens;
    float tokens_per_second = 0.0f;
    size_t peak_memory_bytes = 0;
    int mtp_accepted = 0;
    int layers_skipped = 0;
    bool oom_protected = false;
    int mtp_rejected = 0;
};

using TokenCallback = std::function<void(int32_t token, float prob)>;
using ProgressCallback = std::function<void(float progress)>;

}  // namespace forge

#endif  // FORGE_B200_TYPES_HPP

// forge/layer_skip.hpp — predictive FFN layer skipping of the reference
// (include/forge/layer_skip.hpp:30-89 there); the cached vectors live on the
// GPU and the distance is computed there in the reference's order.
#ifndef FORGE_B200_LAYER_SKIP_HPP
#define FORGE_B200_LAYER_SKIP_HPP

#include <cstdint>
#include <memory>
#include <vector>

#include "types.hpp"

namespace forge {

class FORGE_API LayerSkipController {
public:
    LayerSkipController(const ModelConfig& cfg);
    ~LayerSkipController();
    LayerSkipController(const LayerSkipController&) = delete;
    LayerSkipController& operator=(const LayerSkipController&) = delete;

    // true: skip layer_id's FFN, since the post-attention vector moved less
    // than the (layer-adjusted) threshold from the one of the last computed
    // FFN.  Layers 0, 1 and the last two never skip; anchor tokens never skip.
    bool should_skip_ffn(uint32_t layer_id, const float* hidden_after_attn, uint32_t n_embd);
    void record_layer_output(uint32_t layer_id, const float* hidden_after_ffn, uint32_t n_embd);
    void new_token();
    uint32_t total_skipped() const { return skipped_count_; }
    const std::vector<bool>& skip_mask() const { return skip_mask_; }
    void reset();
    void reset_anchor();
    void set_threshold(float t) { threshold_ = t; }
    float threshold() const { return threshold_; }
    bool is_anchor_token() const { return tokens_since_anchor_ >= interval_; }

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
    ModelConfig cfg_;
    float threshold_;
    uint32_t interval_;
    std::vector<bool> skip_mask_;
    uint32_t skipped_count_ = 0;
    uint32_t tokens_since_anchor_ = 0;
};

}  // namespace forge

#endif  // FORGE_B200_LAYER_SKIP_HPP

// layer_skip.cpp — forge::LayerSkipController with its cached vectors on the
// GPU (decision rules of the reference's src/layer_skip.cpp:8-113).
#include "forge/layer_skip.hpp"

#include <algorithm>

#include "device.hpp"

namespace forge {

struct LayerSkipController::Impl {
    dev::Buffer attn;    // [n_layers][n_embd] post-attention vectors of the last computed FFN
    dev::Buffer hidden;  // [n_layers][n_embd] post-FFN vectors
    dev::Buffer x;       // staging of the caller's vector
    dev::Buffer delta;
    uint32_t n = 0, L = 0;
};

LayerSkipController::LayerSkipController(const ModelConfig& cfg)
    : impl_(new Impl), cfg_(cfg), threshold_(cfg.skip_threshold), interval_(cfg.skip_interval) {
    impl_->L = cfg.n_layers;
    impl_->n = cfg.n_embd;
    skip_mask_.assign(cfg.n_layers, false);
    const size_t bytes = (size_t)cfg.n_layers * cfg.n_embd * sizeof(float);
    if (impl_->attn.reserve(bytes + 16) && impl_->hidden.reserve(bytes + 16)) {
        cudaMemset(impl_->attn.as<void>(), 0, bytes);
        cudaMemset(impl_->hidden.as<void>(), 0, bytes);
    }
    impl_->x.reserve((size_t)cfg.n_embd * sizeof(float) + 16);
    impl_->delta.reserve(16);
}

LayerSkipController::~LayerSkipController() = default;

bool LayerSkipController::should_skip_ffn(uint32_t layer_id, const float* hidden_after_attn, uint32_t n_embd) {
    if (layer_id >= cfg_.n_layers) return false;
    const uint32_t n = std::min(n_embd, impl_->n);
    float* cache = impl_->attn.as<float>() + (size_t)layer_id * impl_->n;
    float* x = impl_->x.as<float>();
    if (!cache || !x || !dev::to_dev(x, hidden_after_attn, (size_t)n * 4, "should_skip_ffn")) return false;
    if (is_anchor_token()) {  // anchors compute every layer and refresh the cache
        skip_mask_[layer_id] = false;
        dev::cuda_ok(cudaMemcpy(cache, x, (size_t)n * 4, cudaMemcpyDeviceToDevice), "should_skip_ffn");
        return false;
    }
    float delta = 0.0f;
    if (!dev::ok(pf_skip_delta(x, cache, n, impl_->delta.as<float>(), nullptr), "should_skip_ffn") ||
        !dev::to_host(&delta, impl_->delta.as<void>(), 4, "should_skip_ffn"))
        return false;
    const uint32_t mid = cfg_.n_layers / 2;
    float t = threshold_;
    if (layer_id > mid / 2 && layer_id < mid + mid / 2) t *= 2.0f;  // middle layers skip more
    if (layer_id < 2 || layer_id >= cfg_.n_layers - 2) t = -1.0f;   // never the outer two
    const bool skip = delta < t;
    skip_mask_[layer_id] = skip;
    if (!skip) dev::cuda_ok(cudaMemcpy(cache, x, (size_t)n * 4, cudaMemcpyDeviceToDevice), "should_skip_ffn");
    return skip;
}

void LayerSkipController::record_layer_output(uint32_t layer_id, const float* hidden_after_ffn, uint32_t n_embd) {
    if (layer_id >= cfg_.n_layers || skip_mask_[layer_id]) return;
    const uint32_t n = std::min(n_embd, impl_->n);
    float* dst = impl_->hidden.as<float>() + (size_t)layer_id * impl_->n;
    if (dst) dev::to_dev(dst, hidden_after_ffn, (size_t)n * 4, "record_layer_output");
}

void LayerSkipController::new_token() {
    tokens_since_anchor_ = (tokens_since_anchor_ + 1) % (interval_ + 1);
    std::fill(skip_mask_.begin(), skip_mask_.end(), false);
}

void LayerSkipController::reset() {
    skipped_count_ = 0;
    tokens_since_anchor_ = 0;
    std::fill(skip_mask_.begin(), skip_mask_.end(), false);
    const size_t bytes = (size_t)impl_->L * impl_->n * sizeof(float);
    if (impl_->attn.as<void>()) cudaMemset(impl_->attn.as<void>(), 0, bytes);
    if (impl_->hidden.as<void>()) cudaMemset(impl_->hidden.as<void>(), 0, bytes);
}

void LayerSkipController::reset_anchor() { tokens_since_anchor_ = 0; }

bool ModelConfig::check_memory_budget() const {
    // The reference's estimate (src/engine.cpp:18-27): int8 KV of the window
    // (capped at 8192) and the 64-entry pool over max_seq_len, the MTP heads
    // at 1.5 bytes per d*d weight, and activation buffers.
    const size_t hd = head_dim();
    const size_t window = kv_cache_size < 8192u ? kv_cache_size : 8192u;
    const size_t pool = max_seq_len > window ? (max_seq_len - window) / 64 : 0;
    const size_t kv = (size_t)n_layers * n_kv_heads * (window + pool) * hd * 2;
    const size_t mtp = (size_t)mtp_heads * n_embd * n_embd * 3 / 2;
    const size_t act = (size_t)n_embd * 20 * 4;
    return kv + mtp + act < max_memory;
}

}  // namespace forge

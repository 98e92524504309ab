// forge/engine.hpp — the reference's single-sequence Engine API
// (include/forge/engine.hpp:15-141 there) on the GPU batch engine with one
// sequence.
//
// load_model reads a .squeeze file (projections, tied embedding, norms); MTP
// heads come from the seeded generator.  generate / forward run the
// speculative-decode step of forge::BatchEngine: verification of the K MTP
// drafts in one batched forward, commit of the accepted prefix only, and
// positions equal to token positions.  The device engine supports head_dim 64.
//
// Reference-compat mode (set_reference_compat(true) before load_model, or
// FORGE_REFERENCE_COMPAT=1 in the environment when the Engine is constructed)
// reproduces the reference's literal Engine instead (src/engine.cpp:47-396,
// 459-854): placeholder projections (the file's layer matrices are never
// loaded), the layer index as RoPE and KV position with theta 5e6, each K head
// rotated once per query head, head outputs as the reference leaves them,
// sequential verification of sampled drafts with no KV rollback, the process-wide
// sampler, MTP weights drawn from rand() (twice, as the reference's load does)
// and its memory statistics.  Its forward runs on the device with the
// reference's float operation order; it needs n_vocab <= 16384 and n_embd <= 4096.
#ifndef FORGE_B200_ENGINE_HPP
#define FORGE_B200_ENGINE_HPP

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "batch_engine.hpp"
#include "kv_cache.hpp"
#include "layer_skip.hpp"
#include "mtp.hpp"
#include "types.hpp"

namespace forge {

class FORGE_API Engine {
public:
    Engine();
    ~Engine();
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    bool load_model(const std::string& squeeze_path);

    // Reference-compat mode (see above); takes effect at the next load_model.
    void set_reference_compat(bool on);
    bool reference_compat() const { return compat_; }

    void set_max_context(uint32_t tokens);
    void set_mtp_enabled(bool enabled);
    void set_layer_skip_threshold(float threshold);
    void set_max_memory(size_t bytes);

    // prompt_tokens + up to max_new_tokens generated tokens in result.tokens;
    // callback(token, 1.0f) once per generated token, progress(fraction).
    GenerationResult generate(const std::vector<int32_t>& prompt_tokens, uint32_t max_new_tokens,
                              TokenCallback callback = nullptr, ProgressCallback progress = nullptr);
    // Logits after the tokens (a fresh sequence): n_vocab values.
    std::vector<float> forward(const std::vector<int32_t>& tokens);
    std::vector<float> forward_with_hidden(const std::vector<int32_t>& tokens, std::vector<float>& hidden_out);

    // Sampling of a host logits vector on the device (src/engine.cpp:881-1003):
    // greedy when cfg.greedy or temperature <= 0, else top-p when 0 < p < 1
    // (top-k then ignored), else top-k when 0 < k < n, else temperature.
    // One uniform per stochastic draw from a std::mt19937 seeded 42.
    int32_t sample(const float* logits, uint32_t n_vocab, const SamplingConfig& cfg = SamplingConfig());
    int32_t sample_greedy(const float* logits, uint32_t n_vocab);
    int32_t sample_top_k(const float* logits, uint32_t n_vocab, uint32_t k, float temp);
    int32_t sample_top_p(const float* logits, uint32_t n_vocab, float p, float temp);

    struct MemoryStats {
        size_t weights_mmap = 0;
        size_t weights_decompressed = 0;
        size_t kv_cache = 0;
        size_t activations = 0;
        size_t prefetch_buffer = 0;
        size_t mtp_heads = 0;
        size_t other = 0;
        size_t total() const;
    };
    MemoryStats get_memory_stats() const;

    const ModelConfig& config() const { return config_; }
    const std::string& last_error() const { return err_; }

private:
    struct Literal;  // the reference-compat engine (forge/literal.hpp)
    bool ensure_engine();
    bool compat_load(const std::string& path);
    GenerationResult compat_generate(const std::vector<int32_t>& prompt, uint32_t max_new, TokenCallback cb,
                                     ProgressCallback progress);
    std::vector<float> compat_forward(const std::vector<int32_t>& tokens, std::vector<float>& hidden_out);
    MemoryStats compat_memory_stats() const;
    void compat_set_max_context(uint32_t tokens);
    ModelConfig config_;
    std::string path_;
    uint32_t max_context_ = 8192;
    bool mtp_enabled_ = true;
    float skip_threshold_ = 0.01f;
    size_t max_memory_ = 250 * 1024 * 1024;
    int qtype_[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // device formats of the 7 projections and the embedding
    std::unique_ptr<BatchEngine> engine_;
    std::string err_;
    struct Sampler;
    std::unique_ptr<Sampler> sampler_;
    bool compat_ = false;
    std::unique_ptr<Literal> lit_;
};

}  // namespace forge

#endif  // FORGE_B200_ENGINE_HPP

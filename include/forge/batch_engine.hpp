// forge/batch_engine.hpp — the multi-sequence MTP speculative-decode engine on
// one GPU (new in this library; the reference has no batch API).
//
// Each step verifies, for every sequence, the pending token and K draft tokens
// from the MTP heads in one batched forward through the quantized
// transformer, accepts the longest draft prefix that matches the sampled /
// greedy verification, emits the token after it, and commits the KV entries
// of the accepted rows only.  One engine owns one GPU; for several GPUs run
// one engine per GPU on disjoint sequences (there is no exchange inside a
// step).  Errors: every call returns false and last_error() says why.
#ifndef FORGE_B200_BATCH_ENGINE_HPP
#define FORGE_B200_BATCH_ENGINE_HPP

#include <cstdint>
#include <string>
#include <vector>

#include "types.hpp"

struct pf_engine;

namespace forge {

// The step's model: ModelConfig plus what the device engine needs.
struct BatchConfig {
    ModelConfig model;            // n_layers .. n_vocab, mtp_heads, kv_cache_size (window), skip_threshold
    uint32_t sink_size = 4;
    uint32_t pool_block = 64;
    uint32_t max_context = 8192;  // window = min(kv_cache_size, max_context)
    float rope_theta = 10000.0f;
    float norm_eps = 1e-6f;
    bool skip_enabled = false;
    // Per-matrix quantization type of the device weights (Q, K, V, O, gate,
    // up, down): 0 int8, 1 Q4, 2 Q2, 3 Q1.5; and of the tied embedding.
    int qtype[7] = {1, 1, 1, 1, 1, 1, 1};
    int emb_qtype = 1;
};

class FORGE_API BatchEngine {
public:
    BatchEngine(const BatchConfig& cfg, uint32_t max_sequences, uint32_t max_positions, int device = 0);
    ~BatchEngine();
    BatchEngine(const BatchEngine&) = delete;
    BatchEngine& operator=(const BatchEngine&) = delete;

    bool ok() const { return e_ != nullptr; }
    const std::string& last_error() const { return err_; }
    const BatchConfig& config() const { return cfg_; }

    // Weights: the seeded synthetic model (N(0, 0.02) through the reference's
    // Quantizer), or the projection / embedding blocks of a .squeeze file.
    // MTP heads are not stored in .squeeze files; they come from the seeded
    // generator of the reference's MTPHeads::init_weights distribution.
    bool load_synthetic(uint32_t seed = 0, uint32_t mtp_seed = 3, int threads = 8);
    bool load_squeeze(const std::string& path, uint32_t mtp_seed = 3);

    bool set_sampling(const SamplingConfig& s);
    bool set_skip_threshold(float t);

    // Resets every sequence and prefills one prompt per sequence (seeds: one
    // per sequence for stochastic sampling, or empty).
    bool prefill(const std::vector<std::vector<int32_t>>& prompts, const std::vector<uint32_t>& seeds = {});
    // One speculative-decode step; emitted[i] receives sequence i's tokens.
    bool step(std::vector<std::vector<int32_t>>* emitted);
    // prefill + steps until every sequence has max_new_tokens; the first
    // token of each sequence comes out of the prefill.
    bool generate(const std::vector<std::vector<int32_t>>& prompts, uint32_t max_new_tokens,
                  std::vector<std::vector<int32_t>>* out, const std::vector<uint32_t>& seeds = {});

    // Logits of the last verify (after prefill: of each prompt's last token),
    // [sequences * (K + 1)][n_vocab].
    bool logits(std::vector<float>* out) const;
    bool positions(std::vector<int32_t>* out) const;  // committed length of each sequence
    bool pending(std::vector<int32_t>* out) const;    // each sequence's next token (not yet forwarded)
    // Verify rows computed / FFNs skipped since prefill (layer skip).
    bool skip_counts(int64_t* computed, int64_t* skipped) const;
    uint32_t sequences() const { return n_seqs_; }
    uint32_t draft_heads() const { return cfg_.model.mtp_heads; }
    // Device bytes the engine allocated.
    size_t device_bytes() const { return dev_bytes_; }

private:
    bool check(int status, const char* what) const;
    BatchConfig cfg_;
    pf_engine* e_ = nullptr;
    uint32_t max_seqs_ = 0, n_seqs_ = 0;
    size_t dev_bytes_ = 0;
    mutable std::string err_;
};

}  // namespace forge

#endif  // FORGE_B200_BATCH_ENGINE_HPP

// engine.cpp — forge::Engine (the reference's single-sequence API) on a
// one-sequence forge::BatchEngine.
#include "forge/engine.hpp"

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>

#include "device.hpp"
#include "literal.hpp"
#include "squeeze.hpp"

namespace forge {

// One generator for every Engine of the process, as the reference's
// file-static std::mt19937 rng_engine(42) (src/engine.cpp:16).
std::mt19937& reference_rng() {
    static std::mt19937 rng(42);
    return rng;
}

struct Engine::Sampler {
    dev::Buffer logits, u, out;
};

size_t Engine::MemoryStats::total() const {
    return weights_mmap + weights_decompressed + kv_cache + activations + prefetch_buffer + mtp_heads + other;
}

Engine::Engine() : sampler_(new Sampler) {
    const char* env = std::getenv("FORGE_REFERENCE_COMPAT");
    compat_ = env && *env && std::strcmp(env, "0") != 0;
}
Engine::~Engine() = default;

void Engine::set_reference_compat(bool on) {
    if (on != compat_) {
        engine_.reset();
        lit_.reset();
        path_.clear();
    }
    compat_ = on;
}

bool Engine::load_model(const std::string& path) {
    if (compat_) return compat_load(path);
    squeeze::File f;
    if (!f.open(path, &err_)) {
        std::fprintf(stderr, "forge::Engine::load_model: %s\n", err_.c_str());
        return false;
    }
    config_ = f.config();
    config_.kv_cache_size = std::min(config_.kv_cache_size, 8192u);
    path_ = path;
    // Device weight formats follow the blocks' types (their int8 values fit).
    for (int j = 0; j < 7; j++) {
        const squeeze::Block* b = f.find(0, (uint32_t)j);
        qtype_[j] = b && b->qtype <= 3 ? (int)b->qtype : 0;
    }
    const squeeze::Block* eb = f.find(0, 10);
    qtype_[7] = eb && eb->qtype <= 3 ? (int)eb->qtype : 0;
    engine_.reset();
    if (!ensure_engine()) {
        std::fprintf(stderr, "forge::Engine::load_model: %s\n", err_.c_str());
        return false;
    }
    return true;
}

bool Engine::ensure_engine() {
    if (engine_) return true;
    if (path_.empty()) {
        err_ = "no model loaded";
        return false;
    }
    BatchConfig bc;
    bc.model = config_;
    bc.model.skip_threshold = skip_threshold_;
    bc.max_context = std::min<uint32_t>(max_context_, config_.max_seq_len ? config_.max_seq_len : max_context_);
    bc.model.kv_cache_size = std::min(config_.kv_cache_size, bc.max_context);
    for (int i = 0; i < 7; i++) bc.qtype[i] = qtype_[i];
    bc.emb_qtype = qtype_[7];
    engine_.reset(new BatchEngine(bc, 1, bc.max_context, 0));
    if (!engine_->ok() || !engine_->load_squeeze(path_)) {
        err_ = engine_->last_error();
        engine_.reset();
        return false;
    }
    return true;
}

void Engine::set_max_context(uint32_t tokens) {
    if (compat_) return compat_set_max_context(tokens);
    if (tokens != max_context_) engine_.reset();
    max_context_ = tokens;
}
void Engine::set_mtp_enabled(bool enabled) {
    mtp_enabled_ = enabled;
    config_.mtp_enabled = enabled;
}
void Engine::set_layer_skip_threshold(float threshold) {
    skip_threshold_ = threshold;
    config_.skip_threshold = threshold;
    if (engine_) engine_->set_skip_threshold(threshold);
}
void Engine::set_max_memory(size_t bytes) {
    max_memory_ = bytes;
    config_.max_memory = bytes;
}

GenerationResult Engine::generate(const std::vector<int32_t>& prompt, uint32_t max_new_tokens, TokenCallback callback,
                                  ProgressCallback progress) {
    if (compat_) return compat_generate(prompt, max_new_tokens, callback, progress);
    GenerationResult r;
    r.tokens = prompt;
    if (prompt.empty() || max_new_tokens == 0 || !ensure_engine()) return r;
    const auto t0 = std::chrono::steady_clock::now();
    if (!engine_->prefill({prompt})) {
        err_ = engine_->last_error();
        std::fprintf(stderr, "forge::Engine::generate: %s\n", err_.c_str());
        return r;
    }
    std::vector<int32_t> gen;
    const uint32_t K = engine_->draft_heads();
    std::vector<std::vector<int32_t>> em;
    // The first token comes out of the prefill (the last prompt token's logits).
    std::vector<int32_t> first;
    if (!engine_->pending(&first)) {
        err_ = engine_->last_error();
        return r;
    }
    gen.push_back(first[0]);
    if (callback) callback(first[0], 1.0f);
    while (gen.size() < max_new_tokens) {
        if (!engine_->step(&em)) {
            err_ = engine_->last_error();
            std::fprintf(stderr, "forge::Engine::generate: %s\n", err_.c_str());
            break;
        }
        const int n = (int)em[0].size();
        r.mtp_accepted += n - 1;
        r.mtp_rejected += (int)K - (n - 1);
        for (int32_t t : em[0]) {
            if (gen.size() >= max_new_tokens) break;
            gen.push_back(t);
            if (callback) callback(t, 1.0f);
        }
        if (progress) progress((float)gen.size() / (float)max_new_tokens);
    }
    const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    r.tokens.insert(r.tokens.end(), gen.begin(), gen.end());
    r.tokens_per_second = el > 0 ? (float)(gen.size() / el) : 0.0f;
    r.peak_memory_bytes = engine_->device_bytes();
    int64_t computed = 0, skipped = 0;
    if (engine_->skip_counts(&computed, &skipped)) r.layers_skipped = (int)skipped;
    return r;
}

std::vector<float> Engine::forward(const std::vector<int32_t>& tokens) {
    std::vector<float> hidden;
    return forward_with_hidden(tokens, hidden);
}

std::vector<float> Engine::forward_with_hidden(const std::vector<int32_t>& tokens, std::vector<float>& hidden_out) {
    if (compat_) return compat_forward(tokens, hidden_out);
    std::vector<float> out;
    if (tokens.empty() || !ensure_engine() || !engine_->prefill({tokens})) return out;
    std::vector<float> lg;
    if (!engine_->logits(&lg)) return out;
    out.assign(lg.begin(), lg.begin() + config_.n_vocab);
    (void)hidden_out;  // the hidden is not copied back (the reference copies only into a non-empty vector)
    return out;
}

int32_t Engine::sample(const float* logits, uint32_t n, const SamplingConfig& cfg) {
    Sampler& s = *sampler_;
    const bool greedy = cfg.greedy || cfg.temperature <= 0.0f;
    float* dl = static_cast<float*>(s.logits.reserve((size_t)n * 4 + 16));
    float* du = static_cast<float*>(s.u.reserve(16));
    int32_t* dout = static_cast<int32_t*>(s.out.reserve(16));
    int32_t tok = 0;
    if (!dl || !du || !dout || !dev::to_dev(dl, logits, (size_t)n * 4, "Engine::sample")) return tok;
    if (greedy) {
        if (dev::ok(pf_argmax_rows(dl, 1, (int32_t)n, dout, nullptr), "Engine::sample")) dev::to_host(&tok, dout, 4, "Engine::sample");
        return tok;
    }
    const float u = std::uniform_real_distribution<float>(0.0f, 1.0f)(reference_rng());
    pf_sampling_config c{cfg.temperature, cfg.top_p, cfg.top_k, 0};
    if (!dev::to_dev(du, &u, 4, "Engine::sample")) return tok;
    if (dev::ok(pf_sample_rows(dl, 1, (int32_t)n, &c, du, dout, nullptr), "Engine::sample"))
        dev::to_host(&tok, dout, 4, "Engine::sample");
    return tok;
}

int32_t Engine::sample_greedy(const float* logits, uint32_t n) {
    SamplingConfig c;
    c.greedy = true;
    return sample(logits, n, c);
}

int32_t Engine::sample_top_k(const float* logits, uint32_t n, uint32_t k, float temp) {
    SamplingConfig c;
    c.temperature = temp;
    c.top_p = 1.0f;  // not a nucleus draw
    c.top_k = k;
    return sample(logits, n, c);
}

int32_t Engine::sample_top_p(const float* logits, uint32_t n, float p, float temp) {
    SamplingConfig c;
    c.temperature = temp;
    c.top_p = p;
    c.top_k = 0;
    return sample(logits, n, c);
}

Engine::MemoryStats Engine::get_memory_stats() const {
    if (compat_) return compat_memory_stats();
    MemoryStats m;
    if (!engine_) return m;
    const ModelConfig& c = config_;
    const size_t hd = c.head_dim(), d = c.n_embd;
    const size_t per_layer = d * c.n_heads * hd + 2 * d * c.n_kv_heads * hd + c.n_heads * hd * d + 3 * d * (size_t)c.n_ff;
    m.weights_decompressed = per_layer * c.n_layers + (size_t)c.n_vocab * d * 2;
    m.mtp_heads = (size_t)c.mtp_heads * 3 * d * (d / 2 + 4);
    const size_t window = std::min<size_t>(c.kv_cache_size, max_context_);
    const size_t pool = max_context_ > window ? (max_context_ - window) / 64 + 1 : 0;
    m.kv_cache = (size_t)c.n_layers * c.n_kv_heads * (4 + window + pool) * (2 * hd + 8);
    const size_t all = engine_->device_bytes();
    const size_t used = m.weights_decompressed + m.mtp_heads + m.kv_cache;
    m.activations = all > used ? all - used : 0;
    return m;
}

}  // namespace forge

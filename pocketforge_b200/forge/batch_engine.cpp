// batch_engine.cpp — forge::BatchEngine over the C ABI of libpf_b200.
#include "forge/batch_engine.hpp"

#include <algorithm>
#include <cstring>

#include "device.hpp"
#include "squeeze.hpp"

namespace forge {

namespace {

pf_model_config to_c(const BatchConfig& b) {
    pf_model_config c{};
    const ModelConfig& m = b.model;
    c.n_layers = (int32_t)m.n_layers;
    c.n_embd = (int32_t)m.n_embd;
    c.n_heads = (int32_t)m.n_heads;
    c.n_kv_heads = (int32_t)m.n_kv_heads;
    c.head_dim = (int32_t)m.head_dim();
    c.n_ff = (int32_t)m.n_ff;
    c.n_vocab = (int32_t)m.n_vocab;
    c.n_mtp_heads = (int32_t)m.mtp_heads;
    c.sink_size = (int32_t)b.sink_size;
    c.window_size = (int32_t)m.kv_cache_size;
    c.pool_block = (int32_t)b.pool_block;
    c.max_context = (int32_t)b.max_context;
    c.rope_theta = b.rope_theta;
    c.norm_eps = b.norm_eps;
    c.skip_enabled = b.skip_enabled ? 1 : 0;
    c.skip_threshold = m.skip_threshold;
    for (int i = 0; i < 7; i++) c.qtype[i] = b.qtype[i];
    c.emb_qtype = b.emb_qtype;
    return c;
}

}  // namespace

bool BatchEngine::check(int status, const char* what) const {
    if (status == PF_OK) return true;
    err_ = std::string(what) + ": " + pf_last_error();
    return false;
}

BatchEngine::BatchEngine(const BatchConfig& cfg, uint32_t max_sequences, uint32_t max_positions, int device)
    : cfg_(cfg), max_seqs_(max_sequences) {
    const pf_model_config c = to_c(cfg);
    size_t free0 = 0, free1 = 0, total = 0;
    cudaSetDevice(device);
    cudaMemGetInfo(&free0, &total);
    pf_engine* e = nullptr;
    if (check(pf_engine_create(&c, (int32_t)max_sequences, (int32_t)max_positions, device, &e), "pf_engine_create"))
        e_ = e;
    cudaMemGetInfo(&free1, &total);
    dev_bytes_ = free0 > free1 ? free0 - free1 : 0;
}

BatchEngine::~BatchEngine() {
    if (e_) pf_engine_destroy(e_);
}

bool BatchEngine::load_synthetic(uint32_t seed, uint32_t mtp_seed, int threads) {
    if (!e_) return false;
    const pf_model_config c = to_c(cfg_);
    return check(pf_engine_load_synthetic(e_, &c, seed, mtp_seed, threads), "pf_engine_load_synthetic");
}

bool BatchEngine::load_squeeze(const std::string& path, uint32_t mtp_seed) {
    if (!e_) return false;
    squeeze::File f;
    if (!f.open(path, &err_)) return false;
    const ModelConfig& fc = f.config();
    const ModelConfig& m = cfg_.model;
    if (fc.n_layers != m.n_layers || fc.n_embd != m.n_embd || fc.n_heads != m.n_heads ||
        fc.n_kv_heads != m.n_kv_heads || fc.n_ff != m.n_ff || fc.n_vocab != m.n_vocab) {
        err_ = path + ": model shape differs from the engine's configuration";
        return false;
    }
    const uint32_t d = m.n_embd, hd = m.head_dim(), q = m.n_heads * hd, kv = m.n_kv_heads * hd, ff = m.n_ff;
    // Shapes of the 7 projections as the engine uses them (rows = outputs).
    const uint32_t rows[7] = {q, kv, kv, d, ff, ff, d};
    const uint32_t cols[7] = {d, d, d, q, d, d, ff};
    squeeze::Matrix mx;
    for (uint32_t l = 0; l < m.n_layers; l++)
        for (uint32_t j = 0; j < 7; j++) {
            if (!f.load(l, j, &mx, &err_)) return false;
            if (mx.rows != rows[j] || mx.cols != cols[j]) {
                err_ = path + ": block (" + std::to_string(l) + ", " + std::to_string(j) + ") is " +
                       std::to_string(mx.rows) + " x " + std::to_string(mx.cols) + ", the engine needs " +
                       std::to_string(rows[j]) + " x " + std::to_string(cols[j]);
                return false;
            }
            if (!check(pf_engine_set_matrix(e_, (int32_t)l, (int32_t)j, mx.data.data(), mx.row_scales.data()),
                       "pf_engine_set_matrix"))
                return false;
        }
    // Tied embedding (layer 0, matrix 10): int8 x global scale.
    if (!f.load(0, 10, &mx, &err_)) return false;
    std::vector<int8_t> emb((size_t)m.n_vocab * d, 0);
    std::copy_n(mx.data.begin(), std::min(mx.data.size(), emb.size()), emb.begin());
    if (!check(pf_engine_set_embedding(e_, emb.data(), mx.global_scale), "pf_engine_set_embedding")) return false;
    // RMSNorm weights where the file holds them (matrices 7, 8 per layer; 9 final), else 1.
    std::vector<float> an((size_t)m.n_layers * d, 1.0f), fn((size_t)m.n_layers * d, 1.0f), fin(d, 1.0f);
    auto norm = [&](uint32_t l, uint32_t j, float* dst) {
        squeeze::Matrix nm;
        std::string e2;
        if (!f.find(l, j) || !f.load(l, j, &nm, &e2)) return;
        const size_t n = std::min<size_t>(d, nm.data.size());
        for (size_t i = 0; i < n; i++) dst[i] = (float)nm.data[i] * nm.global_scale;
    };
    norm(0, 9, fin.data());
    for (uint32_t l = 0; l < m.n_layers; l++) {
        norm(l, 7, an.data() + (size_t)l * d);
        norm(l, 8, fn.data() + (size_t)l * d);
    }
    if (!check(pf_engine_set_norms(e_, an.data(), fn.data(), fin.data()), "pf_engine_set_norms")) return false;
    // MTP heads: not part of .squeeze files; the seeded generator.
    std::vector<uint8_t> g((size_t)d * (d / 2)), u(g.size()), dn(g.size());
    std::vector<float> gs(d), us(d), ds(d);
    for (uint32_t h = 0; h < m.mtp_heads; h++) {
        if (!check(pf_synth_mtp_matrix(mtp_seed, (int32_t)h, 0, (int32_t)d, g.data(), gs.data()), "pf_synth_mtp_matrix") ||
            !check(pf_synth_mtp_matrix(mtp_seed, (int32_t)h, 1, (int32_t)d, u.data(), us.data()), "pf_synth_mtp_matrix") ||
            !check(pf_synth_mtp_matrix(mtp_seed, (int32_t)h, 2, (int32_t)d, dn.data(), ds.data()), "pf_synth_mtp_matrix") ||
            !check(pf_engine_set_mtp_head(e_, (int32_t)h, g.data(), gs.data(), u.data(), us.data(), dn.data(), ds.data()),
                   "pf_engine_set_mtp_head"))
            return false;
    }
    return true;
}

bool BatchEngine::set_sampling(const SamplingConfig& s) {
    if (!e_) return false;
    pf_sampling_config c{s.temperature, s.top_p, s.top_k, s.greedy ? 1 : 0};
    return check(pf_engine_set_sampling(e_, &c), "pf_engine_set_sampling");
}

bool BatchEngine::set_skip_threshold(float t) {
    if (!e_) return false;
    cfg_.model.skip_threshold = t;
    return check(pf_engine_set_skip_threshold(e_, t), "pf_engine_set_skip_threshold");
}

bool BatchEngine::prefill(const std::vector<std::vector<int32_t>>& prompts, const std::vector<uint32_t>& seeds) {
    if (!e_) return false;
    if (prompts.empty() || prompts.size() > max_seqs_) {
        err_ = "prefill: between 1 and " + std::to_string(max_seqs_) + " prompts";
        return false;
    }
    if (!seeds.empty() && seeds.size() != prompts.size()) {
        err_ = "prefill: one seed per prompt";
        return false;
    }
    std::vector<int32_t> toks;
    std::vector<int64_t> off(1, 0);
    for (const auto& p : prompts) {
        toks.insert(toks.end(), p.begin(), p.end());
        off.push_back((int64_t)toks.size());
    }
    if (!check(pf_engine_prefill(e_, (int32_t)prompts.size(), toks.data(), off.data(),
                                 seeds.empty() ? nullptr : seeds.data()),
               "pf_engine_prefill"))
        return false;
    n_seqs_ = (uint32_t)prompts.size();
    return true;
}

bool BatchEngine::step(std::vector<std::vector<int32_t>>* emitted) {
    if (!e_) return false;
    const uint32_t R = cfg_.model.mtp_heads + 1;
    std::vector<int32_t> n(n_seqs_), em((size_t)n_seqs_ * R);
    if (!check(pf_engine_step(e_, n.data(), em.data()), "pf_engine_step")) return false;
    if (emitted) {
        emitted->assign(n_seqs_, {});
        for (uint32_t i = 0; i < n_seqs_; i++) (*emitted)[i].assign(em.begin() + (size_t)i * R, em.begin() + (size_t)i * R + n[i]);
    }
    return true;
}

bool BatchEngine::generate(const std::vector<std::vector<int32_t>>& prompts, uint32_t max_new_tokens,
                           std::vector<std::vector<int32_t>>* out, const std::vector<uint32_t>& seeds) {
    if (!prefill(prompts, seeds)) return false;
    std::vector<std::vector<int32_t>> got(n_seqs_);
    std::vector<int32_t> pending(n_seqs_);
    if (!check(pf_engine_read_pending(e_, pending.data()), "pf_engine_read_pending")) return false;
    for (uint32_t i = 0; i < n_seqs_; i++) got[i].push_back(pending[i]);  // the prefill's token
    auto done = [&] {
        for (const auto& g : got)
            if (g.size() < max_new_tokens) return false;
        return true;
    };
    std::vector<std::vector<int32_t>> em;
    while (!done()) {
        if (!step(&em)) return false;
        for (uint32_t i = 0; i < n_seqs_; i++) got[i].insert(got[i].end(), em[i].begin(), em[i].end());
    }
    for (auto& g : got) g.resize(max_new_tokens);
    if (out) *out = std::move(got);
    return true;
}

bool BatchEngine::logits(std::vector<float>* out) const {
    if (!e_ || !out) return false;
    out->assign((size_t)n_seqs_ * (cfg_.model.mtp_heads + 1) * cfg_.model.n_vocab, 0.0f);
    return check(pf_engine_read_logits(e_, out->data()), "pf_engine_read_logits");
}

bool BatchEngine::positions(std::vector<int32_t>* out) const {
    if (!e_ || !out) return false;
    out->assign(n_seqs_, 0);
    return check(pf_engine_read_positions(e_, out->data()), "pf_engine_read_positions");
}

bool BatchEngine::pending(std::vector<int32_t>* out) const {
    if (!e_ || !out) return false;
    out->assign(n_seqs_, 0);
    return check(pf_engine_read_pending(e_, out->data()), "pf_engine_read_pending");
}

bool BatchEngine::skip_counts(int64_t* computed, int64_t* skipped) const {
    if (!e_) return false;
    return check(pf_engine_read_skip_counts(e_, computed, skipped), "pf_engine_read_skip_counts");
}

}  // namespace forge

// ref_shim.cpp — extern "C" entry points into the REFERENCE's own functions.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's sources where they lie (src/*.cpp of
// tundefund0-gif/pocketforge) into oracle/_ref/libpfref.so.  The pin tests use
// it to check the CPU restatement (oracle/pf_oracle.cpp) bit for bit, and
// `bench.py --impl reference` times it.  Nothing in pocketforge_b200/ links it.
//
// MTPHeads keeps its weights private; D8 injects seeded weights into both
// sides, so this translation unit reads them with `private` redefined.
#include <cstdint>
#include <cstring>
#include <functional>
#include <memory>
#include <string>
#include <vector>
#include <unordered_map>
#include <thread>
#include <mutex>
#include <condition_variable>
#include <atomic>
#include <queue>
#include <random>

#define private public
#include "forge/mtp.hpp"
#include "forge/engine.hpp"
#undef private
#include "forge/kv_cache.hpp"
#include "forge/layer_skip.hpp"
#include "forge/matmul_neon.hpp"
#include "forge/quant_format.hpp"
#include "literal_script.hpp"

namespace forge {
void pf_ref_seed_sampler(unsigned s);
}

extern "C" {

void pfref_quantize_activation_row(const float* s, int8_t* d, float* sc, uint32_t n) {
    forge::quantize_activation_row(s, d, sc, n);
}
void pfref_dequant_q4_to_int8(const uint8_t* s, int8_t* d, uint32_t n) { forge::dequant_q4_to_int8(s, d, 1.0f, n); }
void pfref_dequant_q2_to_int8(const uint8_t* s, int8_t* d, uint32_t n) { forge::dequant_q2_to_int8(s, d, 1.0f, n); }
void pfref_dequant_ternary_to_int8(const uint8_t* s, int8_t* d, uint32_t n) { forge::dequant_ternary_to_int8(s, d, n); }
void pfref_matmul_int8(const int8_t* A, const int8_t* B, int32_t* C, uint32_t M, uint32_t N, uint32_t K) {
    forge::matmul_int8(A, B, C, M, N, K);
}
void pfref_matmul_quantized(const float* A, const int8_t* B, float* C, uint32_t M, uint32_t N, uint32_t K,
                            const float* ws, const float* as) {
    forge::matmul_quantized(A, B, C, M, N, K, ws, as);
}
void pfref_rmsnorm(float* out, const float* x, const float* w, uint32_t n) { forge::rmsnorm(out, x, w, n); }
void pfref_softmax(float* v, uint32_t n) { forge::softmax(v, n); }
float pfref_dot_product(const float* a, const float* b, uint32_t n) { return forge::dot_product(a, b, n); }

// ---- KVCache ----
void* pfref_kv_create(uint32_t L, uint32_t H, uint32_t hd, uint32_t sink, uint32_t window, uint32_t pool,
                      uint32_t max_ctx) {
    forge::KVCacheConfig c;
    c.n_layers = L;
    c.n_kv_heads = H;
    c.head_dim = hd;
    c.sink_size = sink;
    c.window_size = window;
    c.pool_block = pool;
    c.max_context = max_ctx;
    return new forge::KVCache(c);
}
void pfref_kv_destroy(void* c) { delete (forge::KVCache*)c; }
void pfref_kv_store(void* c, uint32_t l, uint32_t h, uint32_t pos, const float* k, const float* v) {
    ((forge::KVCache*)c)->store(l, h, pos, k, v);
}
uint32_t pfref_kv_scores(void* c, uint32_t l, uint32_t h, const float* q, float* out) {
    return ((forge::KVCache*)c)->attention_scores(l, h, q, out);
}
void pfref_kv_weighted_sum(void* c, uint32_t l, uint32_t h, const float* p, float* out, uint32_t cnt) {
    ((forge::KVCache*)c)->attention_weighted_sum(l, h, p, out, cnt);
}
uint32_t pfref_kv_size(void* c) { return ((forge::KVCache*)c)->size(); }
uint64_t pfref_kv_memory(void* c) { return ((forge::KVCache*)c)->memory_usage(); }

// ---- LayerSkipController ----
void* pfref_skip_create(uint32_t L, uint32_t d, float thr, uint32_t interval) {
    forge::ModelConfig c;
    c.n_layers = L;
    c.n_embd = d;
    c.skip_threshold = thr;
    c.skip_interval = interval;
    return new forge::LayerSkipController(c);
}
void pfref_skip_destroy(void* s) { delete (forge::LayerSkipController*)s; }
int pfref_skip_should_skip(void* s, uint32_t l, const float* x, uint32_t n) {
    return ((forge::LayerSkipController*)s)->should_skip_ffn(l, x, n) ? 1 : 0;
}
void pfref_skip_record(void* s, uint32_t l, const float* x, uint32_t n) {
    ((forge::LayerSkipController*)s)->record_layer_output(l, x, n);
}
void pfref_skip_new_token(void* s) { ((forge::LayerSkipController*)s)->new_token(); }
int pfref_skip_is_anchor(void* s) { return ((forge::LayerSkipController*)s)->is_anchor_token() ? 1 : 0; }
uint32_t pfref_skip_total(void* s) { return ((forge::LayerSkipController*)s)->total_skipped(); }
void pfref_skip_reset(void* s) { ((forge::LayerSkipController*)s)->reset(); }
void pfref_skip_set_threshold(void* s, float t) { ((forge::LayerSkipController*)s)->set_threshold(t); }

// ---- MTPHeads ----
void* pfref_mtp_create(uint32_t heads, uint32_t d, uint32_t vocab) {
    forge::MTPConfig c;
    c.n_mtp_heads = heads;
    c.n_embd = d;
    c.n_vocab = vocab;
    c.mtp_ff_dim = d;
    return new forge::MTPHeads(c);
}
void pfref_mtp_destroy(void* m) { delete (forge::MTPHeads*)m; }
void pfref_mtp_set_head(void* mp, uint32_t h, const uint8_t* g, const float* gs, const uint8_t* u, const float* us,
                        const uint8_t* dn, const float* ds) {
    auto* m = (forge::MTPHeads*)mp;
    const size_t d = m->cfg_.n_embd, mb = d * (d / 2);
    auto& w = m->heads_[h];
    w.gate_q4.assign(g, g + mb);
    w.up_q4.assign(u, u + mb);
    w.down_q4.assign(dn, dn + mb);
    w.gate_scale.assign(gs, gs + d);
    w.up_scale.assign(us, us + d);
    w.down_scale.assign(ds, ds + d);
}
void pfref_mtp_forward(void* mp, const float* hidden, const float* emb, uint64_t emb_n, float* logits) {
    auto* m = (forge::MTPHeads*)mp;
    std::vector<float> table(emb, emb + emb_n);
    auto out = m->forward(hidden, table);
    const size_t V = m->cfg_.n_vocab;
    for (size_t h = 0; h < out.size(); h++) std::memcpy(logits + h * V, out[h].data(), V * sizeof(float));
}
void pfref_mtp_quantize_q4(const float* src, uint8_t* dst, float* scales, uint32_t rows, uint32_t cols) {
    std::vector<float> s;
    forge::MTPHeads::quantize_q4(src, dst, s, rows, cols);
    std::memcpy(scales, s.data(), rows * sizeof(float));
}
int32_t pfref_mtp_argmax(const float* v, uint32_t n) { return forge::MTPHeads::argmax(v, n); }
int pfref_mtp_speculative_accept(void* mp, int32_t token, const float* logits, uint32_t heads) {
    auto* m = (forge::MTPHeads*)mp;
    const size_t V = m->cfg_.n_vocab;
    std::vector<std::vector<float>> l(heads);
    for (uint32_t h = 0; h < heads; h++) l[h].assign(logits + h * V, logits + (h + 1) * V);
    return m->speculative_accept(token, l);
}

// ---- Quantizer / WeightLoader ----
uint64_t pfref_quantize_matrix(const float* data, uint32_t rows, uint32_t cols, int qtype, uint8_t* out) {
    forge::ModelConfig c;
    forge::Quantizer q(c);
    auto v = q.quantize_matrix(data, rows, cols, (uint8_t)qtype);
    if (out) std::memcpy(out, v.data(), v.size());
    return v.size();
}
// Writes a one-block .squeeze with the reference Quantizer (zstd-compressed)
// and reads it back through WeightLoader::load_block_with_scales.
int pfref_squeeze_roundtrip(const char* path, const float* data, uint32_t rows, uint32_t cols, int qtype,
                            int8_t* out, float* row_scales, float* global_scale) {
    forge::ModelConfig c;
    c.n_layers = 1;
    forge::Quantizer q(c);
    auto qd = q.quantize_matrix(data, rows, cols, (uint8_t)qtype);
    auto comp = q.compress_block(qd);
    forge::WeightBlock b{};
    b.layer_id = 0;
    b.matrix_id = 4;
    b.n_rows = rows;
    b.n_cols = cols;
    b.compressed_size = (uint32_t)comp.size();
    b.original_size = (uint32_t)qd.size();
    b.quant_type = (uint8_t)qtype;
    b.offset = 0;
    if (!q.write_squeeze(path, {b}, {comp}, c)) return -1;
    forge::WeightLoader ld;
    if (!ld.open(path)) return -2;
    auto r = ld.load_block_with_scales(0, 4);
    if (r.data.size() != (size_t)rows * cols) return -3;
    std::memcpy(out, r.data.data(), r.data.size());
    std::memcpy(row_scales, r.row_scales.data(), r.row_scales.size() * sizeof(float));
    *global_scale = r.global_scale;
    return 0;
}

// ---- The literal reference engine (Engine::load_model / generate) ----
// Writes a .squeeze whose header carries the model shape and whose only block
// is the tied embedding (0,10), quantized by the reference Quantizer from the
// given floats.  The reference engine never loads layer matrices
// (Engine::load_layer_weights has no caller), so this is the complete input
// its generate() reads.
int pfref_write_model(const char* path, uint32_t n_layers, uint32_t d, uint32_t heads, uint32_t kv_heads,
                      uint32_t ff, uint32_t vocab, uint32_t max_seq, uint32_t mtp_heads, const float* emb,
                      int qtype) {
    forge::ModelConfig c;
    c.n_layers = n_layers;
    c.n_embd = d;
    c.n_heads = heads;
    c.n_kv_heads = kv_heads;
    c.n_ff = ff;
    c.n_vocab = vocab;
    c.max_seq_len = max_seq;
    c.mtp_heads = mtp_heads;
    forge::Quantizer q(c);
    auto qd = q.quantize_matrix(emb, vocab, d, (uint8_t)qtype);
    auto comp = q.compress_block(qd);
    forge::WeightBlock b{};
    b.layer_id = 0;
    b.matrix_id = 10;
    b.n_rows = vocab;
    b.n_cols = d;
    b.compressed_size = (uint32_t)comp.size();
    b.original_size = (uint32_t)qd.size();
    b.quant_type = (uint8_t)qtype;
    return q.write_squeeze(path, {b}, {comp}, c) ? 0 : -1;
}

// A whole model through the reference's own writer: every layer matrix
// (layer-major, matrices 0..6 in ModelConfig order: q, k, v, o, gate, up,
// down) and the tied embedding (0,10) quantized by Quantizer::quantize_matrix
// with its format (qtypes[0..6] per matrix, qtypes[7] for the embedding),
// zstd-compressed by compress_block and written by write_squeeze.  `mats`
// holds the float matrices back to back in that order.
int pfref_write_squeeze_model(const char* path, uint32_t n_layers, uint32_t d, uint32_t heads, uint32_t kv_heads,
                              uint32_t ff, uint32_t vocab, uint32_t max_seq, uint32_t mtp_heads, const float* mats,
                              const int* qtypes) {
    forge::ModelConfig c;
    c.n_layers = n_layers;
    c.n_embd = d;
    c.n_heads = heads;
    c.n_kv_heads = kv_heads;
    c.n_ff = ff;
    c.n_vocab = vocab;
    c.max_seq_len = max_seq;
    c.mtp_heads = mtp_heads;
    forge::Quantizer q(c);
    const uint32_t hd = d / heads;
    const uint32_t rows[7] = {heads * hd, kv_heads * hd, kv_heads * hd, d, ff, ff, d};
    const uint32_t cols[7] = {d, d, d, heads * hd, d, d, ff};
    std::vector<forge::WeightBlock> blocks;
    std::vector<std::vector<uint8_t>> data;
    size_t off = 0;
    auto add = [&](uint32_t layer, uint32_t m, uint32_t r, uint32_t cc, int qt) {
        auto qd = q.quantize_matrix(mats + off, r, cc, (uint8_t)qt);
        off += (size_t)r * cc;
        auto comp = q.compress_block(qd);
        forge::WeightBlock b{};
        b.layer_id = layer;
        b.matrix_id = m;
        b.n_rows = r;
        b.n_cols = cc;
        b.compressed_size = (uint32_t)comp.size();
        b.original_size = (uint32_t)qd.size();
        b.quant_type = (uint8_t)qt;
        blocks.push_back(b);
        data.push_back(std::move(comp));
    };
    for (uint32_t l = 0; l < n_layers; l++)
        for (uint32_t m = 0; m < 7; m++) add(l, m, rows[m], cols[m], qtypes[m]);
    add(0, 10, vocab, d, qtypes[7]);
    return q.write_squeeze(path, blocks, data, c) ? 0 : -1;
}

// One block of a .squeeze file as WeightLoader::load_block_with_scales returns
// it: int8 values [rows * cols], row scales [rows] and the global scale.
// Returns the number of values, or a negative code.
int64_t pfref_load_block(const char* path, uint32_t layer, uint32_t matrix, int8_t* out, float* row_scales,
                         float* global_scale, int64_t max_values) {
    forge::WeightLoader ld;
    if (!ld.open(path)) return -1;
    auto r = ld.load_block_with_scales(layer, matrix);
    if (r.data.empty()) return -2;
    if ((int64_t)r.data.size() > max_values) return -3;
    std::memcpy(out, r.data.data(), r.data.size());
    std::memcpy(row_scales, r.row_scales.data(), r.row_scales.size() * sizeof(float));
    *global_scale = r.global_scale;
    return (int64_t)r.data.size();
}

// Engine::generate on one prompt; returns the number of generated tokens and
// the engine's own tokens_per_second (which counts prompt tokens).
int pfref_literal_generate(const char* path, const int32_t* prompt, uint32_t n, uint32_t max_new, int32_t* out,
                           float* engine_tps) {
    forge::Engine e;
    if (!e.load_model(path)) return -1;
    e.set_max_memory((size_t)1 << 40);  // the 250 MB default stops a 1B model before its first token
    std::vector<int32_t> p(prompt, prompt + n);
    auto r = e.generate(p, max_new);
    const size_t gen = r.tokens.size() > n ? r.tokens.size() - n : 0;
    for (size_t i = 0; i < gen; i++) out[i] = r.tokens[n + i];
    *engine_tps = r.tokens_per_second;
    return (int)gen;
}

// The model of the reference's tests/test_engine.cpp: 2 layers, n_embd 64,
// 4 / 2 heads, FFN 256, vocabulary 256, max_seq_len 128, 2 MTP heads; Q8
// layer matrices of uniform [-1, 1] weights after srand(123), no embedding
// block (so the engine runs its placeholder embedding and logits).
int pfref_write_test_engine_model(const char* path) {
    forge::ModelConfig cfg;
    cfg.n_layers = 2;
    cfg.n_embd = 64;
    cfg.n_heads = 4;
    cfg.n_kv_heads = 2;
    cfg.n_ff = 256;
    cfg.n_vocab = 256;
    cfg.max_seq_len = 128;
    cfg.mtp_heads = 2;
    forge::Quantizer q(cfg);
    std::vector<forge::WeightBlock> blocks;
    std::vector<std::vector<uint8_t>> data;
    srand(123);
    for (uint32_t l = 0; l < cfg.n_layers; l++) {
        for (uint32_t m = 0; m < 7; m++) {
            const uint32_t rows = m == 6 ? 256 : 64, cols = (m == 4 || m == 5) ? 256 : 64;
            std::vector<float> w((size_t)rows * cols);
            for (auto& x : w) x = ((float)rand() / RAND_MAX) * 2.0f - 1.0f;
            auto qd = q.quantize_matrix(w.data(), rows, cols, 0);
            auto comp = q.compress_block(qd);
            forge::WeightBlock b{};
            b.layer_id = l;
            b.matrix_id = m;
            b.n_rows = rows;
            b.n_cols = cols;
            b.compressed_size = (uint32_t)comp.size();
            b.original_size = (uint32_t)qd.size();
            b.quant_type = 0;
            blocks.push_back(b);
            data.push_back(std::move(comp));
        }
    }
    return q.write_squeeze(path, blocks, data, cfg) ? 0 : -1;
}

// A model for the literal engine with the blocks it reads: the tied
// embedding (0, 10) from `emb` (vocab x d floats) and, when `norms` is given,
// the attention and FFN norm rows (l, 7), (l, 8) and the output norm (0, 9)
// from norms[(2 * n_layers + 1) x d] (layer-major attention / FFN rows, then
// the output norm), each quantized by Quantizer::quantize_matrix with `qtype`.
int pfref_write_literal_model(const char* path, uint32_t n_layers, uint32_t d, uint32_t heads, uint32_t kv_heads,
                              uint32_t ff, uint32_t vocab, uint32_t max_seq, uint32_t mtp_heads, const float* emb,
                              const float* norms, int qtype) {
    forge::ModelConfig c;
    c.n_layers = n_layers;
    c.n_embd = d;
    c.n_heads = heads;
    c.n_kv_heads = kv_heads;
    c.n_ff = ff;
    c.n_vocab = vocab;
    c.max_seq_len = max_seq;
    c.mtp_heads = mtp_heads;
    forge::Quantizer q(c);
    std::vector<forge::WeightBlock> blocks;
    std::vector<std::vector<uint8_t>> data;
    auto add = [&](uint32_t layer, uint32_t m, const float* x, uint32_t rows, uint32_t cols) {
        auto qd = q.quantize_matrix(x, rows, cols, (uint8_t)qtype);
        auto comp = q.compress_block(qd);
        forge::WeightBlock b{};
        b.layer_id = layer;
        b.matrix_id = m;
        b.n_rows = rows;
        b.n_cols = cols;
        b.compressed_size = (uint32_t)comp.size();
        b.original_size = (uint32_t)qd.size();
        b.quant_type = (uint8_t)qtype;
        blocks.push_back(b);
        data.push_back(std::move(comp));
    };
    add(0, 10, emb, vocab, d);
    if (norms) {
        for (uint32_t l = 0; l < n_layers; l++) {
            add(l, 7, norms + (size_t)(2 * l) * d, 1, d);
            add(l, 8, norms + (size_t)(2 * l + 1) * d, 1, d);
        }
        add(0, 9, norms + (size_t)(2 * n_layers) * d, 1, d);
    }
    return q.write_squeeze(path, blocks, data, c) ? 0 : -1;
}

// The literal-engine script (oracle/literal_script.hpp) on the reference's
// Engine, with its sampler reseeded to 42 as at process start.  Returns the
// transcript length, or -(needed length) when `cap` is too small.
int64_t pfref_literal_script(const char* path, uint32_t seed, uint64_t max_memory, uint32_t long_tokens, char* out,
                             int64_t cap) {
    forge::pf_ref_seed_sampler(42);
    forge::Engine e;
    const std::string t = literal_script::run(e, path, seed, (size_t)max_memory, long_tokens);
    if ((int64_t)t.size() + 1 > cap) return -(int64_t)(t.size() + 1);
    std::memcpy(out, t.c_str(), t.size() + 1);
    return (int64_t)t.size();
}

// ---- Engine sampling (src/engine.cpp:881-1003) ----
void* pfref_engine_create(void) { return new forge::Engine(); }
void pfref_engine_destroy(void* e) { delete (forge::Engine*)e; }
void pfref_seed_sampler(uint32_t s) { forge::pf_ref_seed_sampler(s); }
int32_t pfref_sample(void* e, const float* lg, uint32_t n, float temperature, float top_p, uint32_t top_k,
                     int greedy) {
    forge::SamplingConfig c;
    c.temperature = temperature;
    c.top_p = top_p;
    c.top_k = top_k;
    c.greedy = greedy != 0;
    return ((forge::Engine*)e)->sample(lg, n, c);
}
int32_t pfref_sample_greedy(void* e, const float* lg, uint32_t n) { return ((forge::Engine*)e)->sample_greedy(lg, n); }
int32_t pfref_sample_top_p(void* e, const float* lg, uint32_t n, float p, float t) {
    return ((forge::Engine*)e)->sample_top_p(lg, n, p, t);
}
int32_t pfref_sample_top_k(void* e, const float* lg, uint32_t n, uint32_t k, float t) {
    return ((forge::Engine*)e)->sample_top_k(lg, n, k, t);
}

}  // extern "C"

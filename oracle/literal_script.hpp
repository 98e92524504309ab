// literal_script.hpp — TEST INFRASTRUCTURE: one fixed sequence of forge::Engine
// calls whose transcript the reference-compat parity test compares.
//
// Compiled twice: into oracle/_ref/libpfref.so against the reference's own
// headers and engine (ref_shim.cpp, pfref_literal_script), and into
// tests/cpp/literal_driver.cpp against this repository's forge:: headers with
// reference-compat mode on.  Only the API both share is used.
//
// The sequence follows the reference's tests/test_engine.cpp (one engine:
// generate {101,102,103} x 10, forward {42}, generate {1,2,3} and {10,20,30}
// x 5, MTP off for {5,10,15}, skip threshold 0.5 for {1,2,3}) and then, when
// `long_tokens` > 0, one long generation that fills the KV window, evicts and
// pools, and a last forward.
#pragma once
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

namespace literal_script {

inline void hex_floats(std::string& out, const std::vector<float>& v) {
    char b[16];
    for (float x : v) {
        uint32_t u;
        std::memcpy(&u, &x, 4);
        std::snprintf(b, sizeof b, " %08x", u);
        out += b;
    }
    out += "\n";
}

// srand(seed) immediately before load_model: the MTP weights the engine draws
// from rand() then match on both sides.  max_memory == 0 keeps the default.
template <class Engine>
std::string run(Engine& e, const char* path, unsigned seed, size_t max_memory, uint32_t long_tokens) {
    std::string out;
    char b[256];
    std::srand(seed);
    if (!e.load_model(path)) return "load failed\n";
    if (max_memory) e.set_max_memory(max_memory);
    std::snprintf(b, sizeof b, "config layers=%u embd=%u heads=%u kv=%u vocab=%u seq=%u mtp=%u window=%u\n",
                  e.config().n_layers, e.config().n_embd, e.config().n_heads, e.config().n_kv_heads,
                  e.config().n_vocab, e.config().max_seq_len, e.config().mtp_heads, e.config().kv_cache_size);
    out += b;
    auto gen = [&](const char* name, const std::vector<int32_t>& prompt, uint32_t n) {
        auto r = e.generate(prompt, n);
        std::snprintf(b, sizeof b, "gen %s acc=%d rej=%d oom=%d skipped=%d:", name, r.mtp_accepted, r.mtp_rejected,
                      (int)r.oom_protected, r.layers_skipped);
        out += b;
        for (size_t i = prompt.size(); i < r.tokens.size(); i++) {
            std::snprintf(b, sizeof b, " %d", r.tokens[i]);
            out += b;
        }
        out += "\n";
    };
    auto fwd = [&](const char* name, const std::vector<int32_t>& tokens) {
        std::vector<float> h(e.config().n_embd, 0.0f);
        auto lg = e.forward_with_hidden(tokens, h);
        out += std::string("logits ") + name + ":";
        hex_floats(out, lg);
        out += std::string("hidden ") + name + ":";
        hex_floats(out, h);
    };
    auto mem = [&](const char* name) {
        auto s = e.get_memory_stats();
        std::snprintf(b, sizeof b, "mem %s kv=%zu mtp=%zu act=%zu other=%zu\n", name, s.kv_cache, s.mtp_heads,
                      s.activations, s.other);
        out += b;
    };
    gen("a", {101, 102, 103}, 10);
    fwd("b", {42});
    gen("c", {1, 2, 3}, 5);
    gen("d", {10, 20, 30}, 5);
    e.set_mtp_enabled(false);
    gen("e", {5, 10, 15}, 5);
    e.set_mtp_enabled(true);
    e.set_layer_skip_threshold(0.5f);
    gen("f", {1, 2, 3}, 5);
    e.set_layer_skip_threshold(0.01f);
    mem("g");
    if (long_tokens) {
        gen("h", {7, 8, 9, 10}, long_tokens);
        mem("i");
        fwd("j", {3});
    }
    return out;
}

}  // namespace literal_script

// literal.hpp — state of forge::Engine's reference-compat mode (internal to
// the library; see literal.cpp).
#pragma once
#include <cstdint>
#include <random>
#include <string>
#include <vector>

#include "../csrc/literal.h"
#include "device.hpp"
#include "forge/engine.hpp"

namespace forge {

// The process-wide generator of Engine::sample (the reference's file-static
// std::mt19937 seeded 42, src/engine.cpp:16).
std::mt19937& reference_rng();

namespace detail {

// Size and capacity of a std::vector as libstdc++ grows it (resize or
// push_back past the capacity: new capacity = size + max(size, added)), for
// the reference's memory statistics, which count vector capacities.
struct VecModel {
    size_t size = 0, cap = 0;
    void resize(size_t n) {
        if (n > cap) cap = size + std::max(size, n - size);
        size = n;
    }
    void push_back() { resize(size + 1); }
};

constexpr uint32_t kSinkSize = 4;   // KVCacheConfig sink_size set by load_model
constexpr uint32_t kSinkRows = 8;   // rows the reference allocates for the sink tier
constexpr uint32_t kPoolBlock = 64; // KVCacheConfig pool_block set by load_model
constexpr float kRopeTheta = 5000000.0f;

}  // namespace detail

struct Engine::Literal {
    ModelConfig cfg;
    uint32_t L = 0, d = 0, H = 0, KV = 0, hd = 0, V = 0, ring = 1, max_ctx = 0;
    bool emb_loaded = false, mtp = false, hidden_valid = false;
    uint32_t emb_rows = 0;
    float threshold = 0.01f;

    // Device state.
    dev::Buffer emb, attn_w, ffn_w, rope_c, rope_s;
    dev::Buffer sk, sv, sks, svs, wk, wv, wks, wvs, pk, pv, pks, pvs, ak, av;
    dev::Buffer hidden, last_hidden, q, k, v, attn_out, scores, self_p, skip_cache;
    dev::Buffer logits, mtp_h, mtp_work, mtp_logits, uniforms, tokens;
    struct Head {
        dev::Buffer gate, up, down, gs, us, ds;
    };
    std::vector<Head> heads;
    pf::lit::Model m;

    // Host mirror of each layer's tiers.
    struct Tier {
        uint32_t n_sink = 0, n_win = 0, head = 0, n_pool = 0, n_acc = 0;
    };
    std::vector<Tier> tiers;
    uint32_t pool_cap = 0;

    // Memory statistics as the reference counts them (Engine::get_memory_stats).
    detail::VecModel scores_vec, scores_out_vec;
    std::vector<uint32_t> pool_rows_model;  // pooled rows per layer (all kv heads alike)

    std::string err;

    bool fail(const std::string& e) {
        err = e;
        std::fprintf(stderr, "forge::Engine (reference-compat): %s\n", e.c_str());
        return false;
    }
    bool dev_ok(pf_status s, const char* what) {
        if (s == PF_OK) return true;
        return fail(std::string(what) + ": " + pf_last_error());
    }

    template <class T>
    T* alloc(dev::Buffer& b, size_t n, bool zero = true) {
        void* p = b.reserve(n * sizeof(T) + 16);
        if (p && zero) cudaMemset(p, 0, n * sizeof(T) + 16);
        return static_cast<T*>(p);
    }

    bool load(const std::string& path);
    bool grow_pool();
    bool forward(int32_t token, bool want_logits);
    bool sample_dev(const float* lg, uint32_t rows, bool greedy, int32_t* out);
    bool mtp_drafts(std::vector<int32_t>* preds);
    size_t memory_total(Engine::MemoryStats* s) const;
    GenerationResult generate(const std::vector<int32_t>& prompt, uint32_t max_new, TokenCallback cb,
                              ProgressCallback progress, size_t max_memory);
};

}  // namespace forge

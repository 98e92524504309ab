// literal.cpp — forge::Engine in reference-compat mode: the reference's
// literal Engine (src/engine.cpp:47-203 load_model, :276-396 generate,
// :459-589 forward_with_hidden) with its forward on the device.
//
// What the literal engine computes, and this mode reproduces:
//  - the projection weights of the file are never loaded (load_layer_weights
//    has no caller), so Q = K = V = 0.1 x the normed input and the FFN output
//    is max(0, sum of the normed input x 0.01) in every element;
//  - RoPE and the KV store use the layer index as the position (theta 5e6),
//    a K head is rotated once per query head that maps to it, the attention
//    output of every head but the last lands in entry range 0..head_dim;
//  - generate() forwards the last prompt token again, samples the first token
//    and every MTP draft with the default sampling (top-p 0.95, T 0.8) from
//    the process-wide generator, verifies drafts one forward at a time against
//    the greedy token, samples a corrective token on a mismatch, and never
//    rolls the KV cache back;
//  - the unembedding uses the hidden state before the final norm.
// The host keeps the tier counters of every layer (they do not depend on the
// data: every forward stores one entry per layer at position = layer) and the
// control flow of generate(); the kernels (csrc/literal.cu) do the arithmetic.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>

#include "literal.hpp"
#include "squeeze.hpp"

namespace forge {

using namespace detail;

bool Engine::Literal::load(const std::string& path) {
    squeeze::File f;
    std::string e;
    if (!f.open(path, &e)) return fail(e);
    cfg = f.config();
    // src/engine.cpp:55-59.
    if (!cfg.check_memory_budget()) {
        std::fprintf(stderr, "WARNING: Config may exceed budget. Reducing ctx from %u to %u\n", cfg.kv_cache_size,
                     cfg.kv_cache_size / 2);
        cfg.kv_cache_size /= 2;
    }
    L = cfg.n_layers;
    d = cfg.n_embd;
    H = cfg.n_heads;
    KV = cfg.n_kv_heads;
    hd = cfg.head_dim();
    V = cfg.n_vocab;
    max_ctx = cfg.max_seq_len;
    ring = std::min(std::min(cfg.kv_cache_size, 8192u), max_ctx);
    if (!L || !d || !H || !KV || !hd || !V || ring == 0) return fail("model dimensions or window of zero");
    if (d > pf::lit::kMaxEmbd || H * hd > d || KV * hd > d || d % 2)
        return fail("reference-compat mode needs n_embd even and <= 4096, heads x head_dim <= n_embd");
    if (V > 16384) return fail("reference-compat mode supports vocabularies of up to 16384 entries");
    threshold = cfg.skip_threshold;

    // MTP heads: MTPHeads' constructor draws the weights and load_model draws
    // them again (src/engine.cpp:75-83, src/mtp.cpp:9-44), so rand() advances
    // twice and the second set is kept.
    mtp = cfg.mtp_enabled;
    heads.clear();
    if (mtp) {
        const uint32_t ff = d;
        const float init = 1.0f / std::sqrt((float)d);
        std::vector<float> fw;
        std::vector<uint8_t> qb;
        std::vector<float> sc;
        heads.resize(cfg.mtp_heads);
        for (int pass = 0; pass < 2; pass++) {
            for (auto& h : heads) {
                auto make = [&](uint32_t rows, uint32_t cols, dev::Buffer& wq, dev::Buffer& ws) {
                    fw.resize((size_t)rows * cols);
                    for (auto& x : fw) x = ((float)rand() / (float)RAND_MAX * 2.0f - 1.0f) * init;
                    if (pass == 0) return true;
                    qb.assign((size_t)rows * (cols / 2), 0);
                    sc.assign(rows, 1.0f);
                    detail::quantize_q4_rows(fw.data(), qb.data(), sc.data(), rows, cols);
                    return alloc<uint8_t>(wq, qb.size(), false) && alloc<float>(ws, sc.size(), false) &&
                           dev::to_dev(wq.as<void>(), qb.data(), qb.size(), "compat MTP weights") &&
                           dev::to_dev(ws.as<void>(), sc.data(), sc.size() * 4, "compat MTP weights");
                };
                if (!make(d, ff, h.gate, h.gs) || !make(d, ff, h.up, h.us) || !make(ff, d, h.down, h.ds))
                    return fail("MTP weight upload failed");
            }
        }
    }

    // RoPE tables at position = layer index (src/engine.cpp:646-672).
    std::vector<float> rc((size_t)L * hd), rs((size_t)L * hd);
    for (uint32_t l = 0; l < L; l++) {
        for (uint32_t i = 0; i < hd; i += 2) {
            const float freq = 1.0f / std::pow(kRopeTheta, (float)i / (float)hd);
            rs[(size_t)l * hd + i] = std::sin((float)l * freq);
            rc[(size_t)l * hd + i] = std::cos((float)l * freq);
            if (i + 1 < hd) {
                rs[(size_t)l * hd + i + 1] = rs[(size_t)l * hd + i];
                rc[(size_t)l * hd + i + 1] = rc[(size_t)l * hd + i];
            }
        }
    }

    // Norm weights (l, 7) and (l, 8): int8 x global scale over min(n_embd,
    // n_cols) entries, 1.0 elsewhere (src/engine.cpp:170-201).  The output
    // norm (0, 9) feeds nothing the literal forward returns.
    std::vector<float> aw((size_t)L * d, 1.0f), fwt((size_t)L * d, 1.0f);
    for (uint32_t l = 0; l < L; l++) {
        for (uint32_t mid = 7; mid <= 8; mid++) {
            if (!f.find(l, mid)) continue;
            squeeze::Matrix mt;
            if (!f.load(l, mid, &mt, &e) || mt.data.empty()) continue;
            const uint32_t n = std::min(d, mt.cols);
            float* dst = (mid == 7 ? aw : fwt).data() + (size_t)l * d;
            for (uint32_t i = 0; i < n && i < mt.data.size(); i++) dst[i] = (float)mt.data[i] * mt.global_scale;
        }
    }

    // Embedding table (0, 10): min(n_vocab, 16384) rows, int8 x global scale,
    // filled as far as the block's values reach (src/engine.cpp:143-165).
    emb_loaded = false;
    emb_rows = std::min(V, 16384u);
    std::vector<int8_t> et((size_t)emb_rows * d, 0);
    float emb_scale = 1.0f;
    if (f.find(0, 10)) {
        squeeze::Matrix mt;
        if (f.load(0, 10, &mt, &e) && !mt.data.empty()) {
            std::memcpy(et.data(), mt.data.data(), std::min(et.size(), mt.data.size()));
            emb_scale = mt.global_scale;
            emb_loaded = true;
        }
    }

    // Device buffers.
    const size_t U = (size_t)L * KV;
    pool_cap = 64;
    tiers.assign(L, Tier{});
    pool_rows_model.assign(L, 0);
    hidden_valid = false;
    bool okb = alloc<int8_t>(emb, et.size()) && dev::to_dev(emb.as<void>(), et.data(), et.size(), "compat embedding") &&
               alloc<float>(attn_w, aw.size()) && dev::to_dev(attn_w.as<void>(), aw.data(), aw.size() * 4, "compat") &&
               alloc<float>(ffn_w, fwt.size()) && dev::to_dev(ffn_w.as<void>(), fwt.data(), fwt.size() * 4, "compat") &&
               alloc<float>(rope_c, rc.size()) && dev::to_dev(rope_c.as<void>(), rc.data(), rc.size() * 4, "compat") &&
               alloc<float>(rope_s, rs.size()) && dev::to_dev(rope_s.as<void>(), rs.data(), rs.size() * 4, "compat");
    okb = okb && alloc<int8_t>(sk, U * kSinkRows * hd) && alloc<int8_t>(sv, U * kSinkRows * hd) &&
          alloc<float>(sks, U * kSinkRows) && alloc<float>(svs, U * kSinkRows) && alloc<int8_t>(wk, U * ring * hd) &&
          alloc<int8_t>(wv, U * ring * hd) && alloc<float>(wks, U * ring) && alloc<float>(wvs, U * ring) &&
          alloc<int8_t>(pk, U * pool_cap * hd) && alloc<int8_t>(pv, U * pool_cap * hd) &&
          alloc<float>(pks, U * pool_cap) && alloc<float>(pvs, U * pool_cap) && alloc<double>(ak, U * hd) &&
          alloc<double>(av, U * hd);
    // The reference initialises sink and window scales to 1.0 (src/kv_cache.cpp:44-51).
    if (okb) {
        std::vector<float> ones(U * std::max(kSinkRows, ring), 1.0f);
        okb = dev::to_dev(sks.as<void>(), ones.data(), U * kSinkRows * 4, "compat") &&
              dev::to_dev(svs.as<void>(), ones.data(), U * kSinkRows * 4, "compat") &&
              dev::to_dev(wks.as<void>(), ones.data(), U * ring * 4, "compat") &&
              dev::to_dev(wvs.as<void>(), ones.data(), U * ring * 4, "compat");
    }
    const uint32_t stride = kSinkRows + pool_cap + ring + 1;
    okb = okb && alloc<float>(hidden, d) && alloc<float>(last_hidden, d) && alloc<float>(q, d) &&
          alloc<float>(k, d) && alloc<float>(v, d) && alloc<float>(attn_out, d) &&
          alloc<float>(scores, (size_t)H * stride) && alloc<float>(self_p, H) && alloc<float>(skip_cache, (size_t)L * d) &&
          alloc<float>(logits, V) && alloc<float>(mtp_h, d) && alloc<float>(mtp_work, 3 * (size_t)d) &&
          alloc<float>(mtp_logits, (size_t)std::max(1u, cfg.mtp_heads) * V) &&
          alloc<float>(uniforms, std::max(1u, cfg.mtp_heads)) && alloc<int32_t>(tokens, std::max(1u, cfg.mtp_heads));
    if (!okb) return fail("device allocation failed");

    m = pf::lit::Model{};
    m.n_layers = L;
    m.d = d;
    m.n_heads = H;
    m.n_kv = KV;
    m.hd = hd;
    m.n_vocab = V;
    m.emb_rows = emb_rows;
    m.emb = emb.as<int8_t>();
    m.emb_scale = emb_scale;
    m.emb_loaded = emb_loaded ? 1 : 0;
    m.attn_w = attn_w.as<float>();
    m.ffn_w = ffn_w.as<float>();
    m.rope_cos = rope_c.as<float>();
    m.rope_sin = rope_s.as<float>();
    m.c.sk = sk.as<int8_t>();
    m.c.sv = sv.as<int8_t>();
    m.c.sks = sks.as<float>();
    m.c.svs = svs.as<float>();
    m.c.wk = wk.as<int8_t>();
    m.c.wv = wv.as<int8_t>();
    m.c.wks = wks.as<float>();
    m.c.wvs = wvs.as<float>();
    m.c.pk = pk.as<int8_t>();
    m.c.pv = pv.as<int8_t>();
    m.c.pks = pks.as<float>();
    m.c.pvs = pvs.as<float>();
    m.c.ak = ak.as<double>();
    m.c.av = av.as<double>();
    m.c.sink_cap = kSinkRows;
    m.c.ring = ring;
    m.c.pool_cap = pool_cap;
    m.hidden = hidden.as<float>();
    m.q = q.as<float>();
    m.k = k.as<float>();
    m.v = v.as<float>();
    m.attn_out = attn_out.as<float>();
    m.scores = scores.as<float>();
    m.self_p = self_p.as<float>();
    m.skip_cache = skip_cache.as<float>();
    m.score_stride = stride;
    m.skip_threshold = threshold;
    m.skip_anchor = cfg.skip_interval == 0 ? 1 : 0;

    // The score buffers of the reference (src/engine.cpp:117-119), grown from
    // whatever set_max_context gave them before the load.
    scores_vec.resize((size_t)cfg.kv_cache_size + 4096);
    scores_out_vec.resize((size_t)cfg.kv_cache_size + 4096);
    return true;
}

// Pooled rows outgrew the device arrays: double them, keeping each unit's rows.
bool Engine::Literal::grow_pool() {
    const size_t U = (size_t)L * KV;
    const uint32_t cap2 = pool_cap * 2;
    dev::Buffer nk, nv, nks, nvs, nsc;
    if (!alloc<int8_t>(nk, U * cap2 * hd) || !alloc<int8_t>(nv, U * cap2 * hd) || !alloc<float>(nks, U * cap2) ||
        !alloc<float>(nvs, U * cap2) || !alloc<float>(nsc, (size_t)H * (kSinkRows + cap2 + ring + 1)))
        return fail("device allocation failed (pool tier)");
    auto copy = [&](dev::Buffer& dst, dev::Buffer& src, size_t row_bytes, size_t new_row_bytes) {
        return dev::cuda_ok(cudaMemcpy2D(dst.as<void>(), new_row_bytes, src.as<void>(), row_bytes, row_bytes, U,
                                         cudaMemcpyDeviceToDevice),
                            "compat pool growth");
    };
    if (!copy(nk, pk, (size_t)pool_cap * hd, (size_t)cap2 * hd) || !copy(nv, pv, (size_t)pool_cap * hd, (size_t)cap2 * hd) ||
        !copy(nks, pks, (size_t)pool_cap * 4, (size_t)cap2 * 4) || !copy(nvs, pvs, (size_t)pool_cap * 4, (size_t)cap2 * 4))
        return false;
    pk = std::move(nk);
    pv = std::move(nv);
    pks = std::move(nks);
    pvs = std::move(nvs);
    scores = std::move(nsc);
    pool_cap = cap2;
    m.c.pk = pk.as<int8_t>();
    m.c.pv = pv.as<int8_t>();
    m.c.pks = pks.as<float>();
    m.c.pvs = pvs.as<float>();
    m.c.pool_cap = pool_cap;
    m.scores = scores.as<float>();
    m.score_stride = kSinkRows + pool_cap + ring + 1;
    return true;
}

// One literal forward of `token` (src/engine.cpp:459-589); logits into
// `logits` when asked for (the prompt loop discards them).
bool Engine::Literal::forward(int32_t token, bool want_logits) {
    m.skip_threshold = threshold;
    if (!dev_ok(pf::lit::embed(m, token, nullptr), "embed")) return false;
    for (uint32_t l = 0; l < L; l++) {
        Tier& t = tiers[l];
        pf::lit::Tiers before{t.n_sink, t.n_pool, t.n_win, t.head};
        pf::lit::Store op;
        const uint32_t pos = l;  // the layer index is the position (src/engine.cpp:518, :780-785)
        Tier after = t;
        if (pos < max_ctx) {
            if (pos < kSinkSize) {
                op.kind = 1;
                op.slot = pos;
                after.n_sink = std::max(t.n_sink, pos + 1);
            } else {
                op.kind = 2;
                op.slot = t.head;
                if (t.n_win >= ring) {
                    op.evict = 1;
                    op.acc_n = t.n_acc + 1;
                    op.finalize = op.acc_n >= kPoolBlock ? 1 : 0;
                    op.pool_row = t.n_pool;
                    if (op.finalize && t.n_pool >= pool_cap && !grow_pool()) return false;
                    after.n_acc = op.finalize ? 0 : op.acc_n;
                    if (op.finalize) after.n_pool++;
                } else {
                    after.n_win++;
                }
                after.head = (t.head + 1) % ring;
            }
        }
        if (!dev_ok(pf::lit::layer(m, l, before, op, nullptr), "layer")) return false;
        t = after;
        pool_rows_model[l] = t.n_pool;
    }
    if (!dev::cuda_ok(cudaMemcpyAsync(last_hidden.as<void>(), hidden.as<void>(), (size_t)d * 4,
                                      cudaMemcpyDeviceToDevice, nullptr),
                      "compat forward"))
        return false;
    hidden_valid = true;
    if (!want_logits) return true;
    if (emb_loaded) return dev_ok(pf::lit::unembed(m, hidden.as<float>(), logits.as<float>(), nullptr), "unembed");
    return dev_ok(pf::lit::placeholder_logits(token, V, logits.as<float>(), nullptr), "placeholder logits");
}

// Engine::sample with the default SamplingConfig (top-p 0.95, temperature
// 0.8: one uniform per row from the process-wide generator) or
// Engine::sample_greedy, for `rows` consecutive logit rows on the device.
bool Engine::Literal::sample_dev(const float* lg, uint32_t rows, bool greedy, int32_t* out) {
    int32_t* dt = tokens.as<int32_t>();
    if (greedy) {
        if (!dev_ok(pf_argmax_rows(lg, (int32_t)rows, (int32_t)V, dt, nullptr), "sample_greedy")) return false;
    } else {
        std::vector<float> u(rows);
        for (auto& x : u) x = std::uniform_real_distribution<float>(0.0f, 1.0f)(reference_rng());
        SamplingConfig sc;
        pf_sampling_config c{sc.temperature, sc.top_p, sc.top_k, 0};
        if (!dev::to_dev(uniforms.as<void>(), u.data(), rows * 4, "sample") ||
            !dev_ok(pf_sample_rows(lg, (int32_t)rows, (int32_t)V, &c, uniforms.as<float>(), dt, nullptr), "sample"))
            return false;
    }
    return dev::to_host(out, dt, rows * 4, "sample");
}

// MTPHeads::forward on the last hidden state (src/mtp.cpp:46-127), then one
// default-config sample per head in head order.
bool Engine::Literal::mtp_drafts(std::vector<int32_t>* preds) {
    const uint32_t nh = (uint32_t)heads.size();
    preds->assign(nh, 0);
    if (!nh) return true;
    if (!dev::cuda_ok(cudaMemcpyAsync(mtp_h.as<void>(), last_hidden.as<void>(), (size_t)d * 4,
                                      cudaMemcpyDeviceToDevice, nullptr),
                      "compat MTP"))
        return false;
    for (uint32_t h = 0; h < nh; h++) {
        Head& w = heads[h];
        if (!dev_ok(pf::lit::mtp_ffn(mtp_h.as<float>(), w.gate.as<uint8_t>(), w.gs.as<float>(), w.up.as<uint8_t>(),
                                     w.us.as<float>(), w.down.as<uint8_t>(), w.ds.as<float>(), d, d,
                                     mtp_work.as<float>(), nullptr),
                    "MTP head"))
            return false;
        // Tied unembedding: the table holds n_vocab rows (n_vocab <= 16384).
        if (!dev_ok(pf::lit::unembed(m, mtp_h.as<float>(), mtp_logits.as<float>() + (size_t)h * V, nullptr),
                    "MTP unembed"))
            return false;
    }
    return sample_dev(mtp_logits.as<float>(), nh, false, preds->data());
}

size_t Engine::Literal::memory_total(Engine::MemoryStats* s) const {
    Engine::MemoryStats st;
    // KVCache::memory_usage (src/kv_cache.cpp:218-240): fixed tiers per unit,
    // plus pooled rows in vectors grown by resize / push_back.
    size_t kv_unit = (size_t)kSinkRows * hd * 2 + kSinkRows * 4 * 2 + (size_t)ring * hd * 2 + (size_t)ring * 4 * 3 +
                     (size_t)hd * 8 * 2;
    size_t kv = kv_unit * L * KV;
    for (uint32_t l = 0; l < L; l++) {
        VecModel rows, rec;
        for (uint32_t p = 0; p < pool_rows_model[l]; p++) {
            rows.resize((size_t)(p + 1) * hd);
            rec.push_back();
        }
        kv += (size_t)KV * (rows.cap * 2 + rec.cap * 4 * 4);
    }
    st.kv_cache = kv;
    // MTPHeads::memory_usage (src/mtp.cpp:150-161).
    st.mtp_heads = mtp ? heads.size() * ((size_t)d * (d / 2) * 3 + (size_t)d * 3 * 4) : 0;
    // Activation vectors (src/engine.cpp:1013-1026).
    const size_t attn_sz = std::max((size_t)H * hd, (size_t)d), kv_sz = std::max((size_t)KV * hd, (size_t)d);
    st.activations = ((size_t)d * 6 + attn_sz * 2 + kv_sz * 2 + scores_vec.cap + scores_out_vec.cap + V) * 4;
    if (emb_loaded) st.other = (size_t)emb_rows * d * 4 + (size_t)V * 4;
    if (s) *s = st;
    return st.total();
}

GenerationResult Engine::Literal::generate(const std::vector<int32_t>& prompt, uint32_t max_new, TokenCallback cb,
                                           ProgressCallback progress, size_t max_memory) {
    GenerationResult r;
    const auto t0 = std::chrono::high_resolution_clock::now();
    bool okf = true;
    for (size_t i = 0; i < prompt.size() && okf; i++) {
        okf = forward(prompt[i], false);
        if (progress && i % 10 == 0) progress((float)i / (float)(prompt.size() + max_new));
    }
    r.tokens = prompt;
    uint32_t n_gen = 0;
    int32_t cur = prompt.empty() ? 0 : prompt.back();
    std::vector<int32_t> preds;
    while (okf && n_gen < max_new) {
        if (memory_total(nullptr) > max_memory) {
            std::fprintf(stderr, "OOM protection: hit limit\n");
            r.oom_protected = true;
            break;
        }
        if (cfg.mtp_enabled && mtp && hidden_valid && emb_loaded && n_gen + 4 <= max_new) {
            int32_t t1 = 0;
            if (!(okf = forward(cur, true) && sample_dev(logits.as<float>(), 1, false, &t1))) break;
            r.tokens.push_back(t1);
            n_gen++;
            if (cb) cb(t1, 1.0f);
            if (!(okf = mtp_drafts(&preds))) break;
            int accepted = 0, rejected = 0;
            for (size_t h = 0; h < preds.size(); h++) {
                const int32_t in = h == 0 ? t1 : preds[h - 1];
                int32_t main_pred = 0;
                if (!(okf = forward(in, true) && sample_dev(logits.as<float>(), 1, true, &main_pred))) break;
                if (main_pred == preds[h]) {
                    r.tokens.push_back(preds[h]);
                    n_gen++;
                    accepted++;
                    if (cb) cb(preds[h], 1.0f);
                } else {
                    int32_t corr = 0;
                    if (!(okf = sample_dev(logits.as<float>(), 1, false, &corr))) break;
                    if (corr != preds[h]) {
                        r.tokens.push_back(corr);
                        n_gen++;
                        rejected++;
                        if (cb) cb(corr, 1.0f);
                    }
                    break;
                }
            }
            r.mtp_accepted += accepted;
            r.mtp_rejected += rejected;
            cur = r.tokens.back();
            continue;
        }
        if (!(okf = forward(cur, true))) break;
        if (progress) progress((float)(prompt.size() + n_gen) / (float)(prompt.size() + max_new));
        if (!(okf = sample_dev(logits.as<float>(), 1, false, &cur))) break;
        r.tokens.push_back(cur);
        n_gen++;
        if (cb) cb(cur, 1.0f);
    }
    const float el = std::chrono::duration<float>(std::chrono::high_resolution_clock::now() - t0).count();
    r.tokens_per_second = el > 0 ? (float)r.tokens.size() / el : 0.0f;
    r.peak_memory_bytes = memory_total(nullptr);
    r.layers_skipped = 0;  // LayerSkipController::total_skipped(): the counter is never incremented
    return r;
}

// ---- forge::Engine entry points in reference-compat mode ----

bool Engine::compat_load(const std::string& path) {
    // A fresh literal engine; the score buffers keep what set_max_context did
    // to them before (the reference resizes, never recreates, them).
    std::unique_ptr<Literal> fresh(new Literal);
    if (lit_) {
        fresh->scores_vec = lit_->scores_vec;
        fresh->scores_out_vec = lit_->scores_out_vec;
    }
    lit_ = std::move(fresh);
    if (!lit_->load(path)) {
        err_ = lit_->err;
        lit_->err.clear();
        return false;
    }
    // load_model replaces the config with the file's (src/engine.cpp:52-53):
    // earlier set_mtp_enabled / set_layer_skip_threshold / set_max_memory
    // calls do not survive it.
    config_ = lit_->cfg;
    mtp_enabled_ = config_.mtp_enabled;
    skip_threshold_ = config_.skip_threshold;
    max_memory_ = config_.max_memory;
    return true;
}

GenerationResult Engine::compat_generate(const std::vector<int32_t>& prompt, uint32_t max_new, TokenCallback cb,
                                         ProgressCallback progress) {
    if (!lit_ || !lit_->L) {
        GenerationResult r;
        r.tokens = prompt;
        return r;
    }
    lit_->cfg.mtp_enabled = mtp_enabled_;
    lit_->threshold = skip_threshold_;
    GenerationResult r = lit_->generate(prompt, max_new, cb, progress, max_memory_);
    if (!lit_->err.empty()) err_ = lit_->err;
    return r;
}

std::vector<float> Engine::compat_forward(const std::vector<int32_t>& tokens, std::vector<float>& hidden_out) {
    const uint32_t d = config_.n_embd, V = config_.n_vocab;
    if (tokens.empty()) {
        hidden_out.assign(d, 0.0f);
        return std::vector<float>(V, 0.0f);
    }
    std::vector<float> out;
    if (!lit_ || !lit_->L) return out;
    lit_->threshold = skip_threshold_;
    if (!lit_->forward(tokens.back(), true)) {
        err_ = lit_->err;
        return out;
    }
    out.resize(V);
    if (!dev::to_host(out.data(), lit_->logits.as<void>(), (size_t)V * 4, "Engine::forward")) return {};
    if (!hidden_out.empty())
        dev::to_host(hidden_out.data(), lit_->last_hidden.as<void>(), std::min<size_t>(hidden_out.size(), d) * 4,
                     "Engine::forward_with_hidden");
    return out;
}

Engine::MemoryStats Engine::compat_memory_stats() const {
    MemoryStats s;
    if (lit_) lit_->memory_total(&s);
    return s;
}

void Engine::compat_set_max_context(uint32_t tokens) {
    // src/engine.cpp:257-262: the config and the score buffers follow; the KV
    // cache built by load_model keeps its geometry.
    config_.max_seq_len = std::min(tokens, 131072u);
    config_.kv_cache_size = std::min(tokens, 8192u);
    if (!lit_) lit_.reset(new Literal);
    lit_->scores_vec.resize((size_t)config_.kv_cache_size + 4096);
    lit_->scores_out_vec.resize((size_t)config_.kv_cache_size + 4096);
}

}  // namespace forge

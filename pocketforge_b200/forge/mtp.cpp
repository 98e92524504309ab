// mtp.cpp — forge::MTPHeads on the GPU (behaviour of the reference's
// src/mtp.cpp:14-210): weights drawn from rand() and quantized to Q4 with
// per-row scales at construction, every product of forward() on the device.
#include "forge/mtp.hpp"

#include <algorithm>
#include <cmath>
#include <cstdlib>

#include "device.hpp"

namespace forge {

namespace detail {

// Q4 quantization of an MTP matrix (MTPHeads::quantize_q4, src/mtp.cpp:174-197):
// per-row scale amax/127; the even element of each pair is scaled by
// 127/amax/16*7 and the odd one by 127/amax, both rounded and clamped to
// [-8, 7], stored +8 as low / high nibble.
void quantize_q4_rows(const float* src, uint8_t* dst, float* scales, uint32_t rows, uint32_t cols) {
    for (uint32_t r = 0; r < rows; r++) {
        const float* x = src + (size_t)r * cols;
        float amax = 0.0f;
        for (uint32_t c = 0; c < cols; c++) amax = std::max(amax, std::fabs(x[c]));
        const float inv = amax == 0.0f ? 1.0f : 127.0f / amax;
        scales[r] = amax == 0.0f ? 1.0f : amax / 127.0f;
        for (uint32_t c = 0; c < cols; c += 2) {
            int lo = (int8_t)std::round(x[c] * inv / 16.0f * 7.0f);
            lo = std::max(-8, std::min(7, lo));
            uint8_t b = (uint8_t)(lo + 8);
            if (c + 1 < cols) {
                int hi = (int8_t)std::round(x[c + 1] * inv);
                hi = std::max(-8, std::min(7, hi));
                b |= (uint8_t)((hi + 8) << 4);
            }
            dst[(size_t)r * (cols / 2) + c / 2] = b;
        }
    }
}

}  // namespace detail

using detail::quantize_q4_rows;

struct MTPHeads::Impl {
    // Per head, device: gate [ff][d/2], up [ff][d/2], down [d][ff/2] packed + scales.
    struct Head {
        dev::Buffer gate, up, down, gs, us, ds;
    };
    std::vector<Head> heads;
    size_t bytes = 0;
    mutable dev::Buffer cur, g, u, a, o, emb, logits, idx, scratch;
};

MTPHeads::MTPHeads(const MTPConfig& cfg) : impl_(new Impl), cfg_(cfg) {
    impl_->heads.resize(cfg.n_mtp_heads);
    init_weights();
}

MTPHeads::~MTPHeads() = default;

void MTPHeads::init_weights() {
    const uint32_t d = cfg_.n_embd, ff = cfg_.mtp_ff_dim;
    const float init = 1.0f / std::sqrt((float)d);
    impl_->bytes = 0;
    std::vector<float> f;
    std::vector<uint8_t> q;
    std::vector<float> sc;
    // Draw order of the reference: per head gate (ff x d), up (ff x d), down (d x ff).
    auto make = [&](uint32_t rows, uint32_t cols, dev::Buffer& wq, dev::Buffer& ws) {
        f.resize((size_t)rows * cols);
        for (auto& v : f) v = ((float)rand() / (float)RAND_MAX * 2.0f - 1.0f) * init;
        q.assign((size_t)rows * (cols / 2), 0);
        sc.assign(rows, 1.0f);
        quantize_q4_rows(f.data(), q.data(), sc.data(), rows, cols);
        if (wq.reserve(q.size() + 16) && ws.reserve(sc.size() * 4 + 16)) {
            dev::to_dev(wq.as<void>(), q.data(), q.size(), "MTPHeads::init_weights");
            dev::to_dev(ws.as<void>(), sc.data(), sc.size() * 4, "MTPHeads::init_weights");
        }
        impl_->bytes += q.size() + sc.size() * 4;
    };
    for (auto& h : impl_->heads) {
        make(ff, d, h.gate, h.gs);
        make(ff, d, h.up, h.us);
        make(d, ff, h.down, h.ds);
    }
}

std::vector<std::vector<float>> MTPHeads::forward(const float* hidden,
                                                  const std::vector<float>& embedding_table) const {
    const uint32_t d = cfg_.n_embd, ff = cfg_.mtp_ff_dim, V = cfg_.n_vocab, H = cfg_.n_mtp_heads;
    std::vector<std::vector<float>> out(H);
    const bool tied = embedding_table.size() >= (size_t)V * d;
    Impl& m = *impl_;
    float* cur = static_cast<float*>(m.cur.reserve((size_t)d * 4 + 16));
    float* g = static_cast<float*>(m.g.reserve((size_t)ff * 4 + 16));
    float* u = static_cast<float*>(m.u.reserve((size_t)ff * 4 + 16));
    float* a = static_cast<float*>(m.a.reserve((size_t)ff * 4 + 16));
    float* o = static_cast<float*>(m.o.reserve((size_t)d * 4 + 16));
    float* lg = static_cast<float*>(m.logits.reserve((size_t)H * V * 4 + 16));
    float* emb = tied ? static_cast<float*>(m.emb.reserve((size_t)V * d * 4 + 16)) : nullptr;
    if (!cur || !g || !u || !a || !o || !lg || (tied && !emb)) return out;
    if (!dev::to_dev(cur, hidden, (size_t)d * 4, "MTPHeads::forward")) return out;
    if (tied && !dev::to_dev(emb, embedding_table.data(), (size_t)V * d * 4, "MTPHeads::forward")) return out;
    for (uint32_t h = 0; h < H; h++) {
        const Impl::Head& w = m.heads[h];
        bool good = dev::ok(pf_gemv_q4_rows(cur, w.gate.as<uint8_t>(), w.gs.as<float>(), g, ff, d, nullptr), "MTPHeads::forward") &&
                    dev::ok(pf_gemv_q4_rows(cur, w.up.as<uint8_t>(), w.us.as<float>(), u, ff, d, nullptr), "MTPHeads::forward") &&
                    dev::ok(pf_mtp_silu_mul(g, u, a, ff, nullptr), "MTPHeads::forward") &&
                    dev::ok(pf_gemv_q4_rows(a, w.down.as<uint8_t>(), w.ds.as<float>(), o, d, ff, nullptr), "MTPHeads::forward") &&
                    dev::ok(pf_vec_add(cur, o, d, nullptr), "MTPHeads::forward");
        good = good && (tied ? dev::ok(pf_gemv_f32_rows(cur, emb, lg + (size_t)h * V, V, d, nullptr), "MTPHeads::forward")
                             : dev::ok(pf_mtp_placeholder_logits(lg + (size_t)h * V, V, h, nullptr), "MTPHeads::forward"));
        if (!good) return std::vector<std::vector<float>>(H);
    }
    std::vector<float> all((size_t)H * V);
    if (!dev::to_host(all.data(), lg, all.size() * 4, "MTPHeads::forward")) return out;
    for (uint32_t h = 0; h < H; h++) out[h].assign(all.begin() + (size_t)h * V, all.begin() + (size_t)(h + 1) * V);
    return out;
}

int MTPHeads::speculative_accept(int32_t token, const std::vector<std::vector<float>>& mtp_logits) const {
    // src/mtp.cpp:131-143: head 0 counts as accepted; heads 1.. while their
    // argmax equals `token`.
    int accepted = 1;
    const uint32_t n = std::min((uint32_t)mtp_logits.size(), cfg_.n_mtp_heads);
    for (uint32_t h = 1; h < n; h++) {
        if (argmax(mtp_logits[h].data(), cfg_.n_vocab) == token)
            accepted++;
        else
            break;
    }
    return accepted;
}

int32_t MTPHeads::argmax(const float* logits, uint32_t n) {
    static thread_local dev::Buffer v, r;
    float* dv = static_cast<float*>(v.reserve((size_t)n * 4 + 16));
    int32_t* dr = static_cast<int32_t*>(r.reserve(16));
    int32_t best = 0;
    if (!dv || !dr || n == 0 || !dev::to_dev(dv, logits, (size_t)n * 4, "MTPHeads::argmax")) return best;
    if (dev::ok(pf_argmax_rows(dv, 1, (int32_t)n, dr, nullptr), "MTPHeads::argmax"))
        dev::to_host(&best, dr, 4, "MTPHeads::argmax");
    return best;
}

size_t MTPHeads::memory_usage() const { return impl_->bytes; }

}  // namespace forge

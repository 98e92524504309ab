// synth.cpp — synthetic model weights in the reference's own formats (host).
//
// The benchmark model is a random-init Llama-style decoder written the way
// the reference's tools write a .squeeze file and read it back:
//   floats N(0, 0.02) -> Quantizer::quantize_matrix (src/quant_format.cpp:44-157)
//   -> WeightLoader::load_block_with_scales (src/quant_format.cpp:348-425).
// The loader decodes the first n/2 (Q4) or n/4 (Q2) bytes of the block
// stream as packed codes although the stream interleaves one float scale per
// 32 values; the int8 values it returns are what the engine computes with,
// so they are what this generator returns.  Every (layer, matrix) draws from
// its own std::mt19937 so matrices can be generated in parallel.
// MTP heads: uniform(-1, 1)/sqrt(d) floats (MTPHeads::init_weights,
// src/mtp.cpp:31-39) -> MTPHeads::quantize_q4 (src/mtp.cpp:174-197).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

#include "pf_b200.h"

namespace {

uint32_t mseed(uint32_t seed, uint32_t layer, uint32_t matrix) {
    return seed * 2654435761u + layer * 97u + matrix * 7919u + 1u;
}

// Quantizer::quantize_matrix byte stream for one of the four types.
std::vector<uint8_t> squeeze_stream(const std::vector<float>& f, int qtype) {
    const uint64_t n = f.size(), blocks = (n + 31) / 32;
    std::vector<uint8_t> s;
    auto amax_of = [&](uint64_t a, uint64_t b) {
        float m = 0.0f;
        for (uint64_t i = a; i < b; i++) m = std::max(m, std::fabs(f[i]));
        return m;
    };
    switch (qtype) {
        case PF_QT_Q8: {
            s.assign(blocks * 36, 0);
            for (uint64_t bl = 0; bl < blocks; bl++) {
                const uint64_t a = bl * 32, b = std::min(a + 32, n);
                const float m = amax_of(a, b), sc = m == 0.0f ? 0.0f : 127.0f / m;
                uint8_t* p = s.data() + bl * 36;
                std::memcpy(p, &sc, 4);
                for (uint64_t i = a; i < b; i++)
                    p[4 + (i - a)] = (uint8_t)(int8_t)(int32_t)std::round(f[i] * sc + 0.5f);
            }
            break;
        }
        case PF_QT_Q4: {
            s.assign(blocks * 20, 0);
            for (uint64_t bl = 0; bl < blocks; bl++) {
                const uint64_t a = bl * 32, b = std::min(a + 32, n);
                const float m = amax_of(a, b), sc = m == 0.0f ? 0.0f : 7.0f / m;
                uint8_t* p = s.data() + bl * 20;
                std::memcpy(p, &sc, 4);
                for (uint64_t i = a; i < b; i += 2) {
                    int lo = std::clamp((int)(int8_t)std::round(f[i] * sc), -8, 7);
                    uint8_t byte = (uint8_t)(lo + 8);
                    if (i + 1 < b) byte |= (uint8_t)((std::clamp((int)(int8_t)std::round(f[i + 1] * sc), -8, 7) + 8) << 4);
                    p[4 + (i - a) / 2] = byte;
                }
            }
            break;
        }
        case PF_QT_Q2: {
            s.assign(blocks * 12, 0);
            for (uint64_t bl = 0; bl < blocks; bl++) {
                const uint64_t a = bl * 32, b = std::min(a + 32, n);
                const float m = amax_of(a, b), sc = m == 0.0f ? 0.0f : 1.0f / m;
                uint8_t* p = s.data() + bl * 12;
                std::memcpy(p, &sc, 4);
                for (uint64_t i = a; i < b; i += 4) {
                    uint8_t byte = 0;
                    for (uint64_t j = 0; j < 4 && i + j < b; j++)
                        byte |= (uint8_t)((std::clamp((int)(int8_t)std::round(f[i + j] * sc), -2, 1) + 2) << (2 * j));
                    p[4 + (i - a) / 4] = byte;
                }
            }
            break;
        }
        default: {  // Q1.5: codes 0 (-1), 1 (0), 2 (+1) at |v| > 0.35
            s.assign(blocks * 16, 0);
            for (uint64_t bl = 0; bl < blocks; bl++) {
                const uint64_t a = bl * 32, b = std::min(a + 32, n);
                uint8_t* p = s.data() + bl * 16;
                for (uint64_t i = a; i < b; i += 2) {
                    auto code = [](float v) -> uint8_t { return v > 0.35f ? 2 : (v < -0.35f ? 0 : 1); };
                    uint8_t byte = code(f[i]);
                    if (i + 1 < b) byte |= (uint8_t)(code(f[i + 1]) << 2);
                    p[(i - a) / 2] = byte;
                }
            }
            break;
        }
    }
    return s;
}

void loader_view(const std::vector<uint8_t>& s, int rows, int cols, int qtype, int8_t* out, float* rs, float* gs) {
    const uint64_t n = (uint64_t)rows * cols;
    *gs = 1.0f;
    if (qtype == PF_QT_Q8) {
        const uint32_t bpr = ((uint32_t)cols + 31) / 32;
        std::fill(rs, rs + rows, 0.0f);
        for (uint64_t bl = 0; bl < (n + 31) / 32; bl++) {
            float sc;
            std::memcpy(&sc, s.data() + bl * 36, 4);
            rs[bl / bpr] += sc;
            for (uint64_t i = bl * 32; i < std::min(bl * 32 + 32, n); i++) out[i] = (int8_t)s[bl * 36 + 4 + (i - bl * 32)];
        }
        float tot = 0.0f;
        for (int r = 0; r < rows; r++) {
            rs[r] /= (float)bpr;
            tot += rs[r];
        }
        *gs = tot / (float)rows;
        return;
    }
    for (uint64_t i = 0; i < n; i++) {
        if (qtype == PF_QT_Q4) {
            const uint8_t b = s[i / 2];
            out[i] = (int8_t)((int)((i & 1) ? (b >> 4) : (b & 0xF)) - 8);
        } else if (qtype == PF_QT_Q2) {
            out[i] = (int8_t)((int)((s[i / 4] >> (2 * (i & 3))) & 3) - 2);
        } else {
            static const int8_t lut[4] = {-1, 0, 1, 0};
            out[i] = lut[(s[i / 2] >> (2 * (i & 1))) & 3];
        }
    }
    std::fill(rs, rs + rows, 1.0f);
}

void mtp_q4(const std::vector<float>& src, int d, uint8_t* q4, float* scales) {
    for (int r = 0; r < d; r++) {
        const float* row = src.data() + (size_t)r * d;
        float amax = 0.0f;
        for (int c = 0; c < d; c++) amax = std::max(amax, std::fabs(row[c]));
        const float inv = amax == 0.0f ? 1.0f : 127.0f / amax;
        scales[r] = amax == 0.0f ? 1.0f : amax / 127.0f;
        for (int c = 0; c < d; c += 2) {
            // even columns carry an extra 7/16 factor (src/mtp.cpp:186)
            const int v0 = std::clamp((int)(int8_t)std::round(row[c] * inv / 16.0f * 7.0f), -8, 7);
            uint8_t byte = (uint8_t)(v0 + 8);
            if (c + 1 < d) byte |= (uint8_t)((std::clamp((int)(int8_t)std::round(row[c + 1] * inv), -8, 7) + 8) << 4);
            q4[(size_t)r * (d / 2) + c / 2] = byte;
        }
    }
}

}  // namespace

extern "C" {

PF_API pf_status pf_synth_matrix(uint32_t seed, int32_t layer, int32_t matrix, int32_t rows, int32_t cols,
                                 int32_t qtype, int8_t* out, float* row_scales, float* global_scale) {
    if (rows <= 0 || cols <= 0 || !out || !row_scales || !global_scale || qtype < 0 || qtype > 3) return PF_ERR_INVALID;
    std::mt19937 rng(mseed(seed, (uint32_t)layer, (uint32_t)matrix));
    std::normal_distribution<float> nd(0.0f, 0.02f);
    std::vector<float> f((size_t)rows * cols);
    for (auto& v : f) v = nd(rng);
    loader_view(squeeze_stream(f, qtype), rows, cols, qtype, out, row_scales, global_scale);
    return PF_OK;
}

PF_API pf_status pf_synth_mtp_matrix(uint32_t seed, int32_t head, int32_t which, int32_t d, uint8_t* q4,
                                     float* scales) {
    if (d <= 0 || (d & 1) || !q4 || !scales) return PF_ERR_INVALID;
    std::mt19937 rng(mseed(seed, 1000u + (uint32_t)head, 20u + (uint32_t)which));
    std::uniform_real_distribution<float> ud(0.0f, 1.0f);
    const float init = 1.0f / std::sqrt((float)d);
    std::vector<float> f((size_t)d * d);
    for (auto& v : f) v = (ud(rng) * 2.0f - 1.0f) * init;
    mtp_q4(f, d, q4, scales);
    return PF_OK;
}

PF_API pf_status pf_engine_load_synthetic(pf_engine* e, const pf_model_config* c, uint32_t seed, uint32_t mtp_seed,
                                          int32_t threads) {
    if (!e || !c) return PF_ERR_INVALID;
    const int L = c->n_layers, d = c->n_embd, F = c->n_ff, NQ = c->n_heads * c->head_dim,
              NK = c->n_kv_heads * c->head_dim;
    const int rows[7] = {NQ, NK, NK, d, F, F, d};
    const int cols[7] = {d, d, d, NQ, d, d, F};
    threads = std::max(1, std::min(threads, 7));
    for (int l = 0; l < L; l++) {
        std::vector<std::vector<int8_t>> w(7);
        std::vector<std::vector<float>> rs(7);
        std::vector<float> gs(7);
        std::vector<std::thread> pool;
        std::vector<pf_status> st(7, PF_OK);
        for (int m = 0; m < 7; m++) {
            w[m].resize((size_t)rows[m] * cols[m]);
            rs[m].resize(rows[m]);
        }
        auto work = [&](int m) {
            st[m] = pf_synth_matrix(seed, l, m, rows[m], cols[m], c->qtype[m], w[m].data(), rs[m].data(), &gs[m]);
        };
        for (int m = 0; m < 7; m++) {
            if ((int)pool.size() >= threads) {
                for (auto& t : pool) t.join();
                pool.clear();
            }
            pool.emplace_back(work, m);
        }
        for (auto& t : pool) t.join();
        for (int m = 0; m < 7; m++) {
            if (st[m] != PF_OK) return st[m];
            const pf_status s = pf_engine_set_matrix(e, l, m, w[m].data(), rs[m].data());
            if (s != PF_OK) return s;
        }
    }
    {
        std::vector<int8_t> emb((size_t)c->n_vocab * d);
        std::vector<float> rs(c->n_vocab);
        float gs = 1.0f;
        pf_status s = pf_synth_matrix(seed, 0, 10, c->n_vocab, d, c->emb_qtype, emb.data(), rs.data(), &gs);
        if (s != PF_OK) return s;
        s = pf_engine_set_embedding(e, emb.data(), gs);
        if (s != PF_OK) return s;
    }
    for (int h = 0; h < c->n_mtp_heads; h++) {
        std::vector<uint8_t> q[3];
        std::vector<float> sc[3];
        for (int j = 0; j < 3; j++) {
            q[j].resize((size_t)d * d / 2);
            sc[j].resize(d);
            const pf_status s = pf_synth_mtp_matrix(mtp_seed, h, j, d, q[j].data(), sc[j].data());
            if (s != PF_OK) return s;
        }
        const pf_status s =
            pf_engine_set_mtp_head(e, h, q[0].data(), sc[0].data(), q[1].data(), sc[1].data(), q[2].data(), sc[2].data());
        if (s != PF_OK) return s;
    }
    return PF_OK;
}

}  // extern "C"

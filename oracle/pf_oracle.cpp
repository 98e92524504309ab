// pf_oracle.cpp — CPU restatement of PocketForge's MTP speculative-decode step.
//
// TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path in
// pocketforge_b200/ is compared against.  Only tests/, __graft_entry__.smoke()
// and bench.py's cpu_baseline leg (and `bench.py --impl reference`) may load
// it; the product never links, loads or calls it.
//
// Every function restates the reference's arithmetic in source order (file:line
// citations are into tundefund0-gif/pocketforge).  It is compiled with
// -ffp-contract=off so that each a*b+c rounds twice, as the reference's source
// order says; the reference built with the same flag (oracle/_ref) is the pin
// (tests/test_oracle_pins.py checks the two bit for bit).
//
// The "Level-B" step (the intended batched MTP step) composes the reference's
// functions with these deviations (D1-D12 in the design notes):
//   real projection weights, true token positions for RoPE/KV, one K rotation
//   per kv head, per-head attention output slots, greedy verification with a
//   commit of the accepted prefix only, and K+1 verify rows [pending, drafts].
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <random>
#include <thread>
#include <vector>

#include "../include/pf_b200.h"

namespace po {

// ---------------------------------------------------------------------------
// A1: quantize_activation_row (src/matmul_neon.cpp:16-29)
// ---------------------------------------------------------------------------
static void quant_act_row(const float* src, int8_t* dst, float* scale_out, uint32_t n) {
    float amax = 0.0f;
    for (uint32_t i = 0; i < n; i++) {
        float a = std::fabs(src[i]);
        if (a > amax) amax = a;
    }
    const float mul = (amax == 0.0f) ? 1.0f : 127.0f / amax;
    for (uint32_t i = 0; i < n; i++) dst[i] = (int8_t)std::round(src[i] * mul);
    *scale_out = (amax == 0.0f) ? 1.0f : amax / 127.0f;
}

// KVCache::quantize_row (src/kv_cache.cpp:19-28): same values as A1.
static void quant_kv_row(const float* src, int8_t* dst, float* scale_out, uint32_t n) {
    float amax = 0.0f;
    for (uint32_t i = 0; i < n; i++) {
        float a = std::fabs(src[i]);
        if (a > amax) amax = a;
    }
    *scale_out = (amax == 0.0f) ? 1.0f : amax / 127.0f;
    const float mul = (amax == 0.0f) ? 1.0f : 127.0f / amax;
    for (uint32_t i = 0; i < n; i++) dst[i] = (int8_t)std::round(src[i] * mul);
}

// ---------------------------------------------------------------------------
// A2: nibble / crumb decoders (src/matmul_neon.cpp:34-75)
// ---------------------------------------------------------------------------
static void unpack_q4(const uint8_t* src, int8_t* dst, uint64_t n) {
    for (uint64_t i = 0; i < n; i += 2) {
        const uint8_t b = src[i / 2];
        dst[i] = (int8_t)((int)(b & 0x0F) - 8);
        if (i + 1 < n) dst[i + 1] = (int8_t)((int)(b >> 4) - 8);
    }
}
static void unpack_q2(const uint8_t* src, int8_t* dst, uint64_t n) {
    for (uint64_t i = 0; i < n; i += 4) {
        const uint8_t b = src[i / 4];
        for (uint64_t j = 0; j < 4 && i + j < n; j++)
            dst[i + j] = (int8_t)((int)((b >> (2 * j)) & 3) - 2);
    }
}
static void unpack_ternary(const uint8_t* src, int8_t* dst, uint64_t n) {
    static const int8_t lut[4] = {-1, 0, 1, 0};
    for (uint64_t i = 0; i < n; i += 2) {
        const uint8_t b = src[i / 2];
        dst[i] = lut[b & 3];
        if (i + 1 < n) dst[i + 1] = lut[(b >> 2) & 3];
    }
}

// ---------------------------------------------------------------------------
// A3/A4: matmul_int8, matmul_quantized (src/matmul_neon.cpp:80-181)
// ---------------------------------------------------------------------------
// Host threads the output columns of mm_int8 are split over (the engine's
// prefill sets it; every element is computed the same way on any thread).
static thread_local int tl_mm_threads = 1;

static void mm_int8(const int8_t* A, const int8_t* B, int32_t* C, uint32_t M, uint32_t N,
                    uint32_t K) {
    auto cols = [&](uint32_t j0, uint32_t j1) {
        for (uint32_t i = 0; i < M; i++)
            for (uint32_t j = j0; j < j1; j++) {
                const int8_t* a = A + (size_t)i * K;
                const int8_t* b = B + (size_t)j * K;
                int32_t acc = 0;
                for (uint32_t k = 0; k < K; k++) acc += (int32_t)a[k] * (int32_t)b[k];
                C[(size_t)i * N + j] = acc;
            }
    };
    const int nt = tl_mm_threads;
    if (nt <= 1 || (uint64_t)M * N * K < (1u << 20)) {
        cols(0, N);
        return;
    }
    std::vector<std::thread> pool;
    const uint32_t per = (N + nt - 1) / nt;
    for (int t = 0; t < nt; t++) {
        const uint32_t j0 = t * per, j1 = std::min(N, j0 + per);
        if (j0 < j1) pool.emplace_back(cols, j0, j1);
    }
    for (auto& th : pool) th.join();
}

static void mm_quant(const float* A, const int8_t* B, float* C, uint32_t M, uint32_t N, uint32_t K,
                     const float* w_scales, const float* act_scales) {
    std::vector<int8_t> aq((size_t)M * K);
    std::vector<float> as(M);
    for (uint32_t i = 0; i < M; i++) {
        if (act_scales) {
            as[i] = act_scales[i];
            for (uint32_t k = 0; k < K; k++)
                aq[(size_t)i * K + k] = (int8_t)std::round(A[(size_t)i * K + k] / act_scales[i]);
        } else {
            quant_act_row(A + (size_t)i * K, aq.data() + (size_t)i * K, &as[i], K);
        }
    }
    std::vector<int32_t> acc((size_t)M * N);
    mm_int8(aq.data(), B, acc.data(), M, N, K);
    for (uint32_t i = 0; i < M; i++)
        for (uint32_t j = 0; j < N; j++)
            C[(size_t)i * N + j] = (float)acc[(size_t)i * N + j] * as[i] * w_scales[j];
}

// ---------------------------------------------------------------------------
// A5: rmsnorm (src/matmul_neon.cpp:231-239).
// order 0: the reference's sequential sum of squares.
// order 1: the device order — 256 threads, thread t sums elements t, t+256,
//          ... in sequence; each warp of 32 threads combines with an xor
//          butterfly over offsets 16,8,4,2,1 (every lane ends with the same
//          value); the 8 warp totals are added in warp order.
// ---------------------------------------------------------------------------
static float sumsq_lanes(const float* x, uint32_t n) {
    float warp_total[8];
    for (int w = 0; w < 8; w++) {
        float s[32];
        for (int l = 0; l < 32; l++) {
            float a = 0.0f;
            for (uint32_t i = (uint32_t)(w * 32 + l); i < n; i += 256) a += x[i] * x[i];
            s[l] = a;
        }
        for (int off = 16; off >= 1; off >>= 1) {
            float t[32];
            for (int l = 0; l < 32; l++) t[l] = s[l] + s[l ^ off];
            std::memcpy(s, t, sizeof(s));
        }
        warp_total[w] = s[0];
    }
    float tot = warp_total[0];
    for (int w = 1; w < 8; w++) tot += warp_total[w];
    return tot;
}

static float sumsq(const float* x, uint32_t n, int order) {
    if (order == 1) return sumsq_lanes(x, n);
    float ss = 0.0f;
    for (uint32_t i = 0; i < n; i++) ss += x[i] * x[i];
    return ss;
}

static void rmsnorm(float* out, const float* x, const float* w, uint32_t n, float eps, int order) {
    const float ss = sumsq(x, n, order);
    const float rms = std::sqrt(ss / (float)n + eps);
    const float inv = 1.0f / rms;
    for (uint32_t i = 0; i < n; i++) out[i] = x[i] * inv * w[i];
}

// A9: softmax (src/matmul_neon.cpp:212-226)
static void softmax(float* v, uint32_t n) {
    float mx = v[0];
    for (uint32_t i = 1; i < n; i++)
        if (v[i] > mx) mx = v[i];
    float sum = 0.0f;
    for (uint32_t i = 0; i < n; i++) {
        v[i] = std::exp(v[i] - mx);
        sum += v[i];
    }
    const float inv = 1.0f / (sum + 1e-10f);
    for (uint32_t i = 0; i < n; i++) v[i] *= inv;
}

// Engine FFN activation (src/engine.cpp:834-838): g * (1/(1+exp(-g))) * u
static float swiglu_engine(float g, float u) {
    const float sig = 1.0f / (1.0f + std::exp(-g));
    return g * sig * u;
}
// MTPHeads::silu (src/mtp.cpp:157-159): x / (1 + exp(-x))
static float silu_mtp(float x) { return x / (1.0f + std::exp(-x)); }

// A12 greedy: first index of the maximum (src/engine.cpp:918-928)
static int32_t argmax(const float* v, uint32_t n) {
    int32_t best = 0;
    float bv = v[0];
    for (uint32_t i = 1; i < n; i++)
        if (v[i] > bv) {
            bv = v[i];
            best = (int32_t)i;
        }
    return best;
}

// ---------------------------------------------------------------------------
// A12: Engine::sample / sample_top_p / sample_top_k (src/engine.cpp:881-1003)
// with the uniform draw passed in (the reference draws it from a file-static
// std::mt19937 at the point marked; draw order is the caller's business).
// ---------------------------------------------------------------------------
static int32_t sample_top_p(const float* logits, uint32_t n, float p, float temp, float u) {
    std::vector<std::pair<float, int32_t>> sc;
    sc.reserve(n);
    for (uint32_t i = 0; i < n; i++) sc.emplace_back(logits[i], (int32_t)i);
    std::sort(sc.begin(), sc.end(), [](const std::pair<float, int32_t>& a,
                                       const std::pair<float, int32_t>& b) {
        return a.first > b.first;
    });
    const float mx = sc[0].first;
    const float t = std::max(temp, 0.001f);
    std::vector<float> pr(n);
    float total = 0.0f;
    for (uint32_t i = 0; i < n; i++) {
        pr[i] = std::exp((sc[i].first - mx) / t);
        total += pr[i];
    }
    for (uint32_t i = 0; i < n; i++) pr[i] /= total;
    float cum = 0.0f;
    uint32_t cut = n;
    for (uint32_t i = 0; i < n; i++) {
        cum += pr[i];
        if (cum >= p) {
            cut = i + 1;
            break;
        }
    }
    cum = 0.0f;  // draw happens here in the reference (src/engine.cpp:996)
    for (uint32_t i = 0; i < cut; i++) {
        cum += pr[i];
        if (u <= cum) return sc[i].second;
    }
    return sc[cut - 1].second;
}

static int32_t sample_top_k(const float* logits, uint32_t n, uint32_t k, float temp, float u) {
    std::vector<std::pair<float, int32_t>> sc;
    sc.reserve(n);
    for (uint32_t i = 0; i < n; i++) sc.emplace_back(logits[i], (int32_t)i);
    const uint32_t kk = std::min(k, n);
    std::partial_sort(sc.begin(), sc.begin() + kk, sc.end(),
                      [](const std::pair<float, int32_t>& a, const std::pair<float, int32_t>& b) {
                          return a.first > b.first;
                      });
    const float mx = sc[0].first;
    std::vector<float> pr(kk);
    float total = 0.0f;
    for (uint32_t i = 0; i < kk; i++) {
        pr[i] = std::exp((sc[i].first - mx) / std::max(temp, 0.001f));
        total += pr[i];
    }
    float cum = 0.0f;
    for (uint32_t i = 0; i < kk; i++) {
        cum += pr[i] / total;
        if (u <= cum) return sc[i].second;
    }
    return sc[kk - 1].second;
}

static int32_t sample_temperature(const float* logits, uint32_t n, float temperature, float u) {
    std::vector<float> e(n);
    const float t = std::max(temperature, 0.001f);
    float mx = logits[0];
    for (uint32_t i = 1; i < n; i++)
        if (logits[i] > mx) mx = logits[i];
    float total = 0.0f;
    for (uint32_t i = 0; i < n; i++) {
        e[i] = std::exp((logits[i] - mx) / t);
        total += e[i];
    }
    float cum = 0.0f;
    for (uint32_t i = 0; i < n; i++) {
        cum += e[i] / total;
        if (u <= cum) return (int32_t)i;
    }
    return (int32_t)(n - 1);
}

static bool sampling_is_greedy(const pf_sampling_config& c) {
    return c.greedy || c.temperature <= 0.0f;
}

static int32_t sample(const float* logits, uint32_t n, const pf_sampling_config& c, float u) {
    if (sampling_is_greedy(c)) return argmax(logits, n);
    if (c.top_p < 1.0f && c.top_p > 0.0f) return sample_top_p(logits, n, c.top_p, c.temperature, u);
    if (c.top_k > 0 && c.top_k < n) return sample_top_k(logits, n, c.top_k, c.temperature, u);
    return sample_temperature(logits, n, c.temperature, u);
}

// ---------------------------------------------------------------------------
// Quantizer::quantize_matrix (src/quant_format.cpp:44-157) and the loader's
// view of its output, WeightLoader::load_block_with_scales
// (src/quant_format.cpp:348-425).  The loader decodes the FIRST n/2 (Q4) or
// n/4 (Q2) bytes of the block stream as packed codes even though the stream
// interleaves a float scale per 32 values; this restatement keeps that.
// ---------------------------------------------------------------------------
static std::vector<uint8_t> quantize_matrix(const float* data, uint32_t rows, uint32_t cols,
                                            int qtype) {
    const uint64_t n = (uint64_t)rows * cols;
    const uint64_t nb = (n + 31) / 32;
    std::vector<uint8_t> out;
    auto block_amax = [&](uint64_t s, uint64_t e) {
        float a = 0.0f;
        for (uint64_t i = s; i < e; i++) a = std::max(a, std::fabs(data[i]));
        return a;
    };
    if (qtype == PF_QT_Q8) {
        out.assign(nb * 36, 0);
        uint8_t* p = out.data();
        for (uint64_t b = 0; b < nb; b++) {
            const uint64_t s = b * 32, e = std::min(s + 32, n);
            const float a = block_amax(s, e);
            const float sc = (a == 0.0f) ? 0.0f : 127.0f / a;
            std::memcpy(p, &sc, 4);
            p += 4;
            for (uint64_t i = s; i < e; i++) *p++ = (uint8_t)(int8_t)(int32_t)std::round(data[i] * sc + 0.5f);
            p += (s + 32 - e);
        }
    } else if (qtype == PF_QT_Q4) {
        out.assign(nb * 20, 0);
        uint8_t* p = out.data();
        for (uint64_t b = 0; b < nb; b++) {
            const uint64_t s = b * 32, e = std::min(s + 32, n);
            const float a = block_amax(s, e);
            const float sc = (a == 0.0f) ? 0.0f : 7.0f / a;
            std::memcpy(p, &sc, 4);
            uint8_t* q = p + 4;
            for (uint64_t i = s; i < e; i += 2) {
                int v0 = (int8_t)std::round(data[i] * sc);
                v0 = std::max(-8, std::min(7, v0));
                uint8_t byte = (uint8_t)(v0 + 8);
                if (i + 1 < e) {
                    int v1 = (int8_t)std::round(data[i + 1] * sc);
                    v1 = std::max(-8, std::min(7, v1));
                    byte |= (uint8_t)((v1 + 8) << 4);
                }
                *q++ = byte;
            }
            p += 20;
        }
    } else if (qtype == PF_QT_Q2) {
        out.assign(nb * 12, 0);
        uint8_t* p = out.data();
        for (uint64_t b = 0; b < nb; b++) {
            const uint64_t s = b * 32, e = std::min(s + 32, n);
            const float a = block_amax(s, e);
            const float sc = (a == 0.0f) ? 0.0f : 1.0f / a;
            std::memcpy(p, &sc, 4);
            uint8_t* q = p + 4;
            for (uint64_t i = s; i < e; i += 4) {
                uint8_t byte = 0;
                for (uint64_t j = 0; j < 4 && i + j < e; j++) {
                    int v = (int8_t)std::round(data[i + j] * sc);
                    v = std::max(-2, std::min(1, v));
                    byte |= (uint8_t)((v + 2) << (2 * j));
                }
                *q++ = byte;
            }
            p += 12;
        }
    } else {  // Q1.5 ternary
        out.assign(nb * 16, 0);
        uint8_t* p = out.data();
        for (uint64_t b = 0; b < nb; b++) {
            const uint64_t s = b * 32, e = std::min(s + 32, n);
            for (uint64_t i = s; i < e; i += 2) {
                const float v0 = data[i];
                uint8_t byte = (v0 > 0.35f) ? 2 : ((v0 < -0.35f) ? 0 : 1);
                if (i + 1 < e) {
                    const float v1 = data[i + 1];
                    const uint8_t c1 = (v1 > 0.35f) ? 2 : ((v1 < -0.35f) ? 0 : 1);
                    byte |= (uint8_t)(c1 << 2);
                }
                *p++ = byte;
            }
        }
    }
    return out;
}

static void loader_decode(const std::vector<uint8_t>& blk, uint32_t rows, uint32_t cols, int qtype,
                          int8_t* out, float* row_scales, float* global_scale) {
    const uint64_t n = (uint64_t)rows * cols;
    *global_scale = 1.0f;
    if (qtype == PF_QT_Q8) {
        const uint64_t nb = (n + 31) / 32;
        const uint32_t bpr = (cols + 31) / 32;
        for (uint32_t r = 0; r < rows; r++) row_scales[r] = 0.0f;
        const uint8_t* p = blk.data();
        for (uint64_t b = 0; b < nb; b++) {
            float s;
            std::memcpy(&s, p, 4);
            p += 4;
            row_scales[b / bpr] += s;
            const uint64_t st = b * 32, e = std::min(st + 32, n);
            for (uint64_t i = st; i < e; i++) out[i] = (int8_t)(*p++);
            p += (st + 32 - e);
        }
        float tot = 0.0f;
        for (uint32_t r = 0; r < rows; r++) {
            row_scales[r] /= (float)bpr;
            tot += row_scales[r];
        }
        *global_scale = tot / (float)rows;
        return;
    }
    if (qtype == PF_QT_Q4) unpack_q4(blk.data(), out, n);
    else if (qtype == PF_QT_Q2) unpack_q2(blk.data(), out, n);
    else unpack_ternary(blk.data(), out, n);
    for (uint32_t r = 0; r < rows; r++) row_scales[r] = 1.0f;
}

// Seed of one synthetic matrix: one std::mt19937 per (layer, matrix).
static uint32_t matrix_seed(uint32_t seed, uint32_t layer, uint32_t matrix) {
    return seed * 2654435761u + layer * 97u + matrix * 7919u + 1u;
}

// Synthetic transformer matrix: N(0, 0.02) floats -> Quantizer -> loader.
static void synth_matrix(uint32_t seed, uint32_t layer, uint32_t matrix, uint32_t rows,
                         uint32_t cols, int qtype, int8_t* out, float* row_scales,
                         float* global_scale) {
    std::mt19937 rng(matrix_seed(seed, layer, matrix));
    std::normal_distribution<float> nd(0.0f, 0.02f);
    std::vector<float> f((size_t)rows * cols);
    for (auto& v : f) v = nd(rng);
    auto blk = quantize_matrix(f.data(), rows, cols, qtype);
    loader_decode(blk, rows, cols, qtype, out, row_scales, global_scale);
}

// ---------------------------------------------------------------------------
// A13: MTPHeads (src/mtp.cpp:14-129, 174-209)
// ---------------------------------------------------------------------------
static void mtp_quantize_q4(const float* src, uint8_t* dst, float* scales, uint32_t rows,
                            uint32_t cols) {
    for (uint32_t r = 0; r < rows; r++) {
        float amax = 0.0f;
        for (uint32_t c = 0; c < cols; c++) amax = std::max(amax, std::fabs(src[(size_t)r * cols + c]));
        const float inv = (amax == 0.0f) ? 1.0f : 127.0f / amax;
        scales[r] = (amax == 0.0f) ? 1.0f : amax / 127.0f;
        for (uint32_t c = 0; c < cols; c += 2) {
            int v0 = (int8_t)std::round(src[(size_t)r * cols + c] * inv / 16.0f * 7.0f);
            v0 = std::max(-8, std::min(7, v0));
            uint8_t byte = (uint8_t)(v0 + 8);
            if (c + 1 < cols) {
                int v1 = (int8_t)std::round(src[(size_t)r * cols + c + 1] * inv);
                v1 = std::max(-8, std::min(7, v1));
                byte |= (uint8_t)((v1 + 8) << 4);
            }
            dst[(size_t)r * (cols / 2) + c / 2] = byte;
        }
    }
}

// Synthetic MTP matrix j (0 gate, 1 up, 2 down) of head h: uniform(-1,1)/sqrt(d)
// floats (the distribution of MTPHeads::init_weights, src/mtp.cpp:31-39)
// from a seeded std::mt19937, then quantize_q4.
static void synth_mtp_matrix(uint32_t seed, uint32_t head, uint32_t j, uint32_t d, uint8_t* q4,
                             float* scales) {
    std::mt19937 rng(matrix_seed(seed, 1000u + head, 20u + j));
    std::uniform_real_distribution<float> ud(0.0f, 1.0f);
    const float init = 1.0f / std::sqrt((float)d);
    std::vector<float> f((size_t)d * d);
    for (auto& v : f) v = (ud(rng) * 2.0f - 1.0f) * init;
    mtp_quantize_q4(f.data(), q4, scales, d, d);
}

static void dequant_q4_row_scaled(const uint8_t* src, float* dst, float scale, uint32_t n) {
    for (uint32_t i = 0; i < n; i += 2) {
        const uint8_t b = src[i / 2];
        dst[i] = (float)((int)(b & 0x0F) - 8) * scale;
        if (i + 1 < n) dst[i + 1] = (float)((int)(b >> 4) - 8) * scale;
    }
}

struct MtpHead {
    std::vector<uint8_t> gate, up, down;
    std::vector<float> gs, us, ds;
};

// MTPHeads::forward (src/mtp.cpp:47-129) with the tied fp32 embedding table.
static void mtp_forward(const std::vector<MtpHead>& heads, uint32_t d, const float* hidden,
                        const float* emb, uint32_t vocab, float* logits /* [H][vocab] */,
                        float* final_hidden /* may be null */) {
    std::vector<float> cur(hidden, hidden + d), deq(d), g(d), u(d), a(d), o(d);
    for (size_t h = 0; h < heads.size(); h++) {
        const MtpHead& w = heads[h];
        for (uint32_t j = 0; j < d; j++) {
            dequant_q4_row_scaled(w.gate.data() + (size_t)j * (d / 2), deq.data(), w.gs[j], d);
            float s = 0.0f;
            for (uint32_t i = 0; i < d; i++) s += cur[i] * deq[i];
            g[j] = s;
        }
        for (uint32_t j = 0; j < d; j++) {
            dequant_q4_row_scaled(w.up.data() + (size_t)j * (d / 2), deq.data(), w.us[j], d);
            float s = 0.0f;
            for (uint32_t i = 0; i < d; i++) s += cur[i] * deq[i];
            u[j] = s;
        }
        for (uint32_t j = 0; j < d; j++) a[j] = silu_mtp(g[j]) * u[j];
        for (uint32_t i = 0; i < d; i++) {
            dequant_q4_row_scaled(w.down.data() + (size_t)i * (d / 2), deq.data(), w.ds[i], d);
            float s = 0.0f;
            for (uint32_t j = 0; j < d; j++) s += a[j] * deq[j];
            o[i] = s;
        }
        for (uint32_t i = 0; i < d; i++) cur[i] += o[i];
        float* lg = logits + h * (size_t)vocab;
        for (uint32_t v = 0; v < vocab; v++) {
            const float* e = emb + (size_t)v * d;
            float s = 0.0f;
            for (uint32_t i = 0; i < d; i++) s += cur[i] * e[i];
            lg[v] = s;
        }
    }
    if (final_hidden) std::memcpy(final_hidden, cur.data(), d * sizeof(float));
}

// ---------------------------------------------------------------------------
// A7/A8: the 3-tier int8 KV cache of one (layer, kv head)
// (src/kv_cache.cpp:32-198): sink slots, a circular window, and a pool of
// 64-entry means accumulated in double from evicted window entries.
// ---------------------------------------------------------------------------
struct TierHead {
    uint32_t hd = 0, ring = 0, sink_cap = 8;
    std::vector<int8_t> sk, sv;
    std::vector<float> sks, svs;
    uint32_t n_sink = 0;
    std::vector<int8_t> wk, wv;
    std::vector<float> wks, wvs;
    std::vector<uint32_t> wpos;
    uint32_t head = 0, n_win = 0;
    std::vector<int8_t> pk, pv;
    std::vector<float> pks, pvs;
    uint32_t n_pool = 0;
    std::vector<double> ak, av;
    uint32_t n_acc = 0, acc_first = 0;

    void init(uint32_t hd_, uint32_t ring_) {
        hd = hd_;
        ring = ring_;
        sk.assign(sink_cap * hd, 0);
        sv.assign(sink_cap * hd, 0);
        sks.assign(sink_cap, 1.0f);
        svs.assign(sink_cap, 1.0f);
        wk.assign((size_t)ring * hd, 0);
        wv.assign((size_t)ring * hd, 0);
        wks.assign(ring, 1.0f);
        wvs.assign(ring, 1.0f);
        wpos.assign(ring, 0);
        ak.assign(hd, 0.0);
        av.assign(hd, 0.0);
    }
    uint32_t slot_of(uint32_t i) const { return (n_win < ring) ? i : (head + i) % ring; }
};

struct TierCache {
    uint32_t n_layers = 0, n_kv = 0, hd = 0, sink = 4, window = 0, pool_block = 64,
             max_ctx = 0;
    std::vector<TierHead> heads;  // [layer][kv]
    uint32_t stored = 0;

    void init(uint32_t L, uint32_t H, uint32_t hd_, uint32_t sink_, uint32_t window_,
              uint32_t pool_, uint32_t max_ctx_) {
        n_layers = L;
        n_kv = H;
        hd = hd_;
        sink = sink_;
        window = std::min(window_, max_ctx_);
        pool_block = std::max(1u, pool_);
        max_ctx = max_ctx_;
        heads.resize((size_t)L * H);
        for (auto& t : heads) t.init(hd, window);
    }
    TierHead& at(uint32_t l, uint32_t h) { return heads[(size_t)l * n_kv + h]; }

    void store(uint32_t l, uint32_t h, uint32_t pos, const float* key, const float* val) {
        if (l >= n_layers || h >= n_kv || pos >= max_ctx) return;
        TierHead& c = at(l, h);
        if (pos < sink) {
            if (pos < c.sink_cap) {
                quant_kv_row(key, c.sk.data() + pos * hd, &c.sks[pos], hd);
                quant_kv_row(val, c.sv.data() + pos * hd, &c.svs[pos], hd);
                if (pos >= c.n_sink) c.n_sink = pos + 1;
            }
        } else {
            const uint32_t slot = c.head;
            if (c.n_win >= c.ring) {
                const uint32_t gone = c.wpos[slot];
                if (c.n_acc == 0) c.acc_first = gone;
                for (uint32_t i = 0; i < hd; i++) {
                    c.ak[i] += (double)c.wk[(size_t)slot * hd + i] * c.wks[slot];
                    c.av[i] += (double)c.wv[(size_t)slot * hd + i] * c.wvs[slot];
                }
                c.n_acc++;
                if (c.n_acc >= pool_block) {
                    const float inv = 1.0f / c.n_acc;
                    const uint32_t p = c.n_pool++;
                    c.pk.resize((size_t)(p + 1) * hd);
                    c.pv.resize((size_t)(p + 1) * hd);
                    c.pks.push_back(1.0f);
                    c.pvs.push_back(1.0f);
                    std::vector<float> mean(hd);
                    for (uint32_t i = 0; i < hd; i++) mean[i] = (float)(c.ak[i] * inv);
                    quant_kv_row(mean.data(), c.pk.data() + (size_t)p * hd, &c.pks[p], hd);
                    for (uint32_t i = 0; i < hd; i++) mean[i] = (float)(c.av[i] * inv);
                    quant_kv_row(mean.data(), c.pv.data() + (size_t)p * hd, &c.pvs[p], hd);
                    std::fill(c.ak.begin(), c.ak.end(), 0.0);
                    std::fill(c.av.begin(), c.av.end(), 0.0);
                    c.n_acc = 0;
                }
            } else {
                c.n_win++;
            }
            quant_kv_row(key, c.wk.data() + (size_t)slot * hd, &c.wks[slot], hd);
            quant_kv_row(val, c.wv.data() + (size_t)slot * hd, &c.wvs[slot], hd);
            c.wpos[slot] = pos;
            c.head = (c.head + 1) % c.ring;
        }
        if (pos >= stored) stored = pos + 1;
    }

    // Entries in attention order (sink, pool, window oldest-first).
    uint32_t count(uint32_t l, uint32_t h) {
        TierHead& c = at(l, h);
        return c.n_sink + c.n_pool + c.n_win;
    }
    void entry(uint32_t l, uint32_t h, uint32_t idx, const int8_t** k, float* ks,
               const int8_t** v, float* vs) {
        TierHead& c = at(l, h);
        if (idx < c.n_sink) {
            *k = c.sk.data() + (size_t)idx * hd;
            *v = c.sv.data() + (size_t)idx * hd;
            *ks = c.sks[idx];
            *vs = c.svs[idx];
            return;
        }
        idx -= c.n_sink;
        if (idx < c.n_pool) {
            *k = c.pk.data() + (size_t)idx * hd;
            *v = c.pv.data() + (size_t)idx * hd;
            *ks = c.pks[idx];
            *vs = c.pvs[idx];
            return;
        }
        idx -= c.n_pool;
        const uint32_t s = c.slot_of(idx);
        *k = c.wk.data() + (size_t)s * hd;
        *v = c.wv.data() + (size_t)s * hd;
        *ks = c.wks[s];
        *vs = c.wvs[s];
    }

    // KVCache::attention_scores (src/kv_cache.cpp:129-158)
    uint32_t scores(uint32_t l, uint32_t h, const float* q, float* out) {
        if (l >= n_layers || h >= n_kv) return 0;
        const uint32_t n = count(l, h);
        for (uint32_t e = 0; e < n; e++) {
            const int8_t *k, *v;
            float ks, vs;
            entry(l, h, e, &k, &ks, &v, &vs);
            float s = 0.0f;
            for (uint32_t i = 0; i < hd; i++) s += q[i] * ((float)k[i] * ks);
            out[e] = s;
        }
        return n;
    }
    // KVCache::attention_weighted_sum (src/kv_cache.cpp:160-198)
    void weighted_sum(uint32_t l, uint32_t h, const float* p, float* out, uint32_t cnt) {
        for (uint32_t i = 0; i < hd; i++) out[i] = 0.0f;
        if (l >= n_layers || h >= n_kv || cnt == 0) return;
        const uint32_t n = std::min(count(l, h), cnt);
        for (uint32_t e = 0; e < n; e++) {
            const int8_t *k, *v;
            float ks, vs;
            entry(l, h, e, &k, &ks, &v, &vs);
            const float s = p[e];
            for (uint32_t i = 0; i < hd; i++) out[i] += s * ((float)v[i] * vs);
        }
    }
};

// ---------------------------------------------------------------------------
// A10: LayerSkipController::should_skip_ffn (src/layer_skip.cpp:22-67); the
// anchor never fires because the engine never calls new_token().
// ---------------------------------------------------------------------------
struct SkipState {
    uint32_t L = 0, d = 0;
    float thr = 0.01f;
    std::vector<float> cache;  // [L][d] post-ffn-norm vector of the last computed FFN
    void init(uint32_t L_, uint32_t d_, float t) {
        L = L_;
        d = d_;
        thr = t;
        cache.assign((size_t)L * d, 0.0f);
    }
    static float delta(const float* a, const float* b, uint32_t n, int order) {
        float s = 0.0f;
        if (order == 1) {
            float part[32];
            for (int l = 0; l < 32; l++) {
                float acc = 0.0f;
                for (uint32_t i = (uint32_t)l; i < n; i += 32) {
                    const float df = a[i] - b[i];
                    acc += df * df;
                }
                part[l] = acc;
            }
            for (int off = 16; off >= 1; off >>= 1) {
                float t[32];
                for (int l = 0; l < 32; l++) t[l] = part[l] + part[l ^ off];
                std::memcpy(part, t, sizeof(part));
            }
            s = part[0];
        } else {
            for (uint32_t i = 0; i < n; i++) {
                const float df = a[i] - b[i];
                s += df * df;
            }
        }
        return std::sqrt(s / (float)n);
    }
    float layer_threshold(uint32_t layer) const {
        const uint32_t mid = L / 2;
        float t = thr;
        if (layer > mid / 2 && layer < mid + mid / 2) t *= 2.0f;
        if (layer < 2 || layer >= L - 2) t = -1.0f;
        return t;
    }
    // margin (optional): |delta - threshold| / threshold of this decision, a
    // test diagnostic (a decision within float rounding of its threshold can
    // go either way in another summation order).
    bool should_skip(uint32_t layer, const float* x, int order, float* margin = nullptr) {
        if (layer >= L) return false;
        float* c = cache.data() + (size_t)layer * d;
        const float dl = delta(x, c, d, order);
        const float lt = layer_threshold(layer);
        if (margin) *margin = lt > 0.0f ? std::fabs(dl - lt) / lt : INFINITY;
        const bool skip = dl < lt;
        if (!skip) std::memcpy(c, x, d * sizeof(float));
        return skip;
    }
};

// RoPE table, computed with the float library calls of src/engine.cpp:660-668.
static void rope_row(float theta, uint32_t hd, uint32_t pos, float* cs, float* sn) {
    for (uint32_t i = 0; i < hd; i += 2) {
        const float freq = 1.0f / std::pow(theta, (float)i / (float)hd);
        cs[i / 2] = std::cos((float)pos * freq);
        sn[i / 2] = std::sin((float)pos * freq);
    }
}

// ---------------------------------------------------------------------------
// Level-B engine
// ---------------------------------------------------------------------------
struct Seq {
    TierCache kv;
    SkipState skip;
    uint32_t pos = 0;  // committed length
    int32_t pending = 0;
    std::vector<float> hidden;  // MTP input: hidden of the row that produced `pending`
    std::vector<int32_t> drafts;
    std::mt19937 rng;
    std::vector<float> mtp_logits;  // [K][V] of the last MTP call
    // Committed FFN decisions of this sequence, and the smallest layer-skip
    // decision margin seen (a test diagnostic).  Kept per sequence so that
    // sequences can run on separate host threads; the engine sums them.
    int64_t ffn_computed = 0, ffn_skipped = 0;
    float skip_margin = INFINITY;
};

// Runs f(0..n-1) on up to `threads` host threads.  Each index is one
// sequence: sequences share no mutable state, so the results are the same
// as running them one after another.
template <class F>
static void for_each_seq(int n, int threads, F f) {
    if (threads <= 1 || n <= 1) {
        for (int i = 0; i < n; i++) f(i);
        return;
    }
    std::atomic<int> next{0};
    std::vector<std::thread> pool;
    for (int t = 0; t < std::min(threads, n); t++)
        pool.emplace_back([&]() {
            for (int i; (i = next++) < n;) f(i);
        });
    for (auto& th : pool) th.join();
}

struct Engine {
    pf_model_config cfg{};
    int order = 0;
    pf_sampling_config samp{0.8f, 0.95f, 40, 1};
    std::vector<std::vector<int8_t>> w[PF_MAT_COUNT];
    std::vector<std::vector<float>> rs[PF_MAT_COUNT];
    std::vector<float> attn_norm, ffn_norm, final_norm, emb;
    std::vector<MtpHead> mtp;
    std::vector<Seq> seqs;
    std::vector<float> last_logits;  // [n_seqs*(K+1)][V]
    int threads = 1;                 // host threads over sequences (prefill, step)
    int prefill_threads = 1;         // > 1: prefill one sequence at a time, its matmuls on this many threads

    int64_t ffn_computed() const {
        int64_t n = 0;
        for (const Seq& s : seqs) n += s.ffn_computed;
        return n;
    }
    int64_t ffn_skipped() const {
        int64_t n = 0;
        for (const Seq& s : seqs) n += s.ffn_skipped;
        return n;
    }
    float skip_margin() const {  // smallest decision margin seen (test diagnostic)
        float m = INFINITY;
        for (const Seq& s : seqs) m = std::min(m, s.skip_margin);
        return m;
    }

    uint32_t d() const { return (uint32_t)cfg.n_embd; }
    uint32_t K() const { return (uint32_t)cfg.n_mtp_heads; }
    uint32_t V() const { return (uint32_t)cfg.n_vocab; }

    void init(const pf_model_config& c) {
        cfg = c;
        const uint32_t L = (uint32_t)c.n_layers;
        for (int m = 0; m < PF_MAT_COUNT; m++) {
            w[m].assign(L, {});
            rs[m].assign(L, {});
        }
        attn_norm.assign((size_t)L * c.n_embd, 1.0f);
        ffn_norm.assign((size_t)L * c.n_embd, 1.0f);
        final_norm.assign(c.n_embd, 1.0f);
        mtp.assign(c.n_mtp_heads, {});
    }

    void mat_shape(int m, uint32_t* rows, uint32_t* cols) const {
        const uint32_t q = (uint32_t)(cfg.n_heads * cfg.head_dim);
        const uint32_t kv = (uint32_t)(cfg.n_kv_heads * cfg.head_dim);
        switch (m) {
            case PF_MAT_Q: *rows = q; *cols = d(); break;
            case PF_MAT_K:
            case PF_MAT_V: *rows = kv; *cols = d(); break;
            case PF_MAT_O: *rows = d(); *cols = q; break;
            case PF_MAT_GATE:
            case PF_MAT_UP: *rows = (uint32_t)cfg.n_ff; *cols = d(); break;
            default: *rows = d(); *cols = (uint32_t)cfg.n_ff; break;
        }
    }

    void new_seq(Seq& s, uint32_t seed) {
        s.kv.init(cfg.n_layers, cfg.n_kv_heads, cfg.head_dim, cfg.sink_size, cfg.window_size,
                  cfg.pool_block, cfg.max_context);
        s.skip.init(cfg.n_layers, d(), cfg.skip_threshold);
        s.pos = 0;
        s.pending = 0;
        s.hidden.assign(d(), 0.0f);
        s.drafts.assign(K(), 0);
        s.rng.seed(seed);
        s.mtp_logits.assign((size_t)K() * V(), 0.0f);
    }

    float draw(Seq& s) {
        return std::uniform_real_distribution<float>(0.0f, 1.0f)(s.rng);
    }

    // One token through the whole model at position `pos` (Engine::forward_with_hidden,
    // src/engine.cpp:459-589, with D1-D6), storing its K/V and skip-cache state.
    void forward_row(Seq& s, int32_t token, uint32_t pos, float* logits, float* hid_out) {
        const uint32_t D = d(), H = (uint32_t)cfg.n_heads, G = (uint32_t)cfg.n_kv_heads,
                       hd = (uint32_t)cfg.head_dim, F = (uint32_t)cfg.n_ff;
        std::vector<float> x(D, 0.0f), nrm(D), q(H * hd), k(G * hd), v(G * hd), att(H * hd),
            o(D), g(F), u(F), act(F), dn(D), cs(hd / 2), sn(hd / 2);
        std::vector<float> sc;
        if (token >= 0 && (uint32_t)token < V())
            std::memcpy(x.data(), emb.data() + (size_t)token * D, D * sizeof(float));
        rope_row(cfg.rope_theta, hd, pos, cs.data(), sn.data());
        for (uint32_t l = 0; l < (uint32_t)cfg.n_layers; l++) {
            rmsnorm(nrm.data(), x.data(), attn_norm.data() + (size_t)l * D, D, cfg.norm_eps, order);
            mm_quant(nrm.data(), w[PF_MAT_Q][l].data(), q.data(), 1, H * hd, D, rs[PF_MAT_Q][l].data(), nullptr);
            mm_quant(nrm.data(), w[PF_MAT_K][l].data(), k.data(), 1, G * hd, D, rs[PF_MAT_K][l].data(), nullptr);
            mm_quant(nrm.data(), w[PF_MAT_V][l].data(), v.data(), 1, G * hd, D, rs[PF_MAT_V][l].data(), nullptr);
            // RoPE on every q head and once on every kv head (D3).
            auto rot = [&](float* h) {
                for (uint32_t i = 0; i < hd; i += 2) {
                    const float a = h[i], b = h[i + 1], c = cs[i / 2], si = sn[i / 2];
                    h[i] = a * c - b * si;
                    h[i + 1] = a * si + b * c;
                }
            };
            for (uint32_t h = 0; h < H; h++) rot(q.data() + h * hd);
            for (uint32_t h = 0; h < G; h++) rot(k.data() + h * hd);
            const float scale = 1.0f / std::sqrt((float)hd);
            for (uint32_t h = 0; h < H; h++) {
                const uint32_t kvh = h % G;
                const float* qh = q.data() + h * hd;
                const float* kh = k.data() + kvh * hd;
                const float* vh = v.data() + kvh * hd;
                const uint32_t n = s.kv.count(l, kvh);
                sc.resize(n + 1);
                s.kv.scores(l, kvh, qh, sc.data());
                float self = 0.0f;
                for (uint32_t i = 0; i < hd; i++) self += qh[i] * kh[i];
                sc[n] = self;
                for (uint32_t i = 0; i <= n; i++) sc[i] *= scale;
                softmax(sc.data(), n + 1);
                float* out = att.data() + h * hd;  // D4: own slot
                s.kv.weighted_sum(l, kvh, sc.data(), out, n);
                const float ps = sc[n];
                for (uint32_t i = 0; i < hd; i++) out[i] += ps * vh[i];
            }
            for (uint32_t h = 0; h < G; h++) s.kv.store(l, h, pos, k.data() + h * hd, v.data() + h * hd);
            mm_quant(att.data(), w[PF_MAT_O][l].data(), o.data(), 1, D, H * hd, rs[PF_MAT_O][l].data(), nullptr);
            for (uint32_t i = 0; i < D; i++) x[i] += o[i];
            rmsnorm(nrm.data(), x.data(), ffn_norm.data() + (size_t)l * D, D, cfg.norm_eps, order);
            float mg = INFINITY;
            const bool skip = cfg.skip_enabled ? s.skip.should_skip(l, nrm.data(), order, &mg) : false;
            s.skip_margin = std::min(s.skip_margin, mg);
            if (skip) {
                s.ffn_skipped++;
                continue;
            }
            s.ffn_computed++;
            mm_quant(nrm.data(), w[PF_MAT_GATE][l].data(), g.data(), 1, F, D, rs[PF_MAT_GATE][l].data(), nullptr);
            mm_quant(nrm.data(), w[PF_MAT_UP][l].data(), u.data(), 1, F, D, rs[PF_MAT_UP][l].data(), nullptr);
            for (uint32_t j = 0; j < F; j++) act[j] = swiglu_engine(g[j], u[j]);
            mm_quant(act.data(), w[PF_MAT_DOWN][l].data(), dn.data(), 1, D, F, rs[PF_MAT_DOWN][l].data(), nullptr);
            for (uint32_t i = 0; i < D; i++) x[i] += dn[i];
        }
        if (hid_out) std::memcpy(hid_out, x.data(), D * sizeof(float));
        // Unembed with the pre-final-norm hidden (D6, src/engine.cpp:571-583).
        if (logits) {
            for (uint32_t t = 0; t < V(); t++) {
                const float* e = emb.data() + (size_t)t * D;
                float acc = 0.0f;
                for (uint32_t i = 0; i < D; i++) acc += x[i] * e[i];
                logits[t] = acc;
            }
        }
    }

    // MTP drafts from s.hidden (drafts sampled with one uniform each when not greedy).
    void draft(Seq& s) {
        mtp_forward(mtp, d(), s.hidden.data(), emb.data(), V(), s.mtp_logits.data(), nullptr);
        const bool greedy = sampling_is_greedy(samp);
        for (uint32_t h = 0; h < K(); h++) {
            const float* lg = s.mtp_logits.data() + (size_t)h * V();
            s.drafts[h] = greedy ? argmax(lg, V()) : sample(lg, V(), samp, draw(s));
        }
    }

    void prefill(int32_t n, const int32_t* tok, const int64_t* off, const uint32_t* seeds) {
        seqs.clear();
        seqs.resize(n);
        const bool greedy = sampling_is_greedy(samp);
        for_each_seq(n, prefill_threads > 1 ? 1 : threads, [&](int b) {
            tl_mm_threads = prefill_threads;
            std::vector<float> lg(V());
            Seq& s = seqs[b];
            new_seq(s, seeds ? seeds[b] : 0u);
            const int64_t a = off[b], e = off[b + 1];
            for (int64_t i = a; i < e; i++) {
                const bool last = (i + 1 == e);
                forward_row(s, tok[i], s.pos, last ? lg.data() : nullptr, last ? s.hidden.data() : nullptr);
                s.pos++;
            }
            s.pending = greedy ? argmax(lg.data(), V()) : sample(lg.data(), V(), samp, draw(s));
            draft(s);
            tl_mm_threads = 1;
        });
        last_logits.assign((size_t)n * (K() + 1) * V(), 0.0f);
    }

    // One Level-B step for every sequence.
    void step(int32_t* n_emitted, int32_t* emitted) {
        const uint32_t R = K() + 1;
        const bool greedy = sampling_is_greedy(samp);
        for_each_seq((int)seqs.size(), threads, [&](int b) {
            std::vector<float> hid((size_t)R * d());
            Seq& s = seqs[b];
            std::vector<int32_t> in(R);
            in[0] = s.pending;
            for (uint32_t r = 1; r < R; r++) in[r] = s.drafts[r - 1];
            TierCache kv_keep = s.kv;
            SkipState sk_keep = s.skip;
            const int64_t comp_keep = s.ffn_computed, skip_keep = s.ffn_skipped;
            float* lg = last_logits.data() + (size_t)b * R * V();
            for (uint32_t r = 0; r < R; r++)
                forward_row(s, in[r], s.pos + r, lg + (size_t)r * V(), hid.data() + (size_t)r * d());
            uint32_t acc = 0;
            while (acc < K() && argmax(lg + (size_t)acc * V(), V()) == s.drafts[acc]) acc++;
            const float* fin = lg + (size_t)acc * V();
            const int32_t next = greedy ? argmax(fin, V()) : sample(fin, V(), samp, draw(s));
            // Commit rows 0..acc only (D7): replay them on the saved state.
            s.kv = std::move(kv_keep);
            s.skip = std::move(sk_keep);
            s.ffn_computed = comp_keep;
            s.ffn_skipped = skip_keep;
            for (uint32_t r = 0; r <= acc; r++) forward_row(s, in[r], s.pos + r, nullptr, nullptr);
            if (n_emitted) n_emitted[b] = (int32_t)acc + 1;
            if (emitted) {
                for (uint32_t r = 0; r < R; r++) emitted[b * R + r] = -1;
                for (uint32_t r = 0; r < acc; r++) emitted[b * R + r] = s.drafts[r];
                emitted[b * R + acc] = next;
            }
            s.pos += acc + 1;
            s.pending = next;
            std::memcpy(s.hidden.data(), hid.data() + (size_t)acc * d(), d() * sizeof(float));
            draft(s);
        });
    }
};

}  // namespace po

// ===========================================================================
// extern "C" API (ctypes).  Prefix po_.
// ===========================================================================
extern "C" {

void po_quantize_activation_row(const float* s, int8_t* d, float* sc, uint32_t n) { po::quant_act_row(s, d, sc, n); }
void po_kv_quantize_row(const float* s, int8_t* d, float* sc, uint32_t n) { po::quant_kv_row(s, d, sc, n); }
void po_dequant_q4_to_int8(const uint8_t* s, int8_t* d, uint64_t n) { po::unpack_q4(s, d, n); }
void po_dequant_q2_to_int8(const uint8_t* s, int8_t* d, uint64_t n) { po::unpack_q2(s, d, n); }
void po_dequant_ternary_to_int8(const uint8_t* s, int8_t* d, uint64_t n) { po::unpack_ternary(s, d, n); }
void po_matmul_int8(const int8_t* A, const int8_t* B, int32_t* C, uint32_t M, uint32_t N, uint32_t K) {
    po::mm_int8(A, B, C, M, N, K);
}
void po_matmul_quantized(const float* A, const int8_t* B, float* C, uint32_t M, uint32_t N, uint32_t K,
                         const float* ws, const float* as) {
    po::mm_quant(A, B, C, M, N, K, ws, as);
}
void po_rmsnorm(float* out, const float* x, const float* w, uint32_t n, float eps, int order) {
    po::rmsnorm(out, x, w, n, eps, order);
}
void po_softmax(float* v, uint32_t n) { po::softmax(v, n); }
float po_swiglu_engine(float g, float u) { return po::swiglu_engine(g, u); }
float po_silu_mtp(float x) { return po::silu_mtp(x); }
int32_t po_argmax(const float* v, uint32_t n) { return po::argmax(v, n); }
int32_t po_sample(const float* lg, uint32_t n, const pf_sampling_config* c, float u) {
    return po::sample(lg, n, *c, u);
}
int32_t po_sample_top_p(const float* lg, uint32_t n, float p, float t, float u) { return po::sample_top_p(lg, n, p, t, u); }
int32_t po_sample_top_k(const float* lg, uint32_t n, uint32_t k, float t, float u) { return po::sample_top_k(lg, n, k, t, u); }
// The reference's uniform draws: std::uniform_real_distribution<float>(0,1) over
// std::mt19937(seed) (src/engine.cpp:16,909,952,996).
void po_uniforms(uint32_t seed, uint32_t n, float* out) {
    std::mt19937 r(seed);
    std::uniform_real_distribution<float> u(0.0f, 1.0f);
    for (uint32_t i = 0; i < n; i++) out[i] = u(r);
}
void po_rope_table(float theta, uint32_t hd, uint32_t n_pos, float* cs, float* sn) {
    for (uint32_t p = 0; p < n_pos; p++) po::rope_row(theta, hd, p, cs + (size_t)p * (hd / 2), sn + (size_t)p * (hd / 2));
}
// Quantizer::quantize_matrix: returns the byte size; writes when out != NULL.
uint64_t po_quantize_matrix(const float* data, uint32_t rows, uint32_t cols, int qtype, uint8_t* out) {
    auto v = po::quantize_matrix(data, rows, cols, qtype);
    if (out) std::memcpy(out, v.data(), v.size());
    return v.size();
}
void po_loader_decode(const uint8_t* blk, uint64_t blk_bytes, uint32_t rows, uint32_t cols, int qtype,
                      int8_t* out, float* row_scales, float* global_scale) {
    std::vector<uint8_t> b(blk, blk + blk_bytes);
    po::loader_decode(b, rows, cols, qtype, out, row_scales, global_scale);
}
void po_synth_matrix(uint32_t seed, uint32_t layer, uint32_t matrix, uint32_t rows, uint32_t cols, int qtype,
                     int8_t* out, float* row_scales, float* global_scale) {
    po::synth_matrix(seed, layer, matrix, rows, cols, qtype, out, row_scales, global_scale);
}
void po_synth_normals(uint32_t seed, uint32_t layer, uint32_t matrix, uint64_t n, float* out) {
    std::mt19937 rng(po::matrix_seed(seed, layer, matrix));
    std::normal_distribution<float> nd(0.0f, 0.02f);
    for (uint64_t i = 0; i < n; i++) out[i] = nd(rng);
}
void po_mtp_quantize_q4(const float* src, uint8_t* dst, float* scales, uint32_t rows, uint32_t cols) {
    po::mtp_quantize_q4(src, dst, scales, rows, cols);
}
void po_synth_mtp_matrix(uint32_t seed, uint32_t head, uint32_t j, uint32_t d, uint8_t* q4, float* scales) {
    po::synth_mtp_matrix(seed, head, j, d, q4, scales);
}
// MTPHeads::forward for n_heads heads with weights given as flat arrays
// [head][3 (gate, up, down)][d][d/2] bytes and scales [head][3][d].
void po_mtp_forward(uint32_t n_heads, uint32_t d, const uint8_t* q4, const float* scales,
                    const float* hidden, const float* emb, uint32_t vocab, float* logits,
                    float* final_hidden) {
    std::vector<po::MtpHead> hs(n_heads);
    const size_t mb = (size_t)d * (d / 2);
    for (uint32_t h = 0; h < n_heads; h++) {
        const uint8_t* b = q4 + (size_t)h * 3 * mb;
        const float* s = scales + (size_t)h * 3 * d;
        hs[h].gate.assign(b, b + mb);
        hs[h].up.assign(b + mb, b + 2 * mb);
        hs[h].down.assign(b + 2 * mb, b + 3 * mb);
        hs[h].gs.assign(s, s + d);
        hs[h].us.assign(s + d, s + 2 * d);
        hs[h].ds.assign(s + 2 * d, s + 3 * d);
    }
    po::mtp_forward(hs, d, hidden, emb, vocab, logits, final_hidden);
}

// ---- tiered KV cache object ----
void* po_kv_create(uint32_t L, uint32_t H, uint32_t hd, uint32_t sink, uint32_t window, uint32_t pool,
                   uint32_t max_ctx) {
    auto* c = new po::TierCache();
    c->init(L, H, hd, sink, window, pool, max_ctx);
    return c;
}
void po_kv_destroy(void* c) { delete (po::TierCache*)c; }
void po_kv_store(void* c, uint32_t l, uint32_t h, uint32_t pos, const float* k, const float* v) {
    ((po::TierCache*)c)->store(l, h, pos, k, v);
}
uint32_t po_kv_scores(void* c, uint32_t l, uint32_t h, const float* q, float* out) {
    return ((po::TierCache*)c)->scores(l, h, q, out);
}
void po_kv_weighted_sum(void* c, uint32_t l, uint32_t h, const float* p, float* out, uint32_t cnt) {
    ((po::TierCache*)c)->weighted_sum(l, h, p, out, cnt);
}
uint32_t po_kv_count(void* c, uint32_t l, uint32_t h) { return ((po::TierCache*)c)->count(l, h); }
uint32_t po_kv_size(void* c) { return ((po::TierCache*)c)->stored; }
// Entries in attention order: k,v [count][hd], scales [count].
uint32_t po_kv_dump(void* c, uint32_t l, uint32_t h, int8_t* k, float* ks, int8_t* v, float* vs, uint32_t max_n) {
    auto* t = (po::TierCache*)c;
    const uint32_t n = std::min(t->count(l, h), max_n);
    for (uint32_t e = 0; e < n; e++) {
        const int8_t *kp, *vp;
        float a, b;
        t->entry(l, h, e, &kp, &a, &vp, &b);
        std::memcpy(k + (size_t)e * t->hd, kp, t->hd);
        std::memcpy(v + (size_t)e * t->hd, vp, t->hd);
        ks[e] = a;
        vs[e] = b;
    }
    return n;
}
// fp64 pooling accumulator of one head: count, then hd doubles for K and V.
uint32_t po_kv_acc(void* c, uint32_t l, uint32_t h, double* ak, double* av) {
    auto& t = ((po::TierCache*)c)->at(l, h);
    std::memcpy(ak, t.ak.data(), t.hd * sizeof(double));
    std::memcpy(av, t.av.data(), t.hd * sizeof(double));
    return t.n_acc;
}

// ---- layer skip object ----
void* po_skip_create(uint32_t L, uint32_t d, float thr) {
    auto* s = new po::SkipState();
    s->init(L, d, thr);
    return s;
}
void po_skip_destroy(void* s) { delete (po::SkipState*)s; }
int po_skip_should_skip(void* s, uint32_t layer, const float* x, int order) {
    return ((po::SkipState*)s)->should_skip(layer, x, order) ? 1 : 0;
}
void po_skip_set_threshold(void* s, float t) { ((po::SkipState*)s)->thr = t; }
float po_skip_delta(const float* a, const float* b, uint32_t n, int order) {
    return po::SkipState::delta(a, b, n, order);
}

// ---- Level-B engine ----
void* po_engine_create(const pf_model_config* cfg) {
    auto* e = new po::Engine();
    e->init(*cfg);
    return e;
}
void po_engine_destroy(void* e) { delete (po::Engine*)e; }
void po_engine_set_order(void* e, int order) { ((po::Engine*)e)->order = order; }
void po_engine_set_sampling(void* e, const pf_sampling_config* c) { ((po::Engine*)e)->samp = *c; }
void po_engine_set_skip_threshold(void* e, float t) { ((po::Engine*)e)->cfg.skip_threshold = t; }
void po_engine_set_matrix(void* ep, uint32_t layer, uint32_t m, const int8_t* w, const float* rs) {
    auto* e = (po::Engine*)ep;
    uint32_t r, c;
    e->mat_shape((int)m, &r, &c);
    e->w[m][layer].assign(w, w + (size_t)r * c);
    e->rs[m][layer].assign(rs, rs + r);
}
void po_engine_set_embedding(void* ep, const int8_t* emb, float gscale) {
    auto* e = (po::Engine*)ep;
    const size_t n = (size_t)e->cfg.n_vocab * e->cfg.n_embd;
    e->emb.resize(n);
    for (size_t i = 0; i < n; i++) e->emb[i] = (float)emb[i] * gscale;
}
void po_engine_set_norms(void* ep, const float* a, const float* f, const float* fin) {
    auto* e = (po::Engine*)ep;
    const size_t n = (size_t)e->cfg.n_layers * e->cfg.n_embd;
    if (a) e->attn_norm.assign(a, a + n);
    if (f) e->ffn_norm.assign(f, f + n);
    if (fin) e->final_norm.assign(fin, fin + e->cfg.n_embd);
}
void po_engine_set_mtp_head(void* ep, uint32_t h, const uint8_t* g, const float* gs, const uint8_t* u,
                            const float* us, const uint8_t* dn, const float* ds) {
    auto* e = (po::Engine*)ep;
    const size_t d = e->cfg.n_embd, mb = d * (d / 2);
    auto& m = e->mtp[h];
    m.gate.assign(g, g + mb);
    m.up.assign(u, u + mb);
    m.down.assign(dn, dn + mb);
    m.gs.assign(gs, gs + d);
    m.us.assign(us, us + d);
    m.ds.assign(ds, ds + d);
}
void po_engine_prefill(void* e, int32_t n, const int32_t* tok, const int64_t* off, const uint32_t* seeds) {
    ((po::Engine*)e)->prefill(n, tok, off, seeds);
}
void po_engine_step(void* e, int32_t* n_emitted, int32_t* emitted) { ((po::Engine*)e)->step(n_emitted, emitted); }
void po_engine_read_logits(void* ep, float* out) {
    auto* e = (po::Engine*)ep;
    std::memcpy(out, e->last_logits.data(), e->last_logits.size() * sizeof(float));
}
// Replaces the pending drafts (drafts from another proposer; used to drive
// the acceptance and commit paths in tests).
void po_engine_set_drafts(void* ep, const int32_t* in) {
    auto* e = (po::Engine*)ep;
    for (size_t b = 0; b < e->seqs.size(); b++)
        std::memcpy(e->seqs[b].drafts.data(), in + b * e->K(), e->K() * sizeof(int32_t));
}
void po_engine_read_drafts(void* ep, int32_t* out) {
    auto* e = (po::Engine*)ep;
    for (size_t b = 0; b < e->seqs.size(); b++)
        std::memcpy(out + b * e->K(), e->seqs[b].drafts.data(), e->K() * sizeof(int32_t));
}
void po_engine_read_pending(void* ep, int32_t* out) {
    auto* e = (po::Engine*)ep;
    for (size_t b = 0; b < e->seqs.size(); b++) out[b] = e->seqs[b].pending;
}
void po_engine_read_positions(void* ep, int32_t* out) {
    auto* e = (po::Engine*)ep;
    for (size_t b = 0; b < e->seqs.size(); b++) out[b] = (int32_t)e->seqs[b].pos;
}
void po_engine_read_hidden(void* ep, float* out) {
    auto* e = (po::Engine*)ep;
    for (size_t b = 0; b < e->seqs.size(); b++)
        std::memcpy(out + b * e->d(), e->seqs[b].hidden.data(), e->d() * sizeof(float));
}
void po_engine_read_mtp_logits(void* ep, float* out) {
    auto* e = (po::Engine*)ep;
    const size_t n = (size_t)e->K() * e->V();
    for (size_t b = 0; b < e->seqs.size(); b++)
        std::memcpy(out + b * n, e->seqs[b].mtp_logits.data(), n * sizeof(float));
}
float po_engine_skip_margin(void* ep) { return ((po::Engine*)ep)->skip_margin(); }
void po_engine_read_skip_counts(void* ep, int64_t* comp, int64_t* skip) {
    auto* e = (po::Engine*)ep;
    *comp = e->ffn_computed();
    *skip = e->ffn_skipped();
}
// Host threads over sequences for prefill and step (1: one after another;
// the results do not depend on it).
void po_engine_set_threads(void* ep, int threads) { ((po::Engine*)ep)->threads = std::max(1, threads); }
// > 1: prefill sequences one after another with their matmuls' output columns
// on this many host threads (results do not depend on it).
void po_engine_set_prefill_threads(void* ep, int threads) {
    ((po::Engine*)ep)->prefill_threads = std::max(1, threads);
}
uint32_t po_engine_read_kv(void* ep, int32_t b, uint32_t l, uint32_t h, int8_t* k, float* ks, int8_t* v,
                           float* vs, uint32_t max_n) {
    auto* e = (po::Engine*)ep;
    return po_kv_dump(&e->seqs[b].kv, l, h, k, ks, v, vs, max_n);
}
// Generates (on `threads` host threads) and loads the whole synthetic model.
void po_engine_load_synthetic(void* ep, uint32_t seed, uint32_t mtp_seed, int threads) {
    auto* e = (po::Engine*)ep;
    const uint32_t L = (uint32_t)e->cfg.n_layers;
    std::vector<std::pair<uint32_t, uint32_t>> jobs;
    for (uint32_t l = 0; l < L; l++)
        for (uint32_t m = 0; m < PF_MAT_COUNT; m++) jobs.push_back({l, m});
    std::atomic<size_t> next{0};
    auto work = [&]() {
        for (size_t j; (j = next++) < jobs.size();) {
            const uint32_t l = jobs[j].first, m = jobs[j].second;
            uint32_t r, c;
            e->mat_shape((int)m, &r, &c);
            std::vector<int8_t> w((size_t)r * c);
            std::vector<float> rs(r);
            float gs;
            po::synth_matrix(seed, l, m, r, c, e->cfg.qtype[m], w.data(), rs.data(), &gs);
            e->w[m][l] = std::move(w);
            e->rs[m][l] = std::move(rs);
        }
    };
    std::vector<std::thread> pool;
    for (int t = 0; t < std::max(1, threads); t++) pool.emplace_back(work);
    for (auto& t : pool) t.join();
    const size_t V = e->cfg.n_vocab, d = e->cfg.n_embd;
    std::vector<int8_t> emb(V * d);
    std::vector<float> rs(V);
    float gs;
    po::synth_matrix(seed, 0, 10, (uint32_t)V, (uint32_t)d, e->cfg.emb_qtype, emb.data(), rs.data(), &gs);
    po_engine_set_embedding(ep, emb.data(), gs);
    for (int h = 0; h < e->cfg.n_mtp_heads; h++) {
        std::vector<uint8_t> q[3];
        std::vector<float> s[3];
        for (int j = 0; j < 3; j++) {
            q[j].resize(d * d / 2);
            s[j].resize(d);
            po::synth_mtp_matrix(mtp_seed, h, j, (uint32_t)d, q[j].data(), s[j].data());
        }
        po_engine_set_mtp_head(ep, h, q[0].data(), s[0].data(), q[1].data(), s[1].data(), q[2].data(), s[2].data());
    }
}

// One token through the model for sequence b without changing its state
// (the logits and hidden that row would produce at the next position).
void po_engine_probe_row(void* ep, int32_t b, int32_t token, float* logits, float* hidden) {
    auto* e = (po::Engine*)ep;
    po::Seq s = e->seqs[b];
    e->forward_row(s, token, s.pos, logits, hidden);
}

}  // extern "C"

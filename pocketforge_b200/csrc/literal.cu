// literal.cu — kernels of forge::Engine's reference-compat mode (the
// reference's literal Engine::forward_with_hidden, src/engine.cpp:459-589).
//
// The literal forward is a chain of single-vector steps whose reductions the
// reference runs as plain sequential float loops.  Each kernel here does the
// element-wise parts in parallel and runs every such loop in one thread, in
// the reference's index order, with each product and sum rounded on its own
// (__fmul_rn / __fadd_rn: no contraction into FMA), so the results are the
// reference's bits.  The one exception is std::exp (softmax, SiLU): the device
// rounds the double exponential to float, which is the correctly rounded value;
// glibc's expf can differ from it by one unit in the last place.
#include <cmath>

#include "common.cuh"
#include "literal.h"

namespace pf {
namespace lit {
namespace {

__device__ __forceinline__ float madd(float s, float a, float b) { return __fadd_rn(s, __fmul_rn(a, b)); }
__device__ __forceinline__ float exp_ref(float x) { return (float)exp((double)x); }

constexpr int kRowThreads = 1024;  // one-block phases over n_embd
constexpr int kScoreThreads = 128;
constexpr int kSoftmaxThreads = 256;
constexpr int kStoreThreads = 128;
constexpr int kUnembedRows = 128;
constexpr int kUnembedCols = 128;
constexpr int kTilePitch = kUnembedCols + 4;  // bytes per staged row: word stride 33, no bank conflicts

// Entry e of unit u in the reference's attention order: sink rows, pooled
// rows, then the window oldest first (src/kv_cache.cpp:129-158).
struct Entry {
    const int8_t* row;
    float scale;
};
__device__ __forceinline__ Entry entry(const Cache& c, const Tiers& t, uint32_t u, uint32_t hd, uint32_t e,
                                       bool value) {
    if (e < t.n_sink) {
        const size_t r = (size_t)u * c.sink_cap + e;
        return {(value ? c.sv : c.sk) + r * hd, (value ? c.svs : c.sks)[r]};
    }
    e -= t.n_sink;
    if (e < t.n_pool) {
        const size_t r = (size_t)u * c.pool_cap + e;
        return {(value ? c.pv : c.pk) + r * hd, (value ? c.pvs : c.pks)[r]};
    }
    e -= t.n_pool;
    const uint32_t slot = t.n_win < c.ring ? e : (t.head + e) % c.ring;
    const size_t r = (size_t)u * c.ring + slot;
    return {(value ? c.wv : c.wk) + r * hd, (value ? c.wvs : c.wks)[r]};
}

// RMSNorm of x into out (shared memory), src/matmul_neon.cpp:231-239:
// ss = sum x^2 in order, rms = sqrt(ss / n + 1e-6), out = x * (1/rms) * w.
// `sq` is n floats of shared memory; `inv` one shared float.
__device__ void rmsnorm_block(const float* x, const float* w, uint32_t n, float* sq, float* out, float* inv) {
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) sq[i] = __fmul_rn(x[i], x[i]);
    __syncthreads();
    if (threadIdx.x == 0) {
        float ss = 0.0f;
#pragma unroll 8
        for (uint32_t i = 0; i < n; i++) ss = __fadd_rn(ss, sq[i]);
        *inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), 1e-6f)));
    }
    __syncthreads();
    const float r = *inv;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(x[i], r), w[i]);
    __syncthreads();
}

__global__ void embed_kernel(Model m, int32_t token) {
    const bool table = m.emb_loaded && (uint32_t)token < m.n_vocab;
    const uint64_t seed = (uint64_t)(int64_t)token * 2654435761ull;
    for (uint32_t i = threadIdx.x; i < m.d; i += blockDim.x) {
        float x;
        if (table)
            x = (uint32_t)token < m.emb_rows ? __fmul_rn((float)m.emb[(size_t)token * m.d + i], m.emb_scale) : 0.0f;
        else
            x = __fdiv_rn((float)((seed + (uint64_t)i * 7919ull) % 10000ull), 10000.0f);
        m.hidden[i] = x;
    }
}

// RMSNorm, Q = K = V = 0.1 x normed over the first n_embd entries
// (src/engine.cpp:718-724), then RoPE at position l (:726-750): for each query
// head h in order, its pairs and those of K head h % n_kv are rotated, so a K
// head is rotated once per query head that maps to it.
__global__ void pre_attn_kernel(Model m, uint32_t l) {
    extern __shared__ float sh[];
    float* sq = sh;
    float* nrm = sh + m.d;
    __shared__ float inv;
    rmsnorm_block(m.hidden, m.attn_w + (size_t)l * m.d, m.d, sq, nrm, &inv);
    for (uint32_t i = threadIdx.x; i < m.d; i += blockDim.x) {
        const float t = __fmul_rn(nrm[i], 0.1f);
        m.q[i] = t;
        m.k[i] = t;
        m.v[i] = t;
    }
    __syncthreads();
    const uint32_t hd = m.hd, pairs = (hd + 1) / 2;
    const float* cs = m.rope_cos + (size_t)l * hd;
    const float* sn = m.rope_sin + (size_t)l * hd;
    for (uint32_t idx = threadIdx.x; idx < m.n_kv * pairs; idx += blockDim.x) {
        const uint32_t kv = idx / pairs, i = 2 * (idx % pairs);
        const bool two = i + 1 < hd;
        const float c = cs[i], s = sn[i];
        float* kh = m.k + (size_t)kv * hd;
        for (uint32_t h = kv; h < m.n_heads; h += m.n_kv) {
            float* qh = m.q + (size_t)h * hd;
            const float q0 = qh[i], q1 = two ? qh[i + 1] : 0.0f;
            const float k0 = kh[i], k1 = two ? kh[i + 1] : 0.0f;
            qh[i] = __fsub_rn(__fmul_rn(q0, c), __fmul_rn(q1, s));
            if (two) qh[i + 1] = __fadd_rn(__fmul_rn(q0, s), __fmul_rn(q1, c));
            kh[i] = __fsub_rn(__fmul_rn(k0, c), __fmul_rn(k1, s));
            if (two) kh[i + 1] = __fadd_rn(__fmul_rn(k0, s), __fmul_rn(k1, c));
        }
    }
}

// KVCache::attention_scores for every query head (src/kv_cache.cpp:12-16,
// 129-158) times 1/sqrt(head_dim) (src/engine.cpp:767-768).
__global__ void scores_kernel(Model m, uint32_t l, Tiers t, float scale) {
    const uint32_t e = blockIdx.x * blockDim.x + threadIdx.x, h = blockIdx.y;
    if (e >= t.count()) return;
    const uint32_t u = l * m.n_kv + h % m.n_kv;
    const Entry en = entry(m.c, t, u, m.hd, e, false);
    const float* q = m.q + (size_t)h * m.hd;
    float s = 0.0f;
    for (uint32_t i = 0; i < m.hd; i++) s = madd(s, q[i], __fmul_rn((float)en.row[i], en.scale));
    m.scores[(size_t)h * m.score_stride + e] = __fmul_rn(s, scale);
}

// The float self term, the scale, and softmax over count + 1 scores
// (src/engine.cpp:759-769, src/matmul_neon.cpp:212-227): max in order (a NaN
// first value stays the max, later NaNs are passed over), exp(x - max), the
// sum in order, 1 / (sum + 1e-10), products.
__global__ void softmax_kernel(Model m, Tiers t, float scale) {
    const uint32_t h = blockIdx.x, kv = h % m.n_kv, n = t.count();
    float* sc = m.scores + (size_t)h * m.score_stride;
    __shared__ float red[kSoftmaxThreads / 32];
    __shared__ float bc;
    if (threadIdx.x == 0) {
        const float* q = m.q + (size_t)h * m.hd;
        const float* k = m.k + (size_t)kv * m.hd;
        float s = 0.0f;
        for (uint32_t i = 0; i < m.hd; i++) s = madd(s, q[i], k[i]);
        sc[n] = __fmul_rn(s, scale);
    }
    __syncthreads();
    float mx = -INFINITY;
    for (uint32_t i = threadIdx.x; i <= n; i += blockDim.x) mx = fmaxf(mx, sc[i]);
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        float r = -INFINITY;
        for (int w = 0; w < kSoftmaxThreads / 32; w++) r = fmaxf(r, red[w]);
        const float first = sc[0];
        bc = isnan(first) ? first : fmaxf(r, first);
    }
    __syncthreads();
    mx = bc;
    for (uint32_t i = threadIdx.x; i <= n; i += blockDim.x) sc[i] = exp_ref(__fsub_rn(sc[i], mx));
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f;
#pragma unroll 8
        for (uint32_t i = 0; i <= n; i++) s = __fadd_rn(s, sc[i]);
        bc = __fdiv_rn(1.0f, __fadd_rn(s, 1e-10f));
    }
    __syncthreads();
    const float inv = bc;
    for (uint32_t i = threadIdx.x; i <= n; i += blockDim.x) sc[i] = __fmul_rn(sc[i], inv);
    __syncthreads();
    if (threadIdx.x == 0) m.self_p[h] = sc[n];
}

// Head outputs as the reference leaves them (src/engine.cpp:771-778):
// attention_weighted_sum clears and writes entries [0, hd) of the output for
// every head, so those hold the LAST head's cached sum; each head h adds its
// self term at [h*hd, (h+1)*hd) into a zeroed buffer, where only heads h >= 1
// (and head 0 when it is the only head) survive.  Then the residual.
__global__ void attn_out_kernel(Model m, uint32_t l, Tiers t) {
    const uint32_t hd = m.hd, H = m.n_heads, last = H - 1, n = t.count();
    const uint32_t u = l * m.n_kv + last % m.n_kv;
    const float* p = m.scores + (size_t)last * m.score_stride;
    for (uint32_t j = threadIdx.x; j < hd; j += blockDim.x) {
        float s = 0.0f;
        for (uint32_t e = 0; e < n; e++) {
            const Entry en = entry(m.c, t, u, hd, e, true);
            s = madd(s, p[e], __fmul_rn((float)en.row[j], en.scale));
        }
        if (H == 1) s = madd(s, m.self_p[0], m.v[j]);
        m.attn_out[j] = s;
    }
    for (uint32_t idx = threadIdx.x; idx < (H - 1) * hd; idx += blockDim.x) {
        const uint32_t h = 1 + idx / hd, j = idx % hd;
        m.attn_out[(size_t)h * hd + j] = __fadd_rn(0.0f, __fmul_rn(m.self_p[h], m.v[(size_t)(h % m.n_kv) * hd + j]));
    }
    for (uint32_t i = H * hd + threadIdx.x; i < m.d; i += blockDim.x) m.attn_out[i] = 0.0f;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < m.d; i += blockDim.x) m.hidden[i] = __fadd_rn(m.hidden[i], m.attn_out[i]);
}

// KVCache::quantize_row (src/kv_cache.cpp:19-28) by one block: amax (NaNs
// passed over), scale = amax / 127 and q = round(x * (127 / amax)), 1 for zero rows.
__device__ void quantize_block(const float* x, uint32_t n, int8_t* q, float* scale, float* red) {
    float a = 0.0f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) a = fmaxf(a, fabsf(x[i]));
    for (int o = 16; o; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
    __syncthreads();
    float amax = 0.0f;
    for (uint32_t w = 0; w < blockDim.x / 32; w++) amax = fmaxf(amax, red[w]);
    const float inv = amax == 0.0f ? 1.0f : __fdiv_rn(127.0f, amax);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) q[i] = (int8_t)(int)roundf(__fmul_rn(x[i], inv));
    if (threadIdx.x == 0) *scale = amax == 0.0f ? 1.0f : __fdiv_rn(amax, 127.0f);
    __syncthreads();
}

// KVCache::store(l, kv, pos = l) for every kv head (src/engine.cpp:780-785,
// src/kv_cache.cpp:59-127); the host decides the rows (Store).
__global__ void store_kernel(Model m, uint32_t l, Store op) {
    extern __shared__ float mean[];  // [hd]
    __shared__ float red[kStoreThreads / 32];
    const Cache& c = m.c;
    const uint32_t kv = blockIdx.x, hd = m.hd, u = l * m.n_kv + kv;
    const float* key = m.k + (size_t)kv * hd;
    const float* val = m.v + (size_t)kv * hd;
    if (op.kind == 1) {
        const size_t r = (size_t)u * c.sink_cap + op.slot;
        quantize_block(key, hd, c.sk + r * hd, c.sks + r, red);
        quantize_block(val, hd, c.sv + r * hd, c.svs + r, red);
        return;
    }
    const size_t r = (size_t)u * c.ring + op.slot;
    if (op.evict) {
        double* ak = c.ak + (size_t)u * hd;
        double* av = c.av + (size_t)u * hd;
        const double ks = c.wks[r], vs = c.wvs[r];
        for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) {
            ak[i] += (double)c.wk[r * hd + i] * ks;
            av[i] += (double)c.wv[r * hd + i] * vs;
        }
        __syncthreads();
        if (op.finalize) {
            const double inv = (double)__fdiv_rn(1.0f, (float)op.acc_n);
            const size_t pr = (size_t)u * c.pool_cap + op.pool_row;
            for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) mean[i] = (float)(ak[i] * inv);
            __syncthreads();
            quantize_block(mean, hd, c.pk + pr * hd, c.pks + pr, red);
            for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) mean[i] = (float)(av[i] * inv);
            __syncthreads();
            quantize_block(mean, hd, c.pv + pr * hd, c.pvs + pr, red);
            for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) ak[i] = av[i] = 0.0;
        }
    }
    quantize_block(key, hd, c.wk + r * hd, c.wks + r, red);
    quantize_block(val, hd, c.wv + r * hd, c.wvs + r, red);
}

// RMSNorm, LayerSkipController::should_skip_ffn on the normed vector
// (src/layer_skip.cpp:21-67, hidden_delta :105-113) and, unless skipped, the
// placeholder FFN (src/engine.cpp:840-848): every output element is
// max(0, sum_j normed[j] * 0.01), added to the hidden state.
__global__ void ffn_kernel(Model m, uint32_t l) {
    extern __shared__ float sh[];
    float* sq = sh;
    float* nrm = sh + m.d;
    __shared__ float inv, delta, val;
    rmsnorm_block(m.hidden, m.ffn_w + (size_t)l * m.d, m.d, sq, nrm, &inv);
    float* cache = m.skip_cache + (size_t)l * m.d;
    if (threadIdx.x == 0 && !m.skip_anchor) {
        float s = 0.0f;
#pragma unroll 4
        for (uint32_t i = 0; i < m.d; i++) {
            const float dd = __fsub_rn(nrm[i], cache[i]);
            s = madd(s, dd, dd);
        }
        delta = __fsqrt_rn(__fdiv_rn(s, (float)m.d));
    }
    if (threadIdx.x == 32) {
        float s = 0.0f;
#pragma unroll 8
        for (uint32_t j = 0; j < m.d; j++) s = madd(s, nrm[j], 0.01f);
        val = s;
    }
    __syncthreads();
    bool skip = false;
    if (!m.skip_anchor) {
        const uint32_t L = m.n_layers, mid = L / 2;
        float thr = m.skip_threshold;
        if (l > mid / 2 && l < mid + mid / 2) thr = __fmul_rn(thr, 2.0f);
        if (l < 2 || l >= L - 2) thr = -1.0f;
        skip = delta < thr;
    }
    if (skip) return;
    const float out = 0.0f < val ? val : 0.0f;
    for (uint32_t i = threadIdx.x; i < m.d; i += blockDim.x) {
        cache[i] = nrm[i];
        m.hidden[i] = __fadd_rn(m.hidden[i], out);
    }
}

// logits[v] = sum_i h[i] * (E[v][i] * scale), one thread per vocabulary row in
// index order; the block stages 128 rows x 128 columns of E at a time.
__global__ void unembed_kernel(const int8_t* __restrict__ emb, float scale, const float* __restrict__ h, uint32_t d,
                               uint32_t n_vocab, float* __restrict__ logits) {
    extern __shared__ float hs[];  // [d] floats, then the tile
    uint8_t* tile = reinterpret_cast<uint8_t*>(hs + d);
    for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) hs[i] = h[i];
    const uint32_t v0 = blockIdx.x * kUnembedRows, v = v0 + threadIdx.x;
    const bool words = (d % 4) == 0;
    float s = 0.0f;
    for (uint32_t c0 = 0; c0 < d; c0 += kUnembedCols) {
        const uint32_t cols = min((uint32_t)kUnembedCols, d - c0);
        __syncthreads();
        if (words) {
            const uint32_t wpr = cols / 4;  // words per staged row
            for (uint32_t idx = threadIdx.x; idx < kUnembedRows * wpr; idx += blockDim.x) {
                const uint32_t r = idx / wpr, w = idx % wpr;
                uint32_t x = 0;
                if (v0 + r < n_vocab) x = *reinterpret_cast<const uint32_t*>(emb + (size_t)(v0 + r) * d + c0 + 4 * w);
                *reinterpret_cast<uint32_t*>(tile + r * kTilePitch + 4 * w) = x;
            }
        } else {
            for (uint32_t idx = threadIdx.x; idx < kUnembedRows * cols; idx += blockDim.x) {
                const uint32_t r = idx / cols, cc = idx % cols;
                tile[r * kTilePitch + cc] = v0 + r < n_vocab ? (uint8_t)emb[(size_t)(v0 + r) * d + c0 + cc] : 0;
            }
        }
        __syncthreads();
        const int8_t* row = reinterpret_cast<const int8_t*>(tile + threadIdx.x * kTilePitch);
        for (uint32_t cc = 0; cc < cols; cc++) s = madd(s, hs[c0 + cc], __fmul_rn((float)row[cc], scale));
    }
    if (v < n_vocab) logits[v] = s;
}

__global__ void placeholder_logits_kernel(int32_t token, uint32_t n_vocab, float* logits) {
    const uint32_t v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v >= n_vocab) return;
    const uint64_t h = (uint64_t)(int64_t)token * 2654435761ull + (uint64_t)v * 7919ull;
    logits[v] = __fdiv_rn((float)(h % 10000ull), 10000.0f);
}

// y[r] = sum_i x[i] * ((nibble_i - 8) * scale[r]) for one packed Q4 row per
// thread (MTPHeads::dequant_q4_row then the dot product, src/mtp.cpp:66-101).
__global__ void q4_rows_kernel(const float* __restrict__ x, const uint8_t* __restrict__ w,
                               const float* __restrict__ scale, float* __restrict__ y, uint32_t rows, uint32_t cols) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const uint8_t* wr = w + (size_t)r * (cols / 2);
    const float sc = scale[r];
    float s = 0.0f;
    for (uint32_t i = 0; i < cols; i += 2) {
        const uint8_t b = wr[i / 2];
        s = madd(s, x[i], __fmul_rn((float)((int)(b & 0x0F) - 8), sc));
        if (i + 1 < cols) s = madd(s, x[i + 1], __fmul_rn((float)((int)(b >> 4) - 8), sc));
    }
    y[r] = s;
}
// silu(g) * u with silu(x) = x / (1 + exp(-x)) (src/mtp.cpp:94-96, 146-148).
__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ a,
                                uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) a[i] = __fmul_rn(__fdiv_rn(g[i], __fadd_rn(1.0f, exp_ref(-g[i]))), u[i]);
}
__global__ void add_kernel(float* __restrict__ y, const float* __restrict__ x, uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __fadd_rn(y[i], x[i]);
}

inline unsigned blocks(uint32_t n, unsigned t) { return (unsigned)((n + t - 1) / t); }

pf_status check_model(const Model& m) {
    PF_CHECK(m.d > 0 && m.d <= kMaxEmbd && m.n_heads > 0 && m.n_kv > 0 && m.hd > 0, "literal: bad model dimensions");
    PF_CHECK(m.n_heads * m.hd <= m.d && m.n_kv * m.hd <= m.d, "literal: heads x head_dim exceeds n_embd");
    PF_CHECK(m.hidden && m.q && m.k && m.v && m.attn_out && m.scores && m.self_p && m.skip_cache,
             "literal: work buffers missing");
    return PF_OK;
}

}  // namespace

pf_status embed(const Model& m, int32_t token, void* stream) {
    PF_TRY(require_device());
    PF_TRY(check_model(m));
    PF_CHECK(!m.emb_loaded || m.emb, "literal embed: table missing");
    embed_kernel<<<1, 256, 0, as_stream(stream)>>>(m, token);
    return launch_check("literal embed");
}

pf_status layer(const Model& m, uint32_t l, const Tiers& t, const Store& s, void* stream) {
    PF_TRY(require_device());
    PF_TRY(check_model(m));
    PF_CHECK(l < m.n_layers && m.attn_w && m.ffn_w && m.rope_cos && m.rope_sin, "literal layer: bad arguments");
    PF_CHECK(t.count() + 1 <= m.score_stride, "literal layer: %u cached entries exceed the score buffer", t.count());
    PF_CHECK(t.n_sink <= m.c.sink_cap && t.n_pool <= m.c.pool_cap && t.n_win <= m.c.ring && t.head < m.c.ring,
             "literal layer: tier counts exceed the cache");
    PF_CHECK(s.kind == 0 || (s.kind == 1 && s.slot < m.c.sink_cap) ||
                 (s.kind == 2 && s.slot < m.c.ring && (!s.finalize || (s.evict && s.pool_row < m.c.pool_cap))),
             "literal layer: bad store");
    cudaStream_t st = as_stream(stream);
    const size_t rows_smem = (size_t)2 * m.d * sizeof(float);
    const float scale = 1.0f / std::sqrt((float)m.hd);
    pre_attn_kernel<<<1, kRowThreads, rows_smem, st>>>(m, l);
    PF_TRY(launch_check("literal pre_attn"));
    if (t.count()) {
        scores_kernel<<<dim3(blocks(t.count(), kScoreThreads), m.n_heads), kScoreThreads, 0, st>>>(m, l, t, scale);
        PF_TRY(launch_check("literal scores"));
    }
    softmax_kernel<<<m.n_heads, kSoftmaxThreads, 0, st>>>(m, t, scale);
    PF_TRY(launch_check("literal softmax"));
    attn_out_kernel<<<1, 256, 0, st>>>(m, l, t);
    PF_TRY(launch_check("literal attn_out"));
    if (s.kind) {
        store_kernel<<<m.n_kv, kStoreThreads, m.hd * sizeof(float), st>>>(m, l, s);
        PF_TRY(launch_check("literal store"));
    }
    ffn_kernel<<<1, kRowThreads, rows_smem, st>>>(m, l);
    return launch_check("literal ffn");
}

pf_status unembed(const Model& m, const float* h, float* logits, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(m.emb && h && logits && m.d > 0 && m.d <= kMaxEmbd && m.n_vocab <= m.emb_rows,
             "literal unembed: bad arguments");
    const size_t smem = (size_t)m.d * sizeof(float) + (size_t)kUnembedRows * kTilePitch;
    unembed_kernel<<<blocks(m.n_vocab, kUnembedRows), kUnembedRows, smem, as_stream(stream)>>>(
        m.emb, m.emb_scale, h, m.d, m.n_vocab, logits);
    return launch_check("literal unembed");
}

pf_status placeholder_logits(int32_t token, uint32_t n_vocab, float* logits, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(logits, "literal placeholder_logits: null logits");
    if (n_vocab) placeholder_logits_kernel<<<blocks(n_vocab, 256), 256, 0, as_stream(stream)>>>(token, n_vocab, logits);
    return launch_check("literal placeholder_logits");
}

pf_status mtp_ffn(float* h, const uint8_t* gate, const float* gate_s, const uint8_t* up, const float* up_s,
                  const uint8_t* down, const float* down_s, uint32_t d, uint32_t ff, float* work, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(h && gate && gate_s && up && up_s && down && down_s && work && d && ff && d % 2 == 0 && ff % 2 == 0,
             "literal mtp_ffn: bad arguments");
    cudaStream_t st = as_stream(stream);
    float* g = work;
    float* u = work + ff;
    float* a = work + 2 * ff;  // activations, then (first d entries) the down projection
    q4_rows_kernel<<<blocks(ff, 128), 128, 0, st>>>(h, gate, gate_s, g, ff, d);
    q4_rows_kernel<<<blocks(ff, 128), 128, 0, st>>>(h, up, up_s, u, ff, d);
    silu_mul_kernel<<<blocks(ff, 256), 256, 0, st>>>(g, u, a, ff);
    q4_rows_kernel<<<blocks(d, 128), 128, 0, st>>>(a, down, down_s, g, d, ff);
    add_kernel<<<blocks(d, 256), 256, 0, st>>>(h, g, d);
    return launch_check("literal mtp_ffn");
}

}  // namespace lit
}  // namespace pf

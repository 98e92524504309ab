// forge_compat.cu — device kernels behind the forge:: compatibility classes
// (include/forge/*.hpp): the single-vector operations of the reference's
// MTPHeads, KVCache and LayerSkipController, one call at a time.  They keep the
// reference's summation order (one thread runs a row's loop in sequence), so
// their results are the reference's to the bit wherever the reference's own
// arithmetic is plain float multiply-add.
#include "common.cuh"

namespace pf {
namespace {

__device__ __forceinline__ float mul_add(float s, float a, float b) { return __fadd_rn(s, __fmul_rn(a, b)); }

__global__ void dot_kernel(const float* __restrict__ a, const float* __restrict__ b, uint32_t n, float* out) {
    float s = 0.0f;  // src/matmul_neon.cpp:186-207, in index order
    for (uint32_t i = 0; i < n; i++) s = mul_add(s, a[i], b[i]);
    *out = s;
}

// y[r] = sum_i x[i] * ((nibble_i - 8) * scale[r]) over a row packed two
// values per byte, low nibble first (MTPHeads::dequant_q4_row, src/mtp.cpp).
__global__ void gemv_q4_kernel(const float* __restrict__ x, const uint8_t* __restrict__ w,
                               const float* __restrict__ scale, float* __restrict__ y, uint32_t rows, uint32_t cols) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const uint8_t* wr = w + (size_t)r * (cols / 2);
    const float sc = scale[r];
    float s = 0.0f;
    for (uint32_t i = 0; i < cols; i += 2) {
        const uint8_t b = wr[i / 2];
        s = mul_add(s, x[i], __fmul_rn((float)((int)(b & 0x0F) - 8), sc));
        if (i + 1 < cols) s = mul_add(s, x[i + 1], __fmul_rn((float)((int)(b >> 4) - 8), sc));
    }
    y[r] = s;
}

__global__ void gemv_f32_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ y,
                                uint32_t rows, uint32_t cols) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const float* wr = w + (size_t)r * cols;
    float s = 0.0f;
    for (uint32_t i = 0; i < cols; i++) s = mul_add(s, x[i], wr[i]);
    y[r] = s;
}

// a = silu(g) * u with silu(x) = x / (1 + exp(-x)) (src/mtp.cpp); then the
// residual h += o is a separate launch after the down projection.  The
// exponential is the double one rounded to float (the correctly rounded value).
__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ a,
                                uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) a[i] = __fmul_rn(__fdiv_rn(g[i], __fadd_rn(1.0f, (float)exp((double)-g[i]))), u[i]);
}
__global__ void vec_add_kernel(float* __restrict__ y, const float* __restrict__ x, uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __fadd_rn(y[i], x[i]);
}
// Logits of an MTP head without an embedding table (src/mtp.cpp:118-123).
__global__ void placeholder_logits_kernel(float* __restrict__ logits, uint32_t vocab, uint32_t head) {
    const uint32_t v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v < vocab)
        logits[v] = (float)(((uint64_t)v * 2654435761ULL + (uint64_t)head) % vocab) / (float)vocab;
}

// sqrt(sum (a-b)^2 / n) in index order (LayerSkipController::hidden_delta).
__global__ void skip_delta_kernel(const float* __restrict__ a, const float* __restrict__ b, uint32_t n, float* out) {
    float s = 0.0f;
    for (uint32_t i = 0; i < n; i++) {
        const float d = __fsub_rn(a[i], b[i]);
        s = mul_add(s, d, d);
    }
    *out = __fsqrt_rn(__fdiv_rn(s, (float)n));
}

// KVCache::quantize_row (src/kv_cache.cpp:19-28) of one hd-vector by one
// block: amax, scale = amax/127 (1 for zero rows), q = round(x*127/amax).
__device__ void quant_vec_block(const float* x, uint32_t hd, int8_t* q, float* scale, float* red) {
    float m = 0.0f;
    for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) m = fmaxf(m, fabsf(x[i]));
    red[threadIdx.x] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.0f;
        for (uint32_t t = 0; t < blockDim.x; t++) a = fmaxf(a, red[t]);
        red[blockDim.x] = a;
    }
    __syncthreads();
    const float amax = red[blockDim.x];
    const float mul = amax == 0.0f ? 1.0f : __fdiv_rn(127.0f, amax);
    for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) q[i] = (int8_t)(int)roundf(__fmul_rn(x[i], mul));
    if (threadIdx.x == 0) *scale = amax == 0.0f ? 1.0f : __fdiv_rn(amax, 127.0f);
    __syncthreads();
}

// One KVCache::store into a window slot (src/kv_cache.cpp:59-127): if the
// slot held an entry, add it (dequantized, in double) to the pooling
// accumulators; if that completes a pool block, write the mean as the next
// pool entry and clear the accumulators; then quantize the new key / value
// into the slot.  Sink stores pass no eviction.
struct KvuStore {
    const float* k;
    const float* v;
    uint32_t hd;
    int8_t *dk, *dv;
    float *dks, *dvs;
    const int8_t *ek, *ev;  // evicted slot contents (null: nothing evicted)
    const float *eks, *evs;
    double *acc_k, *acc_v;
    uint32_t acc_n;  // accumulated entries after this eviction
    int finalize;    // acc_n reached the pool block
    int8_t *pk, *pv;
    float *pks, *pvs;
};
__global__ void kvu_store_kernel(KvuStore a) {
    extern __shared__ float sh[];  // [hd] mean + [blockDim + 1] reduction
    float* mean = sh;
    float* red = sh + a.hd;
    if (a.ek) {
        for (uint32_t i = threadIdx.x; i < a.hd; i += blockDim.x) {
            a.acc_k[i] += (double)a.ek[i] * (double)*a.eks;
            a.acc_v[i] += (double)a.ev[i] * (double)*a.evs;
        }
        __syncthreads();
        if (a.finalize) {
            const float inv = 1.0f / (float)a.acc_n;
            for (uint32_t i = threadIdx.x; i < a.hd; i += blockDim.x) mean[i] = (float)(a.acc_k[i] * (double)inv);
            __syncthreads();
            quant_vec_block(mean, a.hd, a.pk, a.pks, red);
            for (uint32_t i = threadIdx.x; i < a.hd; i += blockDim.x) mean[i] = (float)(a.acc_v[i] * (double)inv);
            __syncthreads();
            quant_vec_block(mean, a.hd, a.pv, a.pvs, red);
            for (uint32_t i = threadIdx.x; i < a.hd; i += blockDim.x) a.acc_k[i] = a.acc_v[i] = 0.0;
            __syncthreads();
        }
    }
    quant_vec_block(a.k, a.hd, a.dk, a.dks, red);
    quant_vec_block(a.v, a.hd, a.dv, a.dvs, red);
}

// Entries of one unit in attention order: sink [0, ns), pool [0, np), window
// oldest first (ring slot (head + i) % ring once the ring is full).
struct KvuView {
    const int8_t *sk, *sv, *pk, *pv, *wk, *wv;
    const float *sks, *svs, *pks, *pvs, *wks, *wvs;
    uint32_t hd, ns, np, nw, ring, head;
};
__device__ __forceinline__ void kvu_entry(const KvuView& u, uint32_t e, const int8_t*& k, float& ks, const int8_t*& v,
                                          float& vs) {
    if (e < u.ns) {
        k = u.sk + (size_t)e * u.hd; v = u.sv + (size_t)e * u.hd; ks = u.sks[e]; vs = u.svs[e];
        return;
    }
    e -= u.ns;
    if (e < u.np) {
        k = u.pk + (size_t)e * u.hd; v = u.pv + (size_t)e * u.hd; ks = u.pks[e]; vs = u.pvs[e];
        return;
    }
    e -= u.np;
    const uint32_t s = u.nw < u.ring ? e : (u.head + e) % u.ring;
    k = u.wk + (size_t)s * u.hd; v = u.wv + (size_t)s * u.hd; ks = u.wks[s]; vs = u.wvs[s];
}
// KVCache::attention_scores (src/kv_cache.cpp:129-158): q . (k * scale).
__global__ void kvu_scores_kernel(KvuView u, const float* __restrict__ q, float* __restrict__ out) {
    const uint32_t e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= u.ns + u.np + u.nw) return;
    const int8_t *k, *v;
    float ks, vs;
    kvu_entry(u, e, k, ks, v, vs);
    float s = 0.0f;
    for (uint32_t i = 0; i < u.hd; i++) s = mul_add(s, q[i], __fmul_rn((float)k[i], ks));
    out[e] = s;
}
// KVCache::attention_weighted_sum (src/kv_cache.cpp:160-198): sum_e p_e * (v_e * scale_e).
__global__ void kvu_wsum_kernel(KvuView u, const float* __restrict__ p, uint32_t cnt, float* __restrict__ out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= u.hd) return;
    float s = 0.0f;
    for (uint32_t e = 0; e < cnt; e++) {
        const int8_t *k, *v;
        float ks, vs;
        kvu_entry(u, e, k, ks, v, vs);
        s = mul_add(s, p[e], __fmul_rn((float)v[i], vs));
    }
    out[i] = s;
}

inline unsigned blocks_for(uint32_t n, unsigned t) { return (unsigned)((n + t - 1) / t); }

}  // namespace
}  // namespace pf

using namespace pf;

extern "C" {

pf_status pf_dot_f32(const float* a, const float* b, uint32_t n, float* out, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(a && b && out, "pf_dot_f32: null argument");
    dot_kernel<<<1, 1, 0, as_stream(stream)>>>(a, b, n, out);
    return launch_check("pf_dot_f32");
}

pf_status pf_gemv_q4_rows(const float* x, const uint8_t* w, const float* scale, float* y, uint32_t rows, uint32_t cols,
                          void* stream) {
    PF_TRY(require_device());
    PF_CHECK(x && w && scale && y && rows && cols, "pf_gemv_q4_rows: bad arguments");
    gemv_q4_kernel<<<blocks_for(rows, 128), 128, 0, as_stream(stream)>>>(x, w, scale, y, rows, cols);
    return launch_check("pf_gemv_q4_rows");
}

pf_status pf_gemv_f32_rows(const float* x, const float* w, float* y, uint32_t rows, uint32_t cols, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(x && w && y && rows && cols, "pf_gemv_f32_rows: bad arguments");
    gemv_f32_kernel<<<blocks_for(rows, 128), 128, 0, as_stream(stream)>>>(x, w, y, rows, cols);
    return launch_check("pf_gemv_f32_rows");
}

pf_status pf_mtp_silu_mul(const float* g, const float* u, float* a, uint32_t n, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(g && u && a, "pf_mtp_silu_mul: null argument");
    if (n) silu_mul_kernel<<<blocks_for(n, 256), 256, 0, as_stream(stream)>>>(g, u, a, n);
    return launch_check("pf_mtp_silu_mul");
}

pf_status pf_vec_add(float* y, const float* x, uint32_t n, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(y && x, "pf_vec_add: null argument");
    if (n) vec_add_kernel<<<blocks_for(n, 256), 256, 0, as_stream(stream)>>>(y, x, n);
    return launch_check("pf_vec_add");
}

pf_status pf_mtp_placeholder_logits(float* logits, uint32_t vocab, uint32_t head, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(logits, "pf_mtp_placeholder_logits: null argument");
    if (vocab) placeholder_logits_kernel<<<blocks_for(vocab, 256), 256, 0, as_stream(stream)>>>(logits, vocab, head);
    return launch_check("pf_mtp_placeholder_logits");
}

pf_status pf_skip_delta(const float* a, const float* b, uint32_t n, float* out, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(a && b && out && n, "pf_skip_delta: bad arguments");
    skip_delta_kernel<<<1, 1, 0, as_stream(stream)>>>(a, b, n, out);
    return launch_check("pf_skip_delta");
}

pf_status pf_kvu_store(const float* k, const float* v, uint32_t hd, int8_t* dk, float* dks, int8_t* dv, float* dvs,
                       const int8_t* ek, const float* eks, const int8_t* ev, const float* evs, double* acc_k,
                       double* acc_v, uint32_t acc_n, int32_t finalize, int8_t* pk, float* pks, int8_t* pv, float* pvs,
                       void* stream) {
    PF_TRY(require_device());
    PF_CHECK(k && v && dk && dks && dv && dvs && hd > 0 && hd <= 4096, "pf_kvu_store: bad arguments");
    PF_CHECK(!ek || (eks && ev && evs && acc_k && acc_v && acc_n > 0), "pf_kvu_store: incomplete eviction");
    PF_CHECK(!finalize || (ek && pk && pks && pv && pvs), "pf_kvu_store: incomplete pool entry");
    KvuStore a{k, v, hd, dk, dv, dks, dvs, ek, ev, eks, evs, acc_k, acc_v, acc_n, finalize, pk, pv, pks, pvs};
    const unsigned t = 128;
    kvu_store_kernel<<<1, t, (hd + t + 1) * sizeof(float), as_stream(stream)>>>(a);
    return launch_check("pf_kvu_store");
}

pf_status pf_kvu_scores(const int8_t* const* tier_k, const float* const* tier_ks, const uint32_t* counts,
                        uint32_t ring, uint32_t head, uint32_t hd, const float* q, float* out, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(tier_k && tier_ks && counts && q && out && hd, "pf_kvu_scores: bad arguments");
    KvuView u{tier_k[0], nullptr, tier_k[1], nullptr, tier_k[2], nullptr,
              tier_ks[0], nullptr, tier_ks[1], nullptr, tier_ks[2], nullptr,
              hd, counts[0], counts[1], counts[2], ring, head};
    const uint32_t n = counts[0] + counts[1] + counts[2];
    if (n) kvu_scores_kernel<<<blocks_for(n, 128), 128, 0, as_stream(stream)>>>(u, q, out);
    return launch_check("pf_kvu_scores");
}

pf_status pf_kvu_weighted_sum(const int8_t* const* tier_v, const float* const* tier_vs, const uint32_t* counts,
                              uint32_t ring, uint32_t head, uint32_t hd, const float* p, uint32_t cnt, float* out,
                              void* stream) {
    PF_TRY(require_device());
    PF_CHECK(tier_v && tier_vs && counts && p && out && hd, "pf_kvu_weighted_sum: bad arguments");
    KvuView u{nullptr, tier_v[0], nullptr, tier_v[1], nullptr, tier_v[2],
              nullptr, tier_vs[0], nullptr, tier_vs[1], nullptr, tier_vs[2],
              hd, counts[0], counts[1], counts[2], ring, head};
    const uint32_t n = counts[0] + counts[1] + counts[2];
    kvu_wsum_kernel<<<blocks_for(hd, 128), 128, 0, as_stream(stream)>>>(u, p, cnt < n ? cnt : n, out);
    return launch_check("pf_kvu_weighted_sum");
}

}  // extern "C"

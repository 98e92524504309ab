// kv_cache.cpp — forge::KVCache with its tiers in device memory (behaviour
// of the reference's src/kv_cache.cpp:32-198).  The host keeps each unit's
// counters (which slot a store fills, when an eviction completes a pool
// block); the device kernels (pf_kvu_*) quantize, pool and score.
#include "forge/kv_cache.hpp"

#include <algorithm>

#include "device.hpp"

namespace forge {

struct KVCache::Impl {
    struct Unit {  // one (layer, kv head)
        uint32_t n_sink = 0, head = 0, n_win = 0, n_pool = 0, n_acc = 0;
    };
    KVCacheConfig cfg;
    uint32_t hd = 0, ring = 0, sink_cap = 0, pool_cap = 0, pool_block = 1;
    // Device arrays, all units back to back: [unit][rows][hd] int8 and [unit][rows] fp32.
    dev::Buffer sk, sv, sks, svs, wk, wv, wks, wvs, pk, pv, pks, pvs, ak, av;
    dev::Buffer stage;  // key | value | query / scores / output staging
    std::vector<Unit> units;
    size_t bytes = 0;

    size_t unit(uint32_t l, uint32_t h) const { return (size_t)l * cfg.n_kv_heads + h; }
    template <class T>
    T* at(const dev::Buffer& b, size_t u, size_t rows, size_t row, size_t width) const {
        return b.as<T>() + (u * rows + row) * width;
    }
};

KVCache::KVCache(const KVCacheConfig& cfg) : impl_(new Impl) {
    Impl& m = *impl_;
    m.cfg = cfg;
    m.hd = cfg.head_dim;
    m.ring = std::max(1u, std::min(cfg.window_size, cfg.max_context));
    m.sink_cap = cfg.sink_size;
    m.pool_block = std::max(1u, cfg.pool_block);
    const uint32_t evictable = cfg.max_context > cfg.sink_size + m.ring ? cfg.max_context - cfg.sink_size - m.ring : 0;
    m.pool_cap = evictable / m.pool_block + 1;
    const size_t U = (size_t)cfg.n_layers * cfg.n_kv_heads, hd = m.hd;
    auto alloc = [&](dev::Buffer& b, size_t bytes) {
        if (b.reserve(bytes + 16)) {
            cudaMemset(b.as<void>(), 0, bytes);
            m.bytes += bytes;
        }
    };
    alloc(m.sk, U * m.sink_cap * hd);
    alloc(m.sv, U * m.sink_cap * hd);
    alloc(m.sks, U * m.sink_cap * 4);
    alloc(m.svs, U * m.sink_cap * 4);
    alloc(m.wk, U * m.ring * hd);
    alloc(m.wv, U * m.ring * hd);
    alloc(m.wks, U * m.ring * 4);
    alloc(m.wvs, U * m.ring * 4);
    alloc(m.pk, U * m.pool_cap * hd);
    alloc(m.pv, U * m.pool_cap * hd);
    alloc(m.pks, U * m.pool_cap * 4);
    alloc(m.pvs, U * m.pool_cap * 4);
    alloc(m.ak, U * hd * 8);
    alloc(m.av, U * hd * 8);
    m.stage.reserve(((size_t)2 * hd + std::max<size_t>(hd, (size_t)m.sink_cap + m.pool_cap + m.ring)) * 4 + 64);
    m.units.assign(U, Impl::Unit{});
}

KVCache::~KVCache() = default;

void KVCache::store(uint32_t layer, uint32_t head, uint32_t pos, const float* key, const float* value) {
    Impl& m = *impl_;
    if (layer >= m.cfg.n_layers || head >= m.cfg.n_kv_heads || pos >= m.cfg.max_context) return;
    const size_t u = m.unit(layer, head), hd = m.hd;
    Impl::Unit& c = m.units[u];
    float* k = m.stage.as<float>();
    float* v = k + hd;
    if (!dev::to_dev(k, key, hd * 4, "KVCache::store") || !dev::to_dev(v, value, hd * 4, "KVCache::store")) return;
    if (pos < m.cfg.sink_size) {
        if (!dev::ok(pf_kvu_store(k, v, m.hd, m.at<int8_t>(m.sk, u, m.sink_cap, pos, hd),
                                  m.at<float>(m.sks, u, m.sink_cap, pos, 1), m.at<int8_t>(m.sv, u, m.sink_cap, pos, hd),
                                  m.at<float>(m.svs, u, m.sink_cap, pos, 1), nullptr, nullptr, nullptr, nullptr,
                                  nullptr, nullptr, 0, 0, nullptr, nullptr, nullptr, nullptr, nullptr),
                     "KVCache::store"))
            return;
        c.n_sink = std::max(c.n_sink, pos + 1);
    } else {
        const uint32_t slot = c.head;
        const bool evict = c.n_win >= m.ring;
        bool finalize = false;
        uint32_t acc_n = 0, pool_row = 0;
        if (evict) {
            acc_n = c.n_acc + 1;
            finalize = acc_n >= m.pool_block && c.n_pool < m.pool_cap;
            pool_row = c.n_pool;
        }
        int8_t* dk = m.at<int8_t>(m.wk, u, m.ring, slot, hd);
        int8_t* dv = m.at<int8_t>(m.wv, u, m.ring, slot, hd);
        float* dks = m.at<float>(m.wks, u, m.ring, slot, 1);
        float* dvs = m.at<float>(m.wvs, u, m.ring, slot, 1);
        if (!dev::ok(pf_kvu_store(k, v, m.hd, dk, dks, dv, dvs, evict ? dk : nullptr, evict ? dks : nullptr,
                                  evict ? dv : nullptr, evict ? dvs : nullptr, m.at<double>(m.ak, u, 1, 0, hd),
                                  m.at<double>(m.av, u, 1, 0, hd), acc_n, finalize ? 1 : 0,
                                  m.at<int8_t>(m.pk, u, m.pool_cap, pool_row, hd),
                                  m.at<float>(m.pks, u, m.pool_cap, pool_row, 1),
                                  m.at<int8_t>(m.pv, u, m.pool_cap, pool_row, hd),
                                  m.at<float>(m.pvs, u, m.pool_cap, pool_row, 1), nullptr),
                     "KVCache::store"))
            return;
        if (evict) {
            c.n_acc = finalize ? 0 : acc_n;
            if (finalize) c.n_pool++;
        } else {
            c.n_win++;
        }
        c.head = (c.head + 1) % m.ring;
    }
    total_stored_ = std::max(total_stored_, pos + 1);
}

uint32_t KVCache::attention_scores(uint32_t layer, uint32_t head, const float* query, float* scores_out) {
    Impl& m = *impl_;
    if (layer >= m.cfg.n_layers || head >= m.cfg.n_kv_heads) return 0;
    const size_t u = m.unit(layer, head), hd = m.hd;
    const Impl::Unit& c = m.units[u];
    const uint32_t counts[3] = {c.n_sink, c.n_pool, c.n_win};
    const uint32_t n = counts[0] + counts[1] + counts[2];
    const int8_t* tk[3] = {m.at<int8_t>(m.sk, u, m.sink_cap, 0, hd), m.at<int8_t>(m.pk, u, m.pool_cap, 0, hd),
                           m.at<int8_t>(m.wk, u, m.ring, 0, hd)};
    const float* ts[3] = {m.at<float>(m.sks, u, m.sink_cap, 0, 1), m.at<float>(m.pks, u, m.pool_cap, 0, 1),
                          m.at<float>(m.wks, u, m.ring, 0, 1)};
    float* q = m.stage.as<float>();
    float* out = q + 2 * hd;
    if (n == 0 || !dev::to_dev(q, query, hd * 4, "KVCache::attention_scores")) return 0;
    if (!dev::ok(pf_kvu_scores(tk, ts, counts, m.ring, c.head, m.hd, q, out, nullptr), "KVCache::attention_scores"))
        return 0;
    if (!dev::to_host(scores_out, out, (size_t)n * 4, "KVCache::attention_scores")) return 0;
    return n;
}

void KVCache::attention_weighted_sum(uint32_t layer, uint32_t head, const float* scores, float* output,
                                     uint32_t count) {
    Impl& m = *impl_;
    if (layer >= m.cfg.n_layers || head >= m.cfg.n_kv_heads) return;
    const size_t u = m.unit(layer, head), hd = m.hd;
    const Impl::Unit& c = m.units[u];
    const uint32_t counts[3] = {c.n_sink, c.n_pool, c.n_win};
    const uint32_t n = std::min(count, counts[0] + counts[1] + counts[2]);
    const int8_t* tv[3] = {m.at<int8_t>(m.sv, u, m.sink_cap, 0, hd), m.at<int8_t>(m.pv, u, m.pool_cap, 0, hd),
                           m.at<int8_t>(m.wv, u, m.ring, 0, hd)};
    const float* ts[3] = {m.at<float>(m.svs, u, m.sink_cap, 0, 1), m.at<float>(m.pvs, u, m.pool_cap, 0, 1),
                          m.at<float>(m.wvs, u, m.ring, 0, 1)};
    float* out = m.stage.as<float>();
    float* p = out + 2 * hd;
    if (n > 0 && !dev::to_dev(p, scores, (size_t)n * 4, "KVCache::attention_weighted_sum")) return;
    if (!dev::ok(pf_kvu_weighted_sum(tv, ts, counts, m.ring, c.head, m.hd, p, n, out, nullptr),
                 "KVCache::attention_weighted_sum"))
        return;
    dev::to_host(output, out, hd * 4, "KVCache::attention_weighted_sum");
}

void KVCache::clear() {
    Impl& m = *impl_;
    std::fill(m.units.begin(), m.units.end(), Impl::Unit{});
    const size_t U = m.units.size();
    if (m.ak.as<void>()) cudaMemset(m.ak.as<void>(), 0, U * m.hd * 8);
    if (m.av.as<void>()) cudaMemset(m.av.as<void>(), 0, U * m.hd * 8);
    total_stored_ = 0;
}

size_t KVCache::memory_usage() const { return impl_->bytes; }

}  // namespace forge

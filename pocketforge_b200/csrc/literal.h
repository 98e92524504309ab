// literal.h — device side of forge::Engine's reference-compat mode: the
// reference's literal single-token forward (src/engine.cpp:459-589 with
// compute_attention :600-801 and compute_ffn :807-854 on their placeholder
// branches), one launch per phase of a layer.
//
// Every kernel keeps the reference's float operation order (one thread runs a
// reduction loop in the reference's index order, products and sums rounded
// one at a time), so results are the reference's to the bit except where it
// calls std::exp: the device rounds the double exponential to float, which
// can differ from glibc's expf by one unit in the last place.
//
// Plain C++ (no CUDA types) so that the host half (forge/literal.cpp) builds
// with the host compiler.
#pragma once
#include <cstdint>

#include "../../include/pf_b200.h"

#ifdef __CUDACC__
#define PF_LIT_HD __host__ __device__
#else
#define PF_LIT_HD
#endif

namespace pf {
namespace lit {

// The KV tiers of every (layer, kv head) unit, back to back (unit = layer *
// n_kv_heads + kv head), as the reference's KVCache keeps them per unit
// (src/kv_cache.cpp:32-57): 8 sink rows, a ring of `ring` window rows, a
// growing list of pooled rows, and the fp64 pooling accumulators.
struct Cache {
    int8_t *sk = nullptr, *sv = nullptr;  // [U][sink_cap][hd]
    float *sks = nullptr, *svs = nullptr; // [U][sink_cap]
    int8_t *wk = nullptr, *wv = nullptr;  // [U][ring][hd]
    float *wks = nullptr, *wvs = nullptr; // [U][ring]
    int8_t *pk = nullptr, *pv = nullptr;  // [U][pool_cap][hd]
    float *pks = nullptr, *pvs = nullptr; // [U][pool_cap]
    double *ak = nullptr, *av = nullptr;  // [U][hd]
    uint32_t sink_cap = 8, ring = 1, pool_cap = 0;
};

// One layer's tier counts before this forward's store.  Every store of the
// literal forward writes all kv heads of a layer at the same position (the
// layer index), so the heads of a layer always hold the same counts.
struct Tiers {
    uint32_t n_sink = 0, n_pool = 0, n_win = 0, head = 0;
    PF_LIT_HD uint32_t count() const { return n_sink + n_pool + n_win; }
};

// What this forward's KVCache::store does at one layer (src/kv_cache.cpp:59-127).
struct Store {
    int32_t kind = 0;      // 0: nothing stored, 1: sink row `slot`, 2: window row `slot`
    uint32_t slot = 0;
    int32_t evict = 0;     // the window row held an entry: add it to the accumulators
    uint32_t acc_n = 0;    // accumulated entries after that
    int32_t finalize = 0;  // acc_n reached the pool block: the mean becomes pool row `pool_row`
    uint32_t pool_row = 0;
};

struct Model {
    uint32_t n_layers = 0, d = 0, n_heads = 0, n_kv = 0, hd = 0, n_vocab = 0;
    uint32_t emb_rows = 0;           // rows of the embedding table (min(n_vocab, 16384))
    const int8_t* emb = nullptr;     // [emb_rows][d] int8, value = int8 * emb_scale
    float emb_scale = 1.0f;
    int32_t emb_loaded = 0;
    const float* attn_w = nullptr;   // [n_layers][d] attention RMSNorm weights
    const float* ffn_w = nullptr;    // [n_layers][d]
    const float* rope_cos = nullptr; // [n_layers][hd]: the table at position = layer index
    const float* rope_sin = nullptr;
    Cache c;
    // Work buffers (device): hidden, normed [d]; q, k, v, attn_out [d];
    // scores [n_heads][score_stride]; self_p [n_heads]; skip_cache [n_layers][d].
    float *hidden = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn_out = nullptr;
    float *scores = nullptr, *self_p = nullptr, *skip_cache = nullptr;
    uint32_t score_stride = 0;
    // LayerSkipController (src/layer_skip.cpp:21-67): threshold and whether
    // every token is an anchor (skip_interval == 0).
    float skip_threshold = 0.01f;
    int32_t skip_anchor = 0;
};

// Largest n_embd the one-block phases take (two float rows in shared memory).
constexpr uint32_t kMaxEmbd = 4096;

// hidden = embedding row of `token` (or zeros past the table), or the
// reference's placeholder embedding when no table is loaded (src/engine.cpp:474-491).
pf_status embed(const Model& m, int32_t token, void* stream);
// Layer `l`: RMSNorm, placeholder Q = K = V = 0.1 x normed, RoPE at the layer
// index (K rotated once per query head), attention over the cached tiers plus
// the float self term, head outputs as the reference writes them (slot 0 holds
// the last head's cached sum), residual, the store of K/V into the tiers, then
// RMSNorm, the layer-skip decision and the placeholder FFN.
pf_status layer(const Model& m, uint32_t l, const Tiers& t, const Store& s, void* stream);
// Tied unembedding of h (src/engine.cpp:571-583; MTP heads src/mtp.cpp:106-116):
// logits[v] = sum_i h[i] * (E[v][i] * scale) in index order.
pf_status unembed(const Model& m, const float* h, float* logits, void* stream);
// The reference's placeholder logits of `token` (src/engine.cpp:592-597).
pf_status placeholder_logits(int32_t token, uint32_t n_vocab, float* logits, void* stream);
// One MTP head FFN on h in place (src/mtp.cpp:66-104): gate and up rows of
// Q4 weights (rows x cols packed two per byte, low nibble first), SiLU(gate) * up,
// the down projection and the residual.  `work` holds 3 * ff floats.
pf_status mtp_ffn(float* h, const uint8_t* gate, const float* gate_s, const uint8_t* up, const float* up_s,
                  const uint8_t* down, const float* down_s, uint32_t d, uint32_t ff, float* work, void* stream);

}  // namespace lit
}  // namespace pf

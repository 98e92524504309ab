// kv.cuh — device layout of the 3-tier int8 KV cache and of a row batch.
//
// The reference keeps, per (layer, kv head), a sink of the first 4
// positions, a circular window of the last W positions and a pool of
// 64-entry means of evicted window entries accumulated in double
// (src/kv_cache.cpp:59-127).  Here every (sequence, layer, kv head) "unit"
// owns the same three tiers in HBM, addressed by position instead of by a
// moving head pointer:
//   window-tier position p (p >= S) lives in ring slot (p - S) % Wr,
//   Wr = min(window_size, max_context) (KVCache::window_sz_);
//   after positions [0, L) are stored, E(L) = max(0, L - S - Wr) entries have
//   been evicted and floor(E/pb) pool entries finalized.
// Ring slots are allocated only up to the positions a sequence can reach.
#pragma once
#include "common.cuh"

namespace pf {

// K rows are stored entry-major ([slot][64]).  V is stored dim-major per block
// of 32 slots: block b holds [64 dims][32 bytes] and the byte of slot
// 32b + i sits at position kv_vpos(i) of its dim row — the order in which the
// tensor-core attention consumes entries (attn_decode.cu).
struct KvCache {
    int n_seqs = 0, L = 0, G = 0, hd = 64;
    int S = 4, Wr = 0, W_alloc = 0, P_max = 0, pb = 64, max_pos = 0;
    int W_pad = 0, P_pad = 0;                     // W_alloc, P_max rounded up to 32
    int8_t *ring_k = nullptr, *ring_v = nullptr;  // [unit][W_pad][hd] (V in blocks, see above)
    float *ring_ks = nullptr, *ring_vs = nullptr; // [unit][W_pad]
    int8_t *sink_k = nullptr, *sink_v = nullptr;  // [unit][S][hd] entry-major
    float *sink_ks = nullptr, *sink_vs = nullptr;
    int8_t *pool_k = nullptr, *pool_v = nullptr;  // [unit][P_pad][hd] (V in blocks)
    float *pool_ks = nullptr, *pool_vs = nullptr;
    double *acc_k = nullptr, *acc_v = nullptr;    // [unit][hd]
    __host__ __device__ size_t unit(int seq, int layer, int g) const {
        return ((size_t)seq * L + layer) * G + g;
    }
};

__host__ __device__ inline int kv_vpos(int i) { return ((i & 7) >> 1) * 8 + (i >> 3) * 2 + (i & 1); }
// Byte offset of (entry e, dim d) inside a [n][64] V array stored in blocks.
__host__ __device__ inline size_t kv_voff(size_t e, int d) {
    return (e >> 5) * 2048 + (size_t)d * 32 + kv_vpos((int)(e & 31));
}

__host__ __device__ inline int kv_pool_count(int len, int S, int Wr, int pb) {
    const int e = len - S - Wr;
    return e > 0 ? e / pb : 0;
}

// A batch of rows: rows of sequence b are [row0[b], row0[b] + n[b]) at
// positions len0[b] + r.  Sequences with n[b] == 0 take no part.
struct RowBatch {
    int nb = 0;          // sequences (== engine sequences)
    int M = 0;           // total rows
    const int* row0 = nullptr;
    const int* n = nullptr;
    const int* len0 = nullptr;
    const int* row_pos = nullptr;  // [M]
    int max_rows = 0;    // upper bound of n[b]
};

// Staged K/V of the rows of one layer (quantized like KVCache::store does).
struct Staged {
    int8_t *k = nullptr, *v = nullptr;  // [M][G][hd]
    float *ks = nullptr, *vs = nullptr; // [M][G]
};

// Speculative pool entries a batch finalizes part-way (one layer).
struct SpecPool {
    int per = 0;                        // slots per (seq, g)
    int8_t *k = nullptr, *v = nullptr;  // [nb][G][per][hd]
    float *ks = nullptr, *vs = nullptr; // [nb][G][per]
};

pf_status kv_quant_rows(const float* qkv, int ldqkv, int k_col, int v_col, int M, const int* m_dev, int G, int hd,
                        Staged st, cudaStream_t stream);
pf_status kv_pool_spec(const KvCache& kv, int layer, const RowBatch& rb, SpecPool sp, cudaStream_t stream);
// The QKV projection from K-split int32 slices ([n_parts][M][N] at part_stride):
// scales, RoPE on columns [0, rope_cols), the fp32 rows into qkv (row stride
// N), and the staged K/V of every kv head (as kv_quant_rows).
pf_status qkv_finish(const int32_t* parts, int n_parts, int64_t part_stride, const float* a_s, const float* w_s,
                     int N, int M, const float* rope_cos, const float* rope_sin, const int* row_pos, int rope_cols,
                     int hd, float* qkv, int k_col, int v_col, int G, Staged st, cudaStream_t stream);
pf_status attention(const KvCache& kv, int layer, const RowBatch& rb, const float* qkv, int ldqkv, int k_col,
                    int v_col, int H, Staged st, SpecPool sp, float* out, int ldo, cudaStream_t stream);
// Tensor-core variant: one CTA per (sequence, kv head, group of 32 / (H/G)
// rows of the sequence), for batches whose sink, in-batch pool entries and
// earlier rows fit four 32-entry blocks.  The context of each (sequence, kv
// head, row group) is split over `nsplit` CTAs whose partial softmax states
// meet in `part`; `cnt` ([nb][G][row groups] ints, zero before the first
// launch) counts the arrivals and is left zero.
struct AttnWork {
    int nsplit = 1;
    float* part = nullptr;
    size_t part_floats = 0;
    int* cnt = nullptr;
    size_t cnt_elems = 0;
};
bool attention_decode_supported(const KvCache& kv, int H, int max_rows);
// Sequence rows one attention CTA takes (a batch's rows per sequence split
// into row groups of this many).
int attention_decode_rows_per_cta(const KvCache& kv, int H);
int attention_decode_splits(int nb, int G, int max_splits);
int attention_decode_row_groups(const KvCache& kv, int H, int max_rows);
size_t attention_decode_work_floats(int nb, int G, int nsplit, int nrg);
pf_status attention_decode(const KvCache& kv, int layer, const RowBatch& rb, const float* qkv, int ldqkv, int k_col,
                           int v_col, int H, Staged st, SpecPool sp, const AttnWork& aw, float* out, int ldo,
                           cudaStream_t stream);
// Commits rows [0, n_commit[b]) of every sequence into the cache, all layers.
// `staged` holds layer 0; layer l is at +l*M*G*hd (int8) and +l*M*G (scales).
pf_status kv_commit(const KvCache& kv, const RowBatch& rb, const int* n_commit, Staged staged, int M_stride,
                    cudaStream_t stream);

}  // namespace pf

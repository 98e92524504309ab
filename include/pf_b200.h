/*
 * pf_b200.h — C ABI of the B200 (sm_100a) implementation of PocketForge's MTP
 * speculative-decode step.
 *
 * Conventions
 *   - Plain pointers and sizes; no C++ or torch types cross this boundary.
 *   - Kernel-level entry points (pf_* below "Kernel-level") take CALLER-OWNED
 *     DEVICE pointers and a cudaStream_t passed as `void*` (NULL = legacy
 *     default stream).  They enqueue work and return without synchronising.
 *   - Engine-level entry points (pf_engine_*) own their device memory; their
 *     token / prompt arguments are HOST pointers.
 *   - Every entry point returns pf_status (0 = PF_OK).  The last error text of
 *     the calling thread is available from pf_last_error().
 *   - There is no CPU fallback: when no sm_100 device is present, every
 *     entry point that would launch a kernel returns PF_ERR_NO_DEVICE.
 *
 * Each declaration cites the reference interface it replaces (file:line in
 * tundefund0-gif/pocketforge).  The reference has no FFI of its own: its
 * interface is the C++ headers under include/forge/, which this repository
 * mirrors in include/forge/ on top of this ABI.
 */
#ifndef PF_B200_H
#define PF_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define PF_API __attribute__((visibility("default")))
#else
#define PF_API
#endif

typedef int32_t pf_status;
enum {
    PF_OK = 0,
    PF_ERR_INVALID = 1,    /* bad argument (size, pointer, config)            */
    PF_ERR_CUDA = 2,       /* a CUDA runtime call failed                       */
    PF_ERR_OOM = 3,        /* device allocation failed                         */
    PF_ERR_NO_DEVICE = 4,  /* no sm_100 device visible                         */
    PF_ERR_DEVICE = 5,     /* a kernel latched an error flag (bounds, timeout) */
    PF_ERR_STATE = 6       /* call out of order (e.g. step before prefill)     */
};

/* Quantization types: the codes of Quantizer::quantize_matrix
 * (src/quant_format.cpp:50-154) and WeightBlock::quant_type. */
enum { PF_QT_Q8 = 0, PF_QT_Q4 = 1, PF_QT_Q2 = 2, PF_QT_Q15 = 3 };

/* Matrix ids inside a layer, as written by src/quant_tool.cpp and read by
 * Engine::load_layer_weights (src/engine.cpp:606-640). */
enum { PF_MAT_Q = 0, PF_MAT_K = 1, PF_MAT_V = 2, PF_MAT_O = 3,
       PF_MAT_GATE = 4, PF_MAT_UP = 5, PF_MAT_DOWN = 6, PF_MAT_COUNT = 7 };

/* Model + cache shape.  Mirrors ModelConfig (include/forge/types.hpp:220-254),
 * KVCacheConfig (include/forge/kv_cache.hpp:23-31) and MTPConfig
 * (include/forge/mtp.hpp:23-29); mtp_ff_dim == n_embd as Engine::load_model
 * sets it (src/engine.cpp:79). */
typedef struct pf_model_config {
    int32_t n_layers;
    int32_t n_embd;
    int32_t n_heads;
    int32_t n_kv_heads;
    int32_t head_dim;       /* n_embd / n_heads (ModelConfig::head_dim) */
    int32_t n_ff;
    int32_t n_vocab;
    int32_t n_mtp_heads;    /* draft heads = K */
    int32_t sink_size;      /* 4   (src/engine.cpp:68)  */
    int32_t window_size;    /* min(kv_cache_size, 8192) (src/engine.cpp:66) */
    int32_t pool_block;     /* 64  (src/engine.cpp:69)  */
    int32_t max_context;    /* positions >= max_context are not stored */
    float   rope_theta;
    float   norm_eps;       /* 1e-6f, hard-coded in rmsnorm (src/matmul_neon.cpp:234) */
    int32_t skip_enabled;   /* predictive FFN skip (src/layer_skip.cpp:22-67) */
    float   skip_threshold;
    int32_t qtype[PF_MAT_COUNT];  /* per-matrix quantization type */
    int32_t emb_qtype;            /* type of embedding block (0,10) */
} pf_model_config;

/* SamplingConfig (include/forge/types.hpp:36-41). */
typedef struct pf_sampling_config {
    float    temperature;
    float    top_p;
    uint32_t top_k;
    int32_t  greedy;
} pf_sampling_config;

/* ------------------------------------------------------------------ */
/* Library                                                              */
/* ------------------------------------------------------------------ */
PF_API const char* pf_last_error(void);
/* The device-side error flags latched by kernels of the current device since
 * they were last cleared (bits: 1 index out of range, 2 weight value outside
 * its packed format, 4 token id outside the vocabulary, 8 context full,
 * 16 pipeline wait timed out); with `clear`, resets them.  Synchronises the
 * device. */
PF_API pf_status pf_read_device_error(uint32_t* flags, int32_t clear);
/* Number of visible devices with compute capability 10.x (0 when none). */
PF_API int32_t pf_device_count(void);
/* Bytes of one packed weight matrix on the device for a format. */
PF_API size_t pf_packed_weight_bytes(int32_t rows, int32_t cols, int32_t qtype);

/* ------------------------------------------------------------------ */
/* Kernel-level entry points (device pointers, caller-owned)            */
/* ------------------------------------------------------------------ */

/* forge::quantize_activation_row (include/forge/matmul_neon.hpp:20-25),
 * applied to each of M rows of x[M][K]: q[M][K] int8, scales[M]. */
PF_API pf_status pf_quantize_activation_rows(const float* x, int8_t* q, float* scales,
                                      int32_t M, int32_t K, void* stream);

/* forge::dequant_q4_to_int8 / dequant_q2_to_int8 / dequant_ternary_to_int8
 * (include/forge/matmul_neon.hpp:28-48). `scale` is ignored, as in the
 * reference (src/matmul_neon.cpp:37,53). */
PF_API pf_status pf_dequant_q4_to_int8(const uint8_t* src, int8_t* dst, float scale,
                                int64_t n, void* stream);
PF_API pf_status pf_dequant_q2_to_int8(const uint8_t* src, int8_t* dst, float scale,
                                int64_t n, void* stream);
PF_API pf_status pf_dequant_ternary_to_int8(const uint8_t* src, int8_t* dst,
                                     int64_t n, void* stream);

/* forge::matmul_int8 (include/forge/matmul_neon.hpp:55-62):
 * C[M][N] (int32) = A[M][K] (int8) . B[N][K]^T (int8).  M = 0 does nothing. */
PF_API pf_status pf_matmul_int8(const int8_t* A, const int8_t* B, int32_t* C,
                         int32_t M, int32_t N, int32_t K, void* stream);

/* forge::matmul_quantized (include/forge/matmul_neon.hpp:68-77):
 * C = ((float)(quant(A) . B^T) * a_scale[i]) * w_scale[j].
 * act_scales may be NULL (computed per row, as the engine always does).
 * M = 0 does nothing. */
PF_API pf_status pf_matmul_quantized(const float* A, const int8_t* B, float* C,
                              int32_t M, int32_t N, int32_t K,
                              const float* weight_scales, const float* act_scales,
                              void* stream);

/* forge::rmsnorm (include/forge/matmul_neon.hpp:92) over M rows of n. */
PF_API pf_status pf_rmsnorm_rows(float* out, const float* x, const float* weight,
                          int32_t M, int32_t n, void* stream);

/* forge::softmax (include/forge/matmul_neon.hpp:87), in place over M rows. */
PF_API pf_status pf_softmax_rows(float* vals, int32_t M, int32_t n, void* stream);

/* Engine::sample_greedy / MTPHeads::argmax (src/engine.cpp:918-928,
 * src/mtp.cpp:145-155): first index of the maximum of each row. */
PF_API pf_status pf_argmax_rows(const float* logits, int32_t M, int32_t n,
                         int32_t* out, void* stream);

/* Engine::sample (src/engine.cpp:881-1003) for each row, the uniform draw of
 * row i given in uniforms[i] (host code pre-draws them from the sequence's
 * std::mt19937 exactly as the reference's uniform_real_distribution<float>). */
PF_API pf_status pf_sample_rows(const float* logits, int32_t M, int32_t n,
                         const pf_sampling_config* cfg, const float* uniforms,
                         int32_t* out, void* stream);

/* ---- single-vector operations behind the forge:: compatibility classes ----
 * One call at a time, device pointers, the reference's summation order
 * (one thread walks a row's loop in sequence). */

/* forge::dot_product (src/matmul_neon.cpp:186-207, scalar path): *out = sum a[i]*b[i]. */
PF_API pf_status pf_dot_f32(const float* a, const float* b, uint32_t n, float* out, void* stream);

/* MTPHeads row products (src/mtp.cpp:66-95, 199-210): y[r] = sum_i x[i] *
 * ((nibble - 8) * scale[r]), w[rows][cols/2] two values per byte, low first. */
PF_API pf_status pf_gemv_q4_rows(const float* x, const uint8_t* w, const float* scale, float* y,
                                 uint32_t rows, uint32_t cols, void* stream);

/* MTPHeads tied unembed (src/mtp.cpp:111-117): y[r] = sum_i x[i] * w[r][i]. */
PF_API pf_status pf_gemv_f32_rows(const float* x, const float* w, float* y, uint32_t rows,
                                  uint32_t cols, void* stream);

/* MTPHeads activation (src/mtp.cpp:82-84, 157-159): a = (g / (1 + exp(-g))) * u. */
PF_API pf_status pf_mtp_silu_mul(const float* g, const float* u, float* a, uint32_t n, void* stream);

/* y += x (the MTP residual, src/mtp.cpp:97-99). */
PF_API pf_status pf_vec_add(float* y, const float* x, uint32_t n, void* stream);

/* MTPHeads logits without an embedding table (src/mtp.cpp:118-123). */
PF_API pf_status pf_mtp_placeholder_logits(float* logits, uint32_t vocab, uint32_t head, void* stream);

/* LayerSkipController::hidden_delta (src/layer_skip.cpp:105-113):
 * *out = sqrt(sum (a-b)^2 / n). */
PF_API pf_status pf_skip_delta(const float* a, const float* b, uint32_t n, float* out, void* stream);

/* KVCache::store of one (layer, head) entry (src/kv_cache.cpp:59-127): the
 * caller chooses the destination slot; if ek is not null the slot's previous
 * entry (ek/eks, ev/evs) is added in double to acc_k / acc_v first, and with
 * finalize the acc_n accumulated entries' mean becomes pool entry pk/pv and
 * the accumulators are cleared.  Then k and v are quantized into dk / dv. */
PF_API pf_status pf_kvu_store(const float* k, const float* v, uint32_t hd, int8_t* dk, float* dks,
                              int8_t* dv, float* dvs, const int8_t* ek, const float* eks,
                              const int8_t* ev, const float* evs, double* acc_k, double* acc_v,
                              uint32_t acc_n, int32_t finalize, int8_t* pk, float* pks, int8_t* pv,
                              float* pvs, void* stream);

/* KVCache::attention_scores / attention_weighted_sum (src/kv_cache.cpp:129-198)
 * of one (layer, head): tiers [0] sink, [1] pool, [2] window ring (`ring`
 * slots, oldest at `head` once counts[2] == ring), counts[t] entries each;
 * tier pointers are device arrays of [count][hd] int8 and [count] scales.
 * Scores: out[e] = q . (k_e * ks_e); weighted sum: out[i] = sum_e p[e] * (v_e[i] * vs_e)
 * over the first min(cnt, total) entries. */
PF_API pf_status pf_kvu_scores(const int8_t* const* tier_k, const float* const* tier_ks,
                               const uint32_t* counts, uint32_t ring, uint32_t head, uint32_t hd,
                               const float* q, float* out, void* stream);
PF_API pf_status pf_kvu_weighted_sum(const int8_t* const* tier_v, const float* const* tier_vs,
                                     const uint32_t* counts, uint32_t ring, uint32_t head,
                                     uint32_t hd, const float* p, uint32_t cnt, float* out,
                                     void* stream);

/* Packs an int8 weight matrix w[rows][cols] (values of the reference loader,
 * WeightLoader::load_block_with_scales, src/quant_format.cpp:348-425) into the
 * device format of `qtype` (Q4: 4-bit, Q2/Q1.5: 2-bit, Q8: 8-bit).
 * Values outside the format's range are rejected with PF_ERR_DEVICE. */
PF_API pf_status pf_pack_weights(const int8_t* w, int32_t rows, int32_t cols,
                          int32_t qtype, void* packed, void* stream);

/* The projection kernel of the engine: C = (int32)(Aq . unpack(W)^T) with the
 * scale epilogue of matmul_quantized (src/matmul_neon.cpp:176-180):
 * C[i][j] = ((float)acc * a_scale[i]) * w_scale[j]. Aq int8 [M][K].
 * M = 0 does nothing. */
PF_API pf_status pf_gemm_packed(const int8_t* Aq, const float* a_scale,
                         const void* packed_w, const float* w_scale, int32_t qtype,
                         float* C, int32_t M, int32_t N, int32_t K, void* stream);

/* pf_gemm_packed without any allocation: the same projection, computed with a
 * split-K reduction whose int32 partial sums live in a fixed array inside the
 * library (no counterpart in the reference, which has no device memory).
 * For callers that cannot call cudaMalloc — a runtime whose own pool owns all
 * device memory, or a path that must not risk the device synchronisation an
 * allocation can cause.  Limits: M*N <= 1,048,576 and ceil(M/128)*ceil(N/64)
 * <= 4096 (else PF_ERR_INVALID); M = 0 does nothing.  Every GPU that loads
 * the library holds the 4 MiB array until exit; calls share it, so calls that
 * overlap on the GPU race.  The first call on a device loads the array's
 * module there: make it before any stream capture.  The array's address is
 * looked up on every call, so calls stay valid after cudaDeviceReset. */
PF_API pf_status pf_gemm_packed_static(const int8_t* Aq, const float* a_scale, const void* packed_w,
                                       const float* w_scale, int32_t qtype, float* C, int32_t M, int32_t N,
                                       int32_t K, void* stream);

/* Diagnostic with no counterpart in the reference: checks, on the device,
 * the branch-free correctly rounded reciprocal that the projection kernels'
 * SwiGLU epilogue uses against CUDA's __frcp_rn for every float in
 * [1, +inf].  *mismatches receives the count, *first_bad the lowest
 * mismatching bit pattern (0xFFFFFFFF if none). */
PF_API pf_status pf_check_reciprocal(uint64_t* mismatches, uint32_t* first_bad);

/* Diagnostic with no counterpart in the reference: checks, on the device, the
 * one-warp exact form of the sampler's sequential float sums (the normalising
 * sum and the cumulative scan) against the reference's one-at-a-time float
 * loop.  terms: device [rows][n] (n <= 16384; terms >= 0, inf or NaN);
 * sorted != 0: every row is non-increasing (the sorted rows' early exit is
 * taken); u, p: device [rows], the scan stops at the first partial sum c with
 * u <= c or c >= p.  *mismatches (host) receives the number of rows whose full
 * sum, stop index or stopping sum differ in any bit. */
PF_API pf_status pf_check_ordered_scan(const float* terms, int32_t rows, int32_t n, int32_t sorted, const float* u,
                                       const float* p, uint32_t* mismatches);

/* ------------------------------------------------------------------ */
/* Engine: batched MTP speculative decoding                             */
/* (Engine::generate / forward_with_hidden / MTPHeads::forward,         */
/*  src/engine.cpp:276-589, src/mtp.cpp:47-129)                         */
/* ------------------------------------------------------------------ */
typedef struct pf_engine pf_engine;

/* max_seqs sequences of up to max_positions tokens each.  K = n_mtp_heads. */
PF_API pf_status pf_engine_create(const pf_model_config* cfg, int32_t max_seqs,
                           int32_t max_positions, int32_t device, pf_engine** out);
PF_API void      pf_engine_destroy(pf_engine* e);

/* Weights (host pointers).  Layer matrices: int8 values + per-row scales as the
 * reference's WeightLoader::load_block_with_scales returns them
 * (src/quant_format.cpp:348-425). */
PF_API pf_status pf_engine_set_matrix(pf_engine* e, int32_t layer, int32_t matrix,
                               const int8_t* w, const float* row_scales);
/* Tied embedding: int8 [n_vocab][n_embd] and the block's global_scale
 * (src/engine.cpp:146-165). */
PF_API pf_status pf_engine_set_embedding(pf_engine* e, const int8_t* emb, float global_scale);
/* RMSNorm weights (blocks 7/8/9, src/engine.cpp:171-203); default all 1.0. */
PF_API pf_status pf_engine_set_norms(pf_engine* e, const float* attn_norm, const float* ffn_norm,
                              const float* final_norm);
/* One MTP head: packed Q4 nibbles + per-row scales as MTPHeads::quantize_q4
 * produces them (src/mtp.cpp:174-197). gate/up: [n_embd][n_embd/2] bytes,
 * down: [n_embd][n_embd/2] bytes. */
PF_API pf_status pf_engine_set_mtp_head(pf_engine* e, int32_t head,
                                 const uint8_t* gate_q4, const float* gate_scale,
                                 const uint8_t* up_q4, const float* up_scale,
                                 const uint8_t* down_q4, const float* down_scale);

/* Sampling: greedy when cfg->greedy or temperature <= 0 (src/engine.cpp:883). */
PF_API pf_status pf_engine_set_sampling(pf_engine* e, const pf_sampling_config* cfg);
/* Layer-skip threshold (Engine::set_layer_skip_threshold, src/engine.cpp:266-269). */
PF_API pf_status pf_engine_set_skip_threshold(pf_engine* e, float threshold);

/* Resets all sequences and prefills n_seqs prompts (host arrays; prompt i is
 * tokens[offsets[i] .. offsets[i+1])).  Afterwards each sequence holds its
 * first pending token and K MTP drafts.  seeds[i] seeds sequence i's
 * std::mt19937 for stochastic sampling (may be NULL when greedy). */
PF_API pf_status pf_engine_prefill(pf_engine* e, int32_t n_seqs, const int32_t* tokens,
                            const int64_t* offsets, const uint32_t* seeds);

/* One speculative-decode step for every sequence: verify the K+1 rows
 * [pending, drafts...], accept the longest matching prefix, commit its KV /
 * skip-cache state, emit accepted + 1 tokens, and draft K new tokens.
 * n_emitted[i] (host, may be NULL) receives accepted+1 for sequence i and
 * emitted (host, may be NULL) receives those tokens at emitted[i*(K+1)+j]. */
PF_API pf_status pf_engine_step(pf_engine* e, int32_t* n_emitted, int32_t* emitted);

/* Replaces the pending drafts of every sequence (host [n_seqs][K]): drafts
 * from another proposer, or forced drafts that exercise acceptance. */
PF_API pf_status pf_engine_set_drafts(pf_engine* e, const int32_t* drafts);

/* Runs `steps` steps back to back without host synchronisation in between
 * (tokens stay on the device); for timing. */
PF_API pf_status pf_engine_run_steps(pf_engine* e, int32_t steps);

/* Copies of engine state, for tests (host destinations). */
PF_API pf_status pf_engine_read_logits(pf_engine* e, float* out);       /* [n_seqs*(K+1)][n_vocab] of the last verify */
PF_API pf_status pf_engine_read_drafts(pf_engine* e, int32_t* out);     /* [n_seqs][K]   */
PF_API pf_status pf_engine_read_pending(pf_engine* e, int32_t* out);    /* [n_seqs]      */
PF_API pf_status pf_engine_read_positions(pf_engine* e, int32_t* out);  /* [n_seqs] committed lengths */
PF_API pf_status pf_engine_read_hidden(pf_engine* e, float* out);       /* [n_seqs][n_embd] MTP input */
PF_API pf_status pf_engine_read_mtp_logits(pf_engine* e, float* out);   /* [n_seqs][K][n_vocab] */
PF_API pf_status pf_engine_read_skip_counts(pf_engine* e, int64_t* computed, int64_t* skipped);
/* Every token emitted since prefill: counts[n_seqs], tokens[n_seqs][cap]. */
PF_API pf_status pf_engine_read_log(pf_engine* e, int32_t* counts, int32_t* tokens, int32_t cap);
/* Committed K/V of one (sequence, layer, kv_head) in the reference's logical
 * attention order (sink, pool, window): k,v int8 [count][head_dim] and
 * scales [count].  *count receives the number of entries. */
PF_API pf_status pf_engine_read_kv(pf_engine* e, int32_t seq, int32_t layer, int32_t kv_head,
                            int8_t* k, float* k_scale, int8_t* v, float* v_scale,
                            int32_t max_entries, int32_t* count);
/* Kernels launched by one decode step (nodes of the captured CUDA graph). */
PF_API pf_status pf_engine_launches_per_step(pf_engine* e, int32_t* kernels);
/* Device time of the last pf_engine_step / run_steps call, milliseconds. */
PF_API pf_status pf_engine_last_ms(pf_engine* e, float* ms);

/* Per-kernel timing (no counterpart in the reference): with timing on, the
 * step graph is recaptured with CUDA event pairs around every attention
 * launch and every projection GEMM; after a step, pf_engine_kernel_times
 * returns the summed device milliseconds and launch counts of the last step
 * for [0] attention and [1] projections.  Timing perturbs the graph (the event
 * nodes serialise the launches), so measure the step itself with it off. */
PF_API pf_status pf_engine_set_kernel_timing(pf_engine* e, int32_t on);
/* Number of CTAs over which the verify attention splits the context of each
 * (sequence, kv head), 1..8; 0 (the default) picks about two waves of CTAs
 * for the engine's sequence count.  Results do not depend on it beyond float
 * rounding. */
PF_API pf_status pf_engine_set_attention_splits(pf_engine* e, int32_t n);
PF_API pf_status pf_engine_kernel_times(pf_engine* e, float* ms, int32_t* launches);

/* ------------------------------------------------------------------ */
/* Synthetic model (benchmark and test inputs; host memory)             */
/* ------------------------------------------------------------------ */
/* One transformer matrix as the reference's tools would produce it:
 * N(0, 0.02) floats from a std::mt19937 seeded per (seed, layer, matrix),
 * Quantizer::quantize_matrix (src/quant_format.cpp:44-157), then
 * WeightLoader::load_block_with_scales (src/quant_format.cpp:348-425).
 * The embedding is (layer 0, matrix 10). */
PF_API pf_status pf_synth_matrix(uint32_t seed, int32_t layer, int32_t matrix, int32_t rows, int32_t cols,
                                 int32_t qtype, int8_t* out, float* row_scales, float* global_scale);
/* MTP matrix `which` (0 gate, 1 up, 2 down) of `head`: uniform(-1,1)/sqrt(d)
 * floats (MTPHeads::init_weights, src/mtp.cpp:31-39) through
 * MTPHeads::quantize_q4 (src/mtp.cpp:174-197): q4 [d][d/2], scales [d]. */
PF_API pf_status pf_synth_mtp_matrix(uint32_t seed, int32_t head, int32_t which, int32_t d, uint8_t* q4,
                                     float* scales);
/* Generates every matrix of the model on `threads` host threads and loads it. */
PF_API pf_status pf_engine_load_synthetic(pf_engine* e, const pf_model_config* cfg, uint32_t seed,
                                          uint32_t mtp_seed, int32_t threads);

#ifdef __cplusplus
}
#endif
#endif /* PF_B200_H */

// step.cuh — per-step control state of the engine and the kernels of accept.cu.
#pragma once
#include "common.cuh"

namespace pf {

struct StepBufs {
    int n_seqs = 0, K = 0, max_pos = 0;
    int* pending = nullptr;   // [n_seqs] next token to verify (not yet in the cache)
    int* drafts = nullptr;    // [n_seqs][K]
    int* seq_len = nullptr;   // [n_seqs] committed positions
    int* row_tok = nullptr;   // [M]
    int* row_pos = nullptr;   // [M]
    int* bs_row0 = nullptr;   // [n_seqs]
    int* bs_n = nullptr;      // [n_seqs]
    int* bs_len0 = nullptr;   // [n_seqs]
    int* amax = nullptr;      // [M] greedy token of each verify row
    int* n_commit = nullptr;  // [n_seqs]
    int* final_row = nullptr; // [n_seqs]
    int* emitted = nullptr;   // [n_seqs][K+1]
    int* n_emitted = nullptr; // [n_seqs]
    int* log = nullptr;       // [n_seqs][log_cap] every emitted token
    int log_cap = 0;
    int* n_logged = nullptr;  // [n_seqs]
};

pf_status verify_setup(const StepBufs& s, cudaStream_t st);
pf_status accept(const StepBufs& s, cudaStream_t st);
pf_status finish(const StepBufs& s, const int* next, cudaStream_t st);
pf_status gather_rows(const float* x, int d, const int* idx, int n, float* out, cudaStream_t st);
pf_status sample_rows(const float* logits, int ld, int V, const int* rows, int n, const pf_sampling_config& cfg,
                      const float* uniforms, int ustride, int* out, cudaStream_t st);
pf_status pick(const int* src, const int* idx, int n, int* out, cudaStream_t st);
pf_status put_draft(const int* tok, int n, int K, int h, int* drafts, cudaStream_t st);
// drafts[b][h] = tok[h * stride + b] for every head h < K and sequence b < n.
pf_status put_drafts(const int* tok, int n, int K, int stride, int* drafts, cudaStream_t st);
pf_status skip_decide(int nb, const int* bs_row0, const int* bs_n, int max_rows, const float* normed, int d,
                      const float* cache, size_t cache_stride, float thr_l, uint8_t* skip, cudaStream_t st);
pf_status skip_commit(int nb, int L, int d, int Mst, const int* bs_row0, const int* n_commit, const uint8_t* skip_all,
                      const float* normed_all, float* cache, long long* counts, cudaStream_t st);
pf_status ffn_count(int nb, int L, const int* n_commit, long long* counts, cudaStream_t st);

}  // namespace pf

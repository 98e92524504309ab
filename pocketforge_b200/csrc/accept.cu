// accept.cu — the control kernels of a speculative-decode step: building the
// K+1 verify rows, the greedy acceptance of the drafted prefix, stochastic
// sampling (temperature / top-k / top-p with the reference's quirks),
// predictive FFN layer skipping, and the commit of per-sequence state.
#include <cfloat>

#include "step.cuh"

namespace pf {

// ---------------------------------------------------------------------------
// Verify rows: [pending, d_0 .. d_{K-1}] at positions len .. len+K.
// ---------------------------------------------------------------------------
__global__ void verify_setup_kernel(int n_seqs, int K, int max_pos, const int* __restrict__ pending,
                                    const int* __restrict__ drafts, const int* __restrict__ seq_len,
                                    int* __restrict__ row_tok, int* __restrict__ row_pos, int* __restrict__ bs_row0,
                                    int* __restrict__ bs_n, int* __restrict__ bs_len0, uint32_t* err) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_seqs) return;
    const int R = K + 1;
    const int len = seq_len[b];
    const bool fits = len + R <= max_pos;
    if (!fits) atomicOr(err, ERR_CONTEXT);
    bs_row0[b] = b * R;
    bs_n[b] = fits ? R : 0;
    bs_len0[b] = len;
    for (int r = 0; r < R; r++) {
        row_tok[b * R + r] = (r == 0) ? pending[b] : drafts[b * K + r - 1];
        row_pos[b * R + r] = min(len + r, max_pos - 1);
    }
}

pf_status verify_setup(const StepBufs& s, cudaStream_t st) {
    verify_setup_kernel<<<ceil_div(s.n_seqs, 128), 128, 0, st>>>(s.n_seqs, s.K, s.max_pos, s.pending, s.drafts,
                                                                 s.seq_len, s.row_tok, s.row_pos, s.bs_row0, s.bs_n,
                                                                 s.bs_len0, device_error_flag());
    return launch_check("verify_setup");
}

// ---------------------------------------------------------------------------
// Acceptance (src/engine.cpp:333-365 with D7): accept drafts while the main
// model's greedy token of the previous row equals the draft; the row after
// the accepted prefix gives the next token.
// ---------------------------------------------------------------------------
__global__ void accept_kernel(int n_seqs, int K, const int* __restrict__ amax, const int* __restrict__ drafts,
                              const int* __restrict__ bs_n, int* __restrict__ n_commit, int* __restrict__ final_row) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_seqs) return;
    const int R = K + 1;
    if (bs_n[b] == 0) {
        n_commit[b] = 0;
        final_row[b] = b * R;
        return;
    }
    int a = 0;
    while (a < K && amax[b * R + a] == drafts[b * K + a]) a++;
    n_commit[b] = a + 1;
    final_row[b] = b * R + a;
}

pf_status accept(const StepBufs& s, cudaStream_t st) {
    accept_kernel<<<ceil_div(s.n_seqs, 128), 128, 0, st>>>(s.n_seqs, s.K, s.amax, s.drafts, s.bs_n, s.n_commit,
                                                           s.final_row);
    return launch_check("accept");
}

// ---------------------------------------------------------------------------
// Finish: emitted tokens, pending token, lengths, token log.
// ---------------------------------------------------------------------------
__global__ void finish_kernel(int n_seqs, int K, const int* __restrict__ next, const int* __restrict__ n_commit,
                              const int* __restrict__ drafts, int* __restrict__ pending, int* __restrict__ seq_len,
                              int* __restrict__ emitted, int* __restrict__ n_emitted, int* __restrict__ log,
                              int log_cap, int* __restrict__ n_logged) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_seqs) return;
    const int R = K + 1;
    const int nc = n_commit[b];
    n_emitted[b] = nc;
    for (int j = 0; j < R; j++) {
        int t = -1;
        if (nc > 0) t = (j < nc - 1) ? drafts[b * K + j] : (j == nc - 1 ? next[b] : -1);
        emitted[b * R + j] = t;
    }
    if (nc == 0) return;
    pending[b] = next[b];
    seq_len[b] += nc;
    if (log) {
        int c = n_logged[b];
        for (int j = 0; j < nc && c < log_cap; j++, c++) log[(size_t)b * log_cap + c] = emitted[b * R + j];
        n_logged[b] = c;
    }
}

pf_status finish(const StepBufs& s, const int* next, cudaStream_t st) {
    finish_kernel<<<ceil_div(s.n_seqs, 128), 128, 0, st>>>(s.n_seqs, s.K, next, s.n_commit, s.drafts, s.pending,
                                                           s.seq_len, s.emitted, s.n_emitted, s.log, s.log_cap,
                                                           s.n_logged);
    return launch_check("finish");
}

// Copies row idx[b] of x[.][d] to out[b][d].
__global__ void gather_rows_kernel(const float* __restrict__ x, int d, const int* __restrict__ idx, int n,
                                   float* __restrict__ out) {
    const int b = blockIdx.x;
    if (b >= n) return;
    const float* src = x + (size_t)idx[b] * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) out[(size_t)b * d + i] = src[i];
}

pf_status gather_rows(const float* x, int d, const int* idx, int n, float* out, cudaStream_t st) {
    gather_rows_kernel<<<n, 256, 0, st>>>(x, d, idx, n, out);
    return launch_check("gather_rows");
}

// ---------------------------------------------------------------------------
// Stochastic sampling of one row per sequence (src/engine.cpp:881-1003).
// Dispatch as the reference: top-p when 0<p<1 (top-k is then ignored),
// else top-k when 0<k<V, else plain temperature.  One CTA sorts the row
// (descending value, ascending index on ties; std::sort leaves the order of
// exactly equal logits unspecified) with a bitonic sort in shared memory.
// The exponentials are computed in parallel (double exp rounded to float:
// the correctly rounded value the reference's std::exp returns in all but
// rare halfway cases); the normalising sum and the cumulative scans are
// sequential float additions in the reference's order, so the draw is the
// reference's.  Sorted-descending scans stop at the first zero term (adding
// +0 changes nothing).  The divisions by the sum are independent of one
// another and run on all threads; one thread then adds the quotients in
// order, and a single pass finds both the draw and the top-p cut (the
// reference's two cumulative scans add the same quotients in the same
// order, so their partial sums are the same numbers).
// ---------------------------------------------------------------------------
namespace {
constexpr int SORT_THREADS = 1024;

__device__ __forceinline__ bool before(float va, int ia, float vb, int ib) {
    return va > vb || (va == vb && ia < ib);
}
__device__ __forceinline__ float exp_ref(float x) { return (float)exp((double)x); }

// One thread's ordered pass over a[0, n): f(i, a[i]) for i = 0, 1, ... until
// it returns true; returns that i, or n.  Four terms per 16-byte load, the
// next four loaded before the current ones are used (a is 16-byte aligned).
template <typename F>
__device__ __forceinline__ int ordered_pass(const float* a, int n, F f) {
    const int n4 = n & ~3;
    float4 nxt = n4 > 0 ? *reinterpret_cast<const float4*>(a) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = 0; i < n4; i += 4) {
        const float4 v = nxt;
        if (i + 4 < n4) nxt = *reinterpret_cast<const float4*>(a + i + 4);
        if (f(i, v.x)) return i;
        if (f(i + 1, v.y)) return i + 1;
        if (f(i + 2, v.z)) return i + 2;
        if (f(i + 3, v.w)) return i + 3;
    }
    for (int i = n4; i < n; i++)
        if (f(i, a[i])) return i;
    return n;
}
}  // namespace

__global__ void __launch_bounds__(SORT_THREADS) sample_kernel(const float* __restrict__ logits, int ld, int V, int P2,
                                                              const int* __restrict__ rows, int n, pf_sampling_config cfg,
                                                              const float* __restrict__ uniforms, int ustride,
                                                              int* __restrict__ out) {
    extern __shared__ __align__(16) uint8_t sm[];
    float* key = reinterpret_cast<float*>(sm);
    int* idx = reinterpret_cast<int*>(sm + (size_t)P2 * sizeof(float));
    __shared__ float red[32];
    const int b = blockIdx.x;
    if (b >= n) return;
    const float* lg = logits + (size_t)rows[b] * ld;
    const float u = uniforms[(size_t)b * ustride];
    const float t = fmaxf(cfg.temperature, 0.001f);
    const bool top_p = cfg.top_p < 1.0f && cfg.top_p > 0.0f;
    const bool top_k = !top_p && cfg.top_k > 0 && (int)cfg.top_k < V;
    const int tid = threadIdx.x;
    if (!top_p && !top_k) {  // temperature sampling in index order (src/engine.cpp:895-915)
        float mx = -INFINITY;
        for (int i = tid; i < V; i += blockDim.x) mx = fmaxf(mx, lg[i]);
        for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if ((tid & 31) == 0) red[tid >> 5] = mx;
        __syncthreads();
        if (tid == 0) {
            float m = red[0];
            for (int w = 1; w < (int)(blockDim.x >> 5); w++) m = fmaxf(m, red[w]);
            red[0] = m;
        }
        __syncthreads();
        mx = red[0];
        for (int i = tid; i < V; i += blockDim.x) key[i] = exp_ref(__fdiv_rn(__fsub_rn(lg[i], mx), t));
        __syncthreads();
        if (tid == 0) {
            float sum = 0.0f;
            ordered_pass(key, V, [&](int, float q) {
                sum = __fadd_rn(sum, q);
                return false;
            });
            red[0] = sum;
        }
        __syncthreads();
        const float sum = red[0];
        for (int i = tid; i < V; i += blockDim.x) key[i] = __fdiv_rn(key[i], sum);
        __syncthreads();
        if (tid == 0) {
            float cum = 0.0f;
            const int i = ordered_pass(key, V, [&](int, float q) {
                cum = __fadd_rn(cum, q);
                return u <= cum;
            });
            out[b] = i < V ? i : V - 1;
        }
        return;
    }
    for (int i = tid; i < P2; i += blockDim.x) {
        key[i] = i < V ? lg[i] : -INFINITY;
        idx[i] = i < V ? i : 0x7fffffff;
    }
    __syncthreads();
    for (int k = 2; k <= P2; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < P2; i += blockDim.x) {
                const int p = i ^ j;
                if (p > i) {
                    const bool desc = (i & k) == 0;
                    const bool swap = desc ? before(key[p], idx[p], key[i], idx[i]) : before(key[i], idx[i], key[p], idx[p]);
                    if (swap) {
                        const float tk = key[i];
                        key[i] = key[p];
                        key[p] = tk;
                        const int ti = idx[i];
                        idx[i] = idx[p];
                        idx[p] = ti;
                    }
                }
            }
            __syncthreads();
        }
    const float mx = key[0];
    const int nn = top_p ? V : (int)cfg.top_k;
    __syncthreads();
    // exponentials in sorted order, in place (key[i] is no longer needed after this)
    for (int i = tid; i < nn; i += blockDim.x) key[i] = exp_ref(__fdiv_rn(__fsub_rn(key[i], mx), t));
    __syncthreads();
    __shared__ int s_nz;
    if (tid == 0) {
        float total = 0.0f;
        // terms after the first zero are zero too (sorted descending)
        const int nz = ordered_pass(key, nn, [&](int, float q) {
            if (q == 0.0f) return true;
            total = __fadd_rn(total, q);
            return false;
        });
        red[0] = total;
        s_nz = nz;
    }
    __syncthreads();
    const float total = red[0];
    const int nz = s_nz;
    for (int i = tid; i < nz; i += blockDim.x) key[i] = __fdiv_rn(key[i], total);  // the normalised terms
    __syncthreads();
    if (tid != 0) return;
    if (top_p) {  // src/engine.cpp:972-1002: normalise, cut at cumulative >= p, draw without renormalising
        // The draw scans i < min(cut, nz) with the same partial sums as the
        // cut scan: checking the draw before the cut at each i is both scans.
        int cut = nn;
        float cum = 0.0f;
        int pick = -1;
        ordered_pass(key, nz, [&](int i, float q) {
            cum = __fadd_rn(cum, q);
            if (u <= cum) {
                pick = i;
                return true;
            }
            if (cum >= cfg.top_p) {
                cut = i + 1;
                return true;
            }
            return false;
        });
        out[b] = idx[pick >= 0 ? pick : cut - 1];
    } else {  // top-k (src/engine.cpp:930-959)
        float cum = 0.0f;
        const int i = ordered_pass(key, nz, [&](int, float q) {
            cum = __fadd_rn(cum, q);
            return u <= cum;
        });
        out[b] = idx[i < nz ? i : nn - 1];
    }
}

pf_status sample_rows(const float* logits, int ld, int V, const int* rows, int n, const pf_sampling_config& cfg,
                      const float* uniforms, int ustride, int* out, cudaStream_t st) {
    int P2 = 1;
    while (P2 < V) P2 <<= 1;
    PF_CHECK(P2 <= 16384, "sample_rows: vocabulary above 16384 is not supported");
    const size_t smem = (size_t)P2 * (sizeof(float) + sizeof(int));
    static bool attr = false;
    if (!attr) {
        PF_CUDA(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 16384 * 8));
        attr = true;
    }
    sample_kernel<<<n, SORT_THREADS, smem, st>>>(logits, ld, V, P2, rows, n, cfg, uniforms, ustride, out);
    return launch_check("sample_rows");
}

// Copies idx-selected int values: out[b] = src[idx[b]].
__global__ void pick_kernel(const int* __restrict__ src, const int* __restrict__ idx, int n, int* __restrict__ out) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < n) out[b] = src[idx[b]];
}
pf_status pick(const int* src, const int* idx, int n, int* out, cudaStream_t st) {
    pick_kernel<<<ceil_div(n, 128), 128, 0, st>>>(src, idx, n, out);
    return launch_check("pick");
}

// Writes draft h of every sequence: drafts[b*K + h] = tok[b].
__global__ void put_draft_kernel(const int* __restrict__ tok, int n, int K, int h, int* __restrict__ drafts) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < n) drafts[b * K + h] = tok[b];
}
pf_status put_draft(const int* tok, int n, int K, int h, int* drafts, cudaStream_t st) {
    put_draft_kernel<<<ceil_div(n, 128), 128, 0, st>>>(tok, n, K, h, drafts);
    return launch_check("put_draft");
}

// ---------------------------------------------------------------------------
// Predictive FFN skip (LayerSkipController::should_skip_ffn,
// src/layer_skip.cpp:22-67): rows of a sequence in order, each compared with
// the post-norm vector of the last row whose FFN ran (committed cache at the
// start).  One warp per sequence; the RMS delta uses the device sum order.
// ---------------------------------------------------------------------------
__global__ void skip_decide_kernel(int nb, const int* __restrict__ bs_row0, const int* __restrict__ bs_n,
                                   const float* __restrict__ normed, int d, const float* __restrict__ cache,
                                   size_t cache_stride, float thr_l, uint8_t* __restrict__ skip) {
    const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (b >= nb) return;
    const int n = bs_n[b], row0 = bs_row0[b];
    const float* ref = cache + (size_t)b * cache_stride;
    for (int r = 0; r < n; r++) {
        const float* x = normed + (size_t)(row0 + r) * d;
        float s = 0.0f;
        // the lane's elements in order, 16 at a time with their loads issued first
        for (int i0 = lane; i0 < d; i0 += 32 * 16) {
            float xa[16], ra[16];
#pragma unroll
            for (int k = 0; k < 16; k++) {
                const int i = i0 + 32 * k;
                xa[k] = i < d ? x[i] : 0.0f;
                ra[k] = i < d ? ref[i] : 0.0f;
            }
#pragma unroll
            for (int k = 0; k < 16; k++) {
                if (i0 + 32 * k >= d) break;
                const float df = __fsub_rn(xa[k], ra[k]);
                s = __fadd_rn(s, __fmul_rn(df, df));
            }
        }
        for (int o = 16; o >= 1; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
        const float delta = __fsqrt_rn(__fdiv_rn(s, (float)d));
        const bool sk = delta < thr_l;
        if (lane == 0) skip[row0 + r] = sk ? 1 : 0;
        if (!sk) ref = x;
    }
}

pf_status skip_decide(int nb, const int* bs_row0, const int* bs_n, const float* normed, int d, const float* cache,
                      size_t cache_stride, float thr_l, uint8_t* skip, cudaStream_t st) {
    skip_decide_kernel<<<ceil_div(nb, 4), 128, 0, st>>>(nb, bs_row0, bs_n, normed, d, cache, cache_stride, thr_l,
                                                        skip);
    return launch_check("skip_decide");
}

// After acceptance: the skip cache of layer l becomes the post-norm vector of
// the last committed row whose FFN ran at that layer (unchanged if none).
__global__ void skip_commit_kernel(int nb, int L, int d, int Mst, const int* __restrict__ bs_row0,
                                   const int* __restrict__ n_commit, const uint8_t* __restrict__ skip_all,
                                   const float* __restrict__ normed_all, float* __restrict__ cache,
                                   long long* __restrict__ counts) {
    const int b = blockIdx.x, l = blockIdx.y;
    const int nc = n_commit[b];
    if (nc <= 0) return;
    const int row0 = bs_row0[b];
    const uint8_t* sk = skip_all + (size_t)l * Mst;
    int last = -1, ns = 0;
    for (int r = 0; r < nc; r++) {
        if (!sk[row0 + r]) last = r;
        else ns++;
    }
    if (threadIdx.x == 0) {
        atomicAdd(reinterpret_cast<unsigned long long*>(counts + 0), (unsigned long long)(nc - ns));
        atomicAdd(reinterpret_cast<unsigned long long*>(counts + 1), (unsigned long long)ns);
    }
    if (last < 0) return;
    const float* src = normed_all + ((size_t)l * Mst + row0 + last) * d;
    float* dst = cache + ((size_t)b * L + l) * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) dst[i] = src[i];
}

pf_status skip_commit(int nb, int L, int d, int Mst, const int* bs_row0, const int* n_commit, const uint8_t* skip_all,
                      const float* normed_all, float* cache, long long* counts, cudaStream_t st) {
    dim3 grid(nb, L);
    skip_commit_kernel<<<grid, 256, 0, st>>>(nb, L, d, Mst, bs_row0, n_commit, skip_all, normed_all, cache, counts);
    return launch_check("skip_commit");
}

// Counts rows whose FFN ran / was skipped when no skip cache is kept.
__global__ void ffn_count_kernel(int nb, int L, const int* __restrict__ n_commit, long long* __restrict__ counts) {
    long long tot = 0;
    for (int b = threadIdx.x; b < nb; b += blockDim.x) tot += max(0, n_commit[b]);
    for (int o = 16; o >= 1; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(reinterpret_cast<unsigned long long*>(counts), (unsigned long long)(tot * L));
}
pf_status ffn_count(int nb, int L, const int* n_commit, long long* counts, cudaStream_t st) {
    ffn_count_kernel<<<1, 32, 0, st>>>(nb, L, n_commit, counts);
    return launch_check("ffn_count");
}

}  // namespace pf

// accept.cu — the control kernels of a speculative-decode step: building the
// K+1 verify rows, the greedy acceptance of the drafted prefix, stochastic
// sampling (temperature / top-k / top-p with the reference's quirks),
// predictive FFN layer skipping, and the commit of per-sequence state.
#include <cfloat>

#include "scan.cuh"
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
// exactly equal logits unspecified) with a stable radix sort in shared
// memory.  The exponentials are computed in parallel (double exp rounded to
// float: the correctly rounded value the reference's std::exp returns in all
// but rare halfway cases) and so are the divisions by the sum; the
// normalising sum and the cumulative scan are the reference's sequential
// float additions, reproduced exactly by one warp (ordered_scan_warp), so the
// draw is the reference's.  One cumulative scan
// finds both the draw and the top-p cut: the reference's two cumulative scans
// add the same quotients in the same order, so their partial sums are the
// same numbers, and whichever stops first decides the token.
// ---------------------------------------------------------------------------
namespace {
constexpr int SORT_THREADS = 1024;
constexpr int SORT_WARPS = SORT_THREADS / 32;
constexpr int SORT_IPT = 16;  // items per thread: rows of up to 16384 entries
constexpr int SORT_RADIX = 256;

__device__ __forceinline__ float exp_ref(float x) { return (float)exp((double)x); }

// Sort key whose ascending unsigned order is descending value; -0 and +0 get
// the same key (they compare equal, and every use of the value gives the same
// result for either sign).
__device__ __forceinline__ uint32_t desc_key(float v) {
    uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ~b;
}
__device__ __forceinline__ float key_value(uint32_t k) {
    const uint32_t b = ~k;
    return __uint_as_float((b & 0x80000000u) ? (b & 0x7fffffffu) : ~b);
}

// Stable ascending LSD radix sort (8-bit digits) of the CTA's R*1024 items.
// Item j = w*32R + r*32 + lane sits in k[r] / pv[r] >> 16 of that lane of
// warp w; the sorted keys and payloads end in ks / vs.  Ranks within a warp
// come from ballots of the digit bits in item order (measured faster than
// __match_any_sync here); warps' digit counts are scanned
// digit-major, warp-minor, so equal digits keep their item order (stability).
// The payload (< 65536) sits in pv's high half; the low half holds the item's
// rank among the warp's items of its digit during a pass.
__device__ __forceinline__ void block_radix_sort(uint32_t (&k)[SORT_IPT], uint32_t (&pv)[SORT_IPT], int R,
                                                 uint32_t* ks, uint32_t* vs, uint32_t* hist, uint32_t* wsum) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const uint32_t lt = (1u << lane) - 1u;
    uint32_t* hw = hist + w * SORT_RADIX;
    for (int sh = 0; sh < 32; sh += 8) {
        for (int d = lane; d < SORT_RADIX; d += 32) hw[d] = 0;
        __syncwarp();
#pragma unroll
        for (int r = 0; r < SORT_IPT; r++) {
            if (r < R) {
                const uint32_t d = (k[r] >> sh) & (SORT_RADIX - 1);
                uint32_t peers = 0xffffffffu;  // lanes holding the same digit: one ballot per digit bit
#pragma unroll
                for (int bit = 0; bit < 8; bit++) {
                    const bool on = (d >> bit) & 1u;
                    const uint32_t bal = __ballot_sync(0xffffffffu, on);
                    peers &= on ? bal : ~bal;
                }
                const uint32_t base = hw[d];
                __syncwarp();
                if ((peers & lt) == 0) hw[d] = base + __popc(peers);
                __syncwarp();
                pv[r] = (pv[r] & 0xffff0000u) | (base + __popc(peers & lt));
            }
        }
        __syncthreads();
        {  // exclusive scan of the counts in (digit, warp) order: thread t owns digit t/4, warps (t%4)*8 ..
            const int d = threadIdx.x >> 2, w0 = (threadIdx.x & 3) * 8;
            uint32_t c[8], s = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                c[j] = hist[(w0 + j) * SORT_RADIX + d];
                s += c[j];
            }
            uint32_t incl = s;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            if (lane == 31) wsum[w] = incl;
            __syncthreads();
            if (w == 0) {
                const uint32_t x = wsum[lane];
                uint32_t xi = x;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t y = __shfl_up_sync(0xffffffffu, xi, o);
                    if (lane >= o) xi += y;
                }
                wsum[lane] = xi - x;
            }
            __syncthreads();
            uint32_t run = wsum[w] + incl - s;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                hist[(w0 + j) * SORT_RADIX + d] = run;
                run += c[j];
            }
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < SORT_IPT; r++) {
            if (r < R) {
                const uint32_t dst = hw[(k[r] >> sh) & (SORT_RADIX - 1)] + (pv[r] & 0xffffu);
                ks[dst] = k[r];
                vs[dst] = pv[r] >> 16;
            }
        }
        __syncthreads();
        if (sh == 24) break;
#pragma unroll
        for (int r = 0; r < SORT_IPT; r++) {
            if (r < R) {
                const int j = w * 32 * R + r * 32 + lane;
                k[r] = ks[j];
                pv[r] = vs[j] << 16;
            }
        }
    }
}

constexpr int SORT_BUCKETS = 16384;  // value-range buckets: one per entry of the largest row
constexpr int SORT_BUCKET_MAX = 64;   // larger buckets (many equal or clustered values): radix sort instead

// Value-range bucket sort of the same items into the same order as
// block_radix_sort.  bucket(v) = clamp((int)((hi - v) * (B / (hi - lo))), 0,
// B-1) with [lo, hi] = mean -/+ 5 standard deviations of the row's finite
// values: each float operation and the clamp are monotone, so the bucket
// index never increases with v, the buckets in index order hold descending
// values and equal values share a bucket, while outliers (a tied embedding's
// own-token logit sits tens of deviations above the rest) collect in the end
// buckets instead of stretching the range.  Within a bucket every entry counts
// the entries that order before it (key, then index), all in parallel.  The
// items in k / pv are consumed.  cnt holds SORT_BUCKETS counters, turned into
// the buckets' starts in place.  Returns false, having written nothing the
// radix sort reads, when the spread is not a positive finite number or a
// bucket holds more than SORT_BUCKET_MAX entries; the result is uniform over
// the CTA.
__device__ __forceinline__ bool block_bucket_sort(uint32_t (&k)[SORT_IPT], uint32_t (&pv)[SORT_IPT], int R, int V,
                                                  uint32_t* ks, uint32_t* vs, uint32_t* cnt, float* redf,
                                                  uint32_t* wsum, uint32_t* wmax) {
    constexpr int BPT = SORT_BUCKETS / SORT_THREADS;  // buckets per thread in the scan (16)
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    for (int i = tid; i < SORT_BUCKETS; i += SORT_THREADS) cnt[i] = 0;
    float sx = 0.0f, sxx = 0.0f, nf = 0.0f;
#pragma unroll
    for (int r = 0; r < SORT_IPT; r++) {
        if (r < R) {
            const float v = key_value(k[r]);  // padding entries decode to NaN and are skipped
            if (isfinite(v)) {
                sx += v;
                sxx = fmaf(v, v, sxx);
                nf += 1.0f;
            }
        }
    }
    for (int o = 16; o >= 1; o >>= 1) {
        sx += __shfl_xor_sync(0xffffffffu, sx, o);
        sxx += __shfl_xor_sync(0xffffffffu, sxx, o);
        nf += __shfl_xor_sync(0xffffffffu, nf, o);
    }
    if (lane == 0) {
        redf[w] = sx;
        redf[SORT_WARPS + w] = sxx;
        redf[2 * SORT_WARPS + w] = nf;
    }
    __syncthreads();
    sx = sxx = nf = 0.0f;
    for (int i = 0; i < SORT_WARPS; i++) {
        sx += redf[i];
        sxx += redf[SORT_WARPS + i];
        nf += redf[2 * SORT_WARPS + i];
    }
    const float mean = sx / nf, sd = sqrtf(fmaxf(sxx / nf - mean * mean, 0.0f));
    const float hi = mean + 5.0f * sd, range = 10.0f * sd;
    const float scale = __fdiv_rn((float)SORT_BUCKETS, range);
    if (!(range > 0.0f && scale > 0.0f && isfinite(scale) && isfinite(hi))) return false;
    auto bucket = [&](float v) {
        return min(SORT_BUCKETS - 1, max(0, (int)__fmul_rn(__fsub_rn(hi, v), scale)));
    };
#pragma unroll
    for (int r = 0; r < SORT_IPT; r++) {
        if (r < R && w * 32 * R + r * 32 + lane < V)
            pv[r] = (pv[r] & 0xffff0000u) | atomicAdd(&cnt[bucket(key_value(k[r]))], 1u);
    }
    __syncthreads();
    // exclusive scan of the counts (thread t: buckets BPT*t ..) and the largest count
    uint4* c4 = reinterpret_cast<uint4*>(cnt) + tid * (BPT / 4);
    uint32_t s = 0, mc = 0;
#pragma unroll
    for (int q = 0; q < BPT / 4; q++) {
        const uint4 c = c4[q];
        s += c.x + c.y + c.z + c.w;
        mc = max(mc, max(max(c.x, c.y), max(c.z, c.w)));
    }
    uint32_t incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
        mc = max(mc, __shfl_xor_sync(0xffffffffu, mc, o));
    }
    if (lane == 31) wsum[w] = incl;
    if (lane == 0) wmax[w] = mc;
    __syncthreads();
    uint32_t run = incl - s;
    for (int i = 0; i < SORT_WARPS; i++) {
        if (i < w) run += wsum[i];
        mc = max(mc, wmax[i]);
    }
    if (mc > (uint32_t)SORT_BUCKET_MAX) return false;
#pragma unroll
    for (int q = 0; q < BPT / 4; q++) {  // this thread's own counters, read again and replaced by starts
        const uint4 c = c4[q];
        uint4 o;
        o.x = run;
        run += c.x;
        o.y = run;
        run += c.y;
        o.z = run;
        run += c.z;
        o.w = run;
        run += c.w;
        c4[q] = o;
    }
    __syncthreads();
    const uint32_t* start = cnt;
#pragma unroll
    for (int r = 0; r < SORT_IPT; r++) {
        const int j = w * 32 * R + r * 32 + lane;
        if (r < R && j < V) {
            const uint32_t pos = start[bucket(key_value(k[r]))] + (pv[r] & 0xffffu);
            ks[pos] = k[r];
            vs[pos] = (uint32_t)j;
        }
    }
    __syncthreads();
    // Order within the buckets: the entry at position i moves to its bucket's
    // start + the number of the bucket's entries ordered before it (key, then
    // index: a permutation, the indices being distinct).  Ranks are taken for
    // all positions before any entry moves.
#pragma unroll
    for (int r = 0; r < SORT_IPT; r++) {
        const int i = tid + r * SORT_THREADS;
        if (r < R && i < V) {
            const uint32_t kk = ks[i], vv = vs[i];
            const int bk = bucket(key_value(kk));
            const int s0 = (int)start[bk], e = bk + 1 < SORT_BUCKETS ? (int)start[bk + 1] : V;
            const unsigned long long me = ((unsigned long long)kk << 32) | vv;
            int rank = 0;
            for (int j = s0; j < e; j++) rank += (((unsigned long long)ks[j] << 32) | vs[j]) < me;
            k[r] = kk;
            pv[r] = ((uint32_t)(s0 + rank) << 16) | vv;
        }
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < SORT_IPT; r++) {
        const int i = tid + r * SORT_THREADS;
        if (r < R && i < V) {
            ks[pv[r] >> 16] = k[r];
            vs[pv[r] >> 16] = pv[r] & 0xffffu;
        }
    }
    __syncthreads();
    return true;
}

}  // namespace

__global__ void __launch_bounds__(SORT_THREADS, 1)
    sample_kernel(const float* __restrict__ logits, int ld, int V, int R, const int* __restrict__ rows, int n,
                  pf_sampling_config cfg, const float* __restrict__ uniforms, int ustride, int* __restrict__ out) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int cap = R * SORT_THREADS;
    uint32_t* ks = reinterpret_cast<uint32_t*>(sm);
    uint32_t* vs = ks + cap;
    uint32_t* hist = vs + cap;
    float* key = reinterpret_cast<float*>(sm);  // values / terms, in place of ks
    __shared__ float red[3 * SORT_WARPS];
    __shared__ uint32_t wsum[SORT_WARPS], wmax[SORT_WARPS];
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
            for (int w = 1; w < SORT_WARPS; w++) m = fmaxf(m, red[w]);
            red[0] = m;
        }
        __syncthreads();
        mx = red[0];
        for (int i = tid; i < V; i += blockDim.x) key[i] = exp_ref(__fdiv_rn(__fsub_rn(lg[i], mx), t));
        __syncthreads();
        if (tid < 32) {
            float sum = 0.0f;
            ordered_scan_warp<false>(key, V, sum, [](float) { return false; });
            if (tid == 0) red[1] = sum;
        }
        __syncthreads();
        const float sum = red[1];
        for (int i = tid; i < V; i += blockDim.x) key[i] = __fdiv_rn(key[i], sum);
        __syncthreads();
        if (tid < 32) {
            float cum = 0.0f;
            const int i = ordered_scan_warp<false>(key, V, cum, [u](float c) { return u <= c; });
            if (tid == 0) out[b] = i < V ? i : V - 1;
        }
        return;
    }
    {
        const int lane = tid & 31, w = tid >> 5;
        uint32_t k[SORT_IPT], pv[SORT_IPT];
#pragma unroll
        for (int r = 0; r < SORT_IPT; r++) {
            if (r < R) {
                const int j = w * 32 * R + r * 32 + lane;
                k[r] = j < V ? desc_key(lg[j]) : 0xffffffffu;  // padding sorts after every real entry
                pv[r] = (uint32_t)(j < V ? j : 0xffff) << 16;
            }
        }
        if (!block_bucket_sort(k, pv, R, V, ks, vs, hist, red, wsum, wmax))
            block_radix_sort(k, pv, R, ks, vs, hist, wsum);
    }
    const float mx = key_value(ks[0]);
    const int nn = top_p ? V : (int)cfg.top_k;
    __syncthreads();
    // exponentials in sorted order, in place of the keys
    for (int i = tid; i < nn; i += blockDim.x) key[i] = exp_ref(__fdiv_rn(__fsub_rn(key_value(ks[i]), mx), t));
    __syncthreads();
    if (tid < 32) {
        float total = 0.0f;
        ordered_scan_warp<true>(key, nn, total, [](float) { return false; });
        if (tid == 0) red[0] = total;
    }
    __syncthreads();
    const float total = red[0];
    for (int i = tid; i < nn; i += blockDim.x) key[i] = __fdiv_rn(key[i], total);  // the normalised terms
    __syncthreads();
    if (tid >= 32) return;
    float cum = 0.0f;
    int i;
    if (top_p) {
        // src/engine.cpp:972-1002: normalise, cut at cumulative >= p, draw
        // without renormalising.  The draw stops at the first u <= cum; the cut
        // at the first cum >= p keeps entries 0..i, and a draw that found no
        // entry by then takes the last kept one, entry i.  Either way the
        // token is the entry where the first of the two holds.
        const float p = cfg.top_p;
        i = ordered_scan_warp<true>(key, nn, cum, [u, p](float c) { return u <= c || c >= p; });
    } else {  // top-k (src/engine.cpp:930-959)
        i = ordered_scan_warp<true>(key, nn, cum, [u](float c) { return u <= c; });
    }
    if (tid == 0) out[b] = (int)vs[i < nn ? i : nn - 1];
}

pf_status sample_rows(const float* logits, int ld, int V, const int* rows, int n, const pf_sampling_config& cfg,
                      const float* uniforms, int ustride, int* out, cudaStream_t st) {
    PF_CHECK(V >= 1 && V <= SORT_THREADS * SORT_IPT, "sample_rows: vocabulary above 16384 is not supported");
    const int R = (V + SORT_THREADS - 1) / SORT_THREADS;
    // keys + indices, then the bucket counters (the radix histogram shares their space)
    constexpr size_t kCounters = SORT_BUCKETS * sizeof(uint32_t);
    static_assert(SORT_WARPS * SORT_RADIX * sizeof(uint32_t) <= kCounters, "histogram fits the counters");
    const size_t smem = (size_t)R * SORT_THREADS * 2 * sizeof(uint32_t) + kCounters;
    static std::atomic<uint64_t> attr{0};
    PF_TRY(raise_smem_limit(sample_kernel, SORT_THREADS * SORT_IPT * 2 * sizeof(uint32_t) + kCounters, attr));
    sample_kernel<<<n, SORT_THREADS, smem, st>>>(logits, ld, V, R, rows, n, cfg, uniforms, ustride, out);
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
// Every head at once: drafts[b][h] = tok[h * stride + b].
__global__ void put_drafts_kernel(const int* __restrict__ tok, int n, int K, int stride, int* __restrict__ drafts) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * K) return;
    const int b = i / K, h = i % K;
    drafts[i] = tok[(size_t)h * stride + b];
}
pf_status put_drafts(const int* tok, int n, int K, int stride, int* drafts, cudaStream_t st) {
    put_drafts_kernel<<<ceil_div(n * K, 128), 128, 0, st>>>(tok, n, K, stride, drafts);
    return launch_check("put_drafts");
}

// ---------------------------------------------------------------------------
// Predictive FFN skip (LayerSkipController::should_skip_ffn,
// src/layer_skip.cpp:22-67): rows of a sequence in order, each compared with
// the post-norm vector of the last row whose FFN ran (committed cache at the
// start); the row skips when the RMS of the difference is below the layer's
// threshold.  The RMS delta uses the device sum order below.
// ---------------------------------------------------------------------------
namespace {
// One warp's sum of (x - ref)^2 over d: each lane adds its elements
// lane, lane+32, ... in order (loads issued 16 at a time ahead of the adds),
// then a butterfly over the lanes.  Every caller uses this order, so a
// difference computed twice is the same number.
__device__ __forceinline__ float warp_sqdiff(const float* __restrict__ x, const float* __restrict__ ref, int d,
                                             int lane) {
    float s = 0.0f;
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
    return s;
}
__device__ __forceinline__ bool skip_rule(float s, int d, float thr_l) {
    return __fsqrt_rn(__fdiv_rn(s, (float)d)) < thr_l;
}
constexpr int SKIP_PAIR_ROWS = 9;  // rows per sequence of the pairwise form (K + 1 for K <= 8)
constexpr int SKIP_PAIR_WARPS = 16;
}  // namespace

// Long row batches (prefill chunks): one warp per sequence walks its rows.
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
        const bool sk = skip_rule(warp_sqdiff(x, ref, d, lane), d, thr_l);
        if (lane == 0) skip[row0 + r] = sk ? 1 : 0;
        if (!sk) ref = x;
    }
}

// Verify steps (at most SKIP_PAIR_ROWS rows per sequence): the reference row
// of row r is the cache or one of rows 0..r-1, so the r+1 candidate
// differences of every row are computed at once, one warp per (row, candidate)
// pair, and one thread then walks the rows through that table.  Same sums and
// same decisions as the walk above, without the rows waiting on each other.
__global__ void __launch_bounds__(SKIP_PAIR_WARPS * 32)
    skip_decide_pairs_kernel(const int* __restrict__ bs_row0, const int* __restrict__ bs_n,
                             const float* __restrict__ normed, int d, const float* __restrict__ cache,
                             size_t cache_stride, float thr_l, uint8_t* __restrict__ skip) {
    __shared__ uint8_t tab[SKIP_PAIR_ROWS * (SKIP_PAIR_ROWS + 1) / 2];
    const int b = blockIdx.x;
    const int n = min(bs_n[b], SKIP_PAIR_ROWS), row0 = bs_row0[b];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const float* c = cache + (size_t)b * cache_stride;
    // pair index of (row r, candidate j): r(r+1)/2 + j, j = 0 the cache, j >= 1 row j-1
    for (int pr = w; pr < n * (n + 1) / 2; pr += SKIP_PAIR_WARPS) {
        int r = 0;
        while ((r + 1) * (r + 2) / 2 <= pr) r++;
        const int j = pr - r * (r + 1) / 2;
        const float* x = normed + (size_t)(row0 + r) * d;
        const float* ref = j == 0 ? c : normed + (size_t)(row0 + j - 1) * d;
        const bool sk = skip_rule(warp_sqdiff(x, ref, d, lane), d, thr_l);
        if (lane == 0) tab[pr] = sk ? 1 : 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int j = 0;
        for (int r = 0; r < n; r++) {
            const bool sk = tab[r * (r + 1) / 2 + j] != 0;
            skip[row0 + r] = sk ? 1 : 0;
            if (!sk) j = r + 1;
        }
    }
}

pf_status skip_decide(int nb, const int* bs_row0, const int* bs_n, int max_rows, const float* normed, int d,
                      const float* cache, size_t cache_stride, float thr_l, uint8_t* skip, cudaStream_t st) {
    if (nb <= 0) return PF_OK;
    if (max_rows <= SKIP_PAIR_ROWS)
        skip_decide_pairs_kernel<<<nb, SKIP_PAIR_WARPS * 32, 0, st>>>(bs_row0, bs_n, normed, d, cache, cache_stride,
                                                                       thr_l, skip);
    else
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

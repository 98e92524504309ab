// engine.cu — the batched MTP speculative-decode engine (host side).
//
// One engine per GPU holds a full replica of the model (packed weights, tied
// embedding, MTP heads), the 3-tier KV cache of up to max_seqs sequences and
// every activation buffer, all allocated once at creation.  A decode step is
// a fixed sequence of kernels on one stream with no host synchronisation, so
// it is captured once into a CUDA graph and replayed.
//
// Reference mapping: Engine::generate's MTP loop (src/engine.cpp:304-373),
// forward_with_hidden (:459-589), compute_attention (:646-799), compute_ffn
// (:805-854), MTPHeads::forward (src/mtp.cpp:47-129), KVCache
// (src/kv_cache.cpp), LayerSkipController (src/layer_skip.cpp).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <random>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"
#include "gemm_tc.cuh"
#include "kv.cuh"
#include "rows.cuh"
#include "step.cuh"

using namespace pf;

namespace {

constexpr int kUniformSteps = 64;  // uniforms pre-drawn per sequence (steps)

template <typename T>
pf_status dalloc(T** p, size_t n, std::vector<void*>& owned) {
    *p = nullptr;
    if (n == 0) return PF_OK;
    const cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T));
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("cudaMalloc of %zu bytes failed: %s", n * sizeof(T), cudaGetErrorString(e));
        return PF_ERR_OOM;
    }
    owned.push_back(*p);
    return PF_OK;
}

}  // namespace

__global__ void pack_step_kernel(int n, int R, const int* __restrict__ n_emitted, const int* __restrict__ emitted,
                                 const int* __restrict__ seq_len, const uint32_t* __restrict__ err, int* __restrict__ out) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        out[i] = n_emitted[i];
        out[n * (R + 1) + i] = seq_len[i];
    }
    for (int i = threadIdx.x; i < n * R; i += blockDim.x) out[n + i] = emitted[i];
    if (threadIdx.x == 0) out[n * (R + 2)] = err ? (int)*err : 0;
}

static pf_status pack_step(int n, int R, const int* n_emitted, const int* emitted, const int* seq_len,
                           const uint32_t* err, int* out, cudaStream_t st) {
    pack_step_kernel<<<1, 256, 0, st>>>(n, R, n_emitted, emitted, seq_len, err, out);
    return launch_check("pack_step");
}

struct pf_engine {
    pf_model_config cfg{};
    int dev = 0;
    cudaStream_t st = nullptr;
    std::vector<void*> owned;
    int max_seqs = 0, max_pos = 0, K = 0, R = 0, Mv = 0, Mcap = 0;
    int d = 0, H = 0, G = 0, hd = 64, F = 0, V = 0, L = 0, NQ = 0, NK = 0, NQKV = 0;
    int fmt_qkv = WF_Q4, fmt_o = WF_Q4, fmt_gu = WF_Q4, fmt_down = WF_Q4, fmt_emb = WF_Q4;
    bool skip_on = false;
    float skip_thr = 0.0f;
    bool evicting = false;

    // weights
    std::vector<void*> w_qkv, w_o, w_gu, w_down;
    std::vector<float*> s_qkv, s_o, s_gu, s_down;
    std::vector<uint32_t> loaded;  // bit mask of matrices set per layer
    std::vector<std::vector<int8_t>> pend;   // host copies of fused matrices until complete
    std::vector<std::vector<float>> pend_s;
    int8_t* emb_i8 = nullptr;
    void* emb_packed = nullptr;
    float emb_gscale = 1.0f;
    bool emb_set = false;
    float *attn_norm = nullptr, *ffn_norm = nullptr, *final_norm = nullptr;
    std::vector<void*> mtp_gu, mtp_down;
    std::vector<float*> mtp_gu_s, mtp_down_s;
    std::vector<bool> mtp_set;
    float *rope_cos = nullptr, *rope_sin = nullptr;

    // cache
    KvCache kv;
    // activations
    float* x = nullptr;
    int8_t* xq = nullptr;
    float* xs = nullptr;
    float* qkv = nullptr;
    float* att = nullptr;
    float* act = nullptr;
    Staged stage{};
    SpecPool sp{};
    float* normed_all = nullptr;
    uint8_t* skip_all = nullptr;
    float* skip_cache = nullptr;
    long long* ffn_counts = nullptr;
    int8_t* digits = nullptr;
    float* dscale = nullptr;
    float* logits = nullptr;
    float* mtp_in = nullptr;   // [max_seqs][d] MTP input (hidden of the row that produced `pending`)
    float* mtp_cur = nullptr;
    float* mtp_logits = nullptr;
    int* mtp_tok = nullptr;            // [K][max_seqs]
    int8_t* mdig = nullptr;            // every head's output digit planes, [3][K * max_seqs][d]
    float* mdscale = nullptr;          // [K * max_seqs]
    int* next = nullptr;
    int* iota = nullptr;
    int* last_row = nullptr;
    float* uniforms = nullptr;  // [kUniformSteps][max_seqs][R]
    int* ustep = nullptr;
    float* cur_u = nullptr;     // [max_seqs][R]
    StepBufs sb{};
    int32_t* gws = nullptr;
    int* gcnt = nullptr;
    size_t gws_elems = 0, gcnt_elems = 0;
    // int32 partial products of the K-split projections, [splits][M][N]: O
    // and down (summed by resid_rmsnorm_quant), QKV (summed by qkv_finish).
    int32_t* rws = nullptr;
    size_t rws_elems = 0;
    // Split-context attention: partial softmax states and arrival counters.
    static constexpr int kMaxAttnSplits = 8;
    int attn_splits = 0;  // 0: automatic
    float* attn_part = nullptr;
    int* attn_cnt = nullptr;
    size_t attn_part_floats = 0, attn_cnt_elems = 0;

    pf_sampling_config samp{0.8f, 0.95f, 40, 1};
    std::vector<std::mt19937> rngs;
    int u_filled = 0;  // steps of uniforms uploaded and not yet consumed
    int n_seqs = 0;
    bool prefilled = false;
    std::vector<int> host_len;  // host view of the committed lengths (upper bound)

    cudaGraphExec_t graph = nullptr;
    bool graph_dirty = true;
    int graph_kernels = 0;  // kernel nodes of the captured step
    int graph_n = -1;       // sequences the captured step was built for
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    float last_ms = 0.0f;
    // What the host reads after every step, packed on the device and copied
    // once into pinned memory by the step graph: [n_emitted n][emitted n R]
    // [seq_len n][device error flag].
    int* dpack = nullptr;
    int* hpin = nullptr;
    // Optional per-kernel timing: event pairs captured into the step graph
    // around every attention (category 0) and projection (category 1) launch.
    static constexpr int kTimedLaunches = 512;
    bool ktiming = false;
    std::vector<cudaEvent_t> kev;  // 2 * kTimedLaunches
    std::vector<int> kev_cat;
    int kev_used = 0;
    bool kev_over = false;

    ~pf_engine() {
        if (graph) cudaGraphExecDestroy(graph);
        if (hpin) cudaFreeHost(hpin);
        for (cudaEvent_t v : kev) cudaEventDestroy(v);
        if (ev0) cudaEventDestroy(ev0);
        if (ev1) cudaEventDestroy(ev1);
        for (void* p : owned) cudaFree(p);
        if (st) cudaStreamDestroy(st);
    }

    bool greedy() const { return samp.greedy || samp.temperature <= 0.0f; }

    float layer_threshold(int l) const {  // src/layer_skip.cpp:46-55
        const int mid = L / 2;
        float t = skip_thr;
        if (l > mid / 2 && l < mid + mid / 2) t *= 2.0f;
        if (l < 2 || l >= L - 2) t = -1.0f;
        return t;
    }

    // Projections run on the tcgen05 kernel (gemm_tc.cu); digit-plane
    // activations are laid out [3][Mcap][lda].
    pf_status tbegin(int cat) {
        if (!ktiming) return PF_OK;
        if (kev_used >= kTimedLaunches) {
            kev_over = true;
            return PF_OK;
        }
        kev_cat[kev_used] = cat;
        PF_CUDA(cudaEventRecordWithFlags(kev[2 * kev_used], st, cudaEventRecordExternal));
        return PF_OK;
    }
    pf_status tend() {
        if (!ktiming || kev_used >= kTimedLaunches) return PF_OK;
        PF_CUDA(cudaEventRecordWithFlags(kev[2 * kev_used + 1], st, cudaEventRecordExternal));
        kev_used++;
        return PF_OK;
    }

    pf_status gemm(GemmParams p, int planes) {
        // Whole-K tiles: at these shapes the split-K reduction costs more
        // than the idle SMs it fills.
        p.splits = 1;
        p.pdl = true;
        p.ws = gws;
        p.counters = gcnt;
        p.ws_elems = gws_elems;
        p.cnt_elems = gcnt_elems;
        PF_TRY(tbegin(1));
        PF_TRY(gemm_tc_launch(p, planes, Mcap, st));
        return tend();
    }

    // ---- one pass of all layers over a row batch ---------------------------------
    // A residual projection (O or down) whose K-split int32 slices are still
    // to be added to x; the next RMSNorm kernel adds them.
    struct PendingResid {
        int parts = 0;
        const float* w_scale = nullptr;
        const uint8_t* row_skip = nullptr;
    };

    // O / down projection into rws slices: x += (xq . W^T) * scales happens
    // in resid_rmsnorm_quant.
    pf_status resid_gemm(const void* W, int wf, const float* w_scale, int M, int K, const uint8_t* row_skip,
                         PendingResid* pend) {
        GemmParams p;
        p.A = xq; p.lda = K; p.a_scale = xs; p.M = M; p.N = d; p.K = K;
        p.W = W; p.wf = wf; p.w_scale = w_scale;
        p.epi = EPI_I32; p.out_i32 = rws; p.ldo = d;
        p.splits = gemm_tc_slices(M, d, K);
        p.slice_stride = (int64_t)M * d;
        PF_CHECK((size_t)p.splits * M * d <= rws_elems, "residual workspace too small");
        p.pdl = true;
        PF_TRY(tbegin(1));
        PF_TRY(gemm_tc_launch(p, 1, Mcap, st));
        PF_TRY(tend());
        pend->parts = p.splits;
        pend->w_scale = w_scale;
        pend->row_skip = row_skip;
        return PF_OK;
    }

    // x += pending residual (if any), then RMSNorm with `norm` + quantization
    // into xq / xs (norm == nullptr: only the residual).
    pf_status norm_rows(PendingResid* pend, const float* norm, int M, float* normed) {
        if (pend->parts == 0) {
            if (!norm) return PF_OK;
            return rmsnorm_quant(x, norm, d, cfg.norm_eps, M, nullptr, normed, xq, xs, d, st);
        }
        const int parts = pend->parts;
        pend->parts = 0;
        return resid_rmsnorm_quant(x, rws, parts, (int64_t)M * d, xs, pend->w_scale, pend->row_skip, norm, d,
                                   cfg.norm_eps, M, normed, norm ? xq : nullptr, xs, d, st);
    }

    pf_status layers(const RowBatch& rb, int M) {
        const size_t sM = (size_t)Mcap;
        PendingResid pend;
        for (int l = 0; l < L; l++) {
            Staged sl;
            sl.k = stage.k + (size_t)l * sM * G * 64;
            sl.v = stage.v + (size_t)l * sM * G * 64;
            sl.ks = stage.ks + (size_t)l * sM * G;
            sl.vs = stage.vs + (size_t)l * sM * G;
            PF_TRY(norm_rows(&pend, attn_norm + (size_t)l * d, M, nullptr));
            {
                // K split into int32 slices (the tiles alone fill half the SMs);
                // qkv_finish applies the scales and RoPE and stages K / V.
                GemmParams p;
                p.A = xq; p.lda = d; p.a_scale = xs; p.M = M; p.N = NQKV; p.K = d;
                p.W = w_qkv[l]; p.wf = fmt_qkv; p.w_scale = s_qkv[l];
                p.epi = EPI_I32; p.out_i32 = rws; p.ldo = NQKV;
                p.splits = gemm_tc_slices(M, NQKV, d);
                p.slice_stride = (int64_t)M * NQKV;
                PF_CHECK((size_t)p.splits * M * NQKV <= rws_elems, "projection workspace too small");
                p.pdl = true;
                PF_TRY(tbegin(1));
                PF_TRY(gemm_tc_launch(p, 1, Mcap, st));
                PF_TRY(tend());
                PF_TRY(qkv_finish(rws, p.splits, p.slice_stride, xs, s_qkv[l], NQKV, M, rope_cos, rope_sin, rb.row_pos,
                                  NQ + NK, hd, qkv, NQ, NQ + NK, G, sl, st));
            }
            if (evicting) PF_TRY(kv_pool_spec(kv, l, rb, sp, st));
            PF_TRY(tbegin(0));
            if (attention_decode_supported(kv, H, rb.max_rows)) {
                AttnWork aw;
                const int nrg = attention_decode_row_groups(kv, H, rb.max_rows);
                aw.nsplit = attn_splits > 0 ? attn_splits : attention_decode_splits(rb.nb * nrg, G, kMaxAttnSplits);
                // (wide prefill batches have row groups enough: no split there)
                if (attention_decode_work_floats(rb.nb, G, aw.nsplit, nrg) > attn_part_floats ||
                    (size_t)rb.nb * G * nrg > attn_cnt_elems)
                    aw.nsplit = 1;
                aw.part = attn_part;
                aw.part_floats = attn_part_floats;
                aw.cnt = attn_cnt;
                aw.cnt_elems = attn_cnt_elems;
                PF_TRY(attention_decode(kv, l, rb, qkv, NQKV, NQ, NQ + NK, H, sl, sp, aw, att, NQ, st));
            }
            else
                PF_TRY(attention(kv, l, rb, qkv, NQKV, NQ, NQ + NK, H, sl, sp, att, NQ, st));
            PF_TRY(tend());
            PF_TRY(quant_rows(att, NQ, NQ, M, nullptr, xq, xs, NQ, st));
            PF_TRY(resid_gemm(w_o[l], fmt_o, s_o[l], M, NQ, nullptr, &pend));
            float* normed = skip_on ? normed_all + (size_t)l * sM * d : nullptr;
            uint8_t* skipl = skip_on ? skip_all + (size_t)l * sM : nullptr;
            PF_TRY(norm_rows(&pend, ffn_norm + (size_t)l * d, M, normed));
            if (skip_on)
                PF_TRY(skip_decide(rb.nb, rb.row0, rb.n, rb.max_rows, normed, d, skip_cache + (size_t)l * d,
                                   (size_t)L * d, layer_threshold(l), skipl, st));
            {
                GemmParams p;
                p.A = xq; p.lda = d; p.a_scale = xs; p.M = M; p.N = 2 * F; p.K = d;
                p.W = w_gu[l]; p.wf = fmt_gu; p.w_scale = s_gu[l];
                p.epi = EPI_SWIGLU; p.out = act; p.ldo = F;
                PF_TRY(gemm(p, 1));
            }
            PF_TRY(quant_rows(act, F, F, M, nullptr, xq, xs, F, st));
            PF_TRY(resid_gemm(w_down[l], fmt_down, s_down[l], M, F, skipl, &pend));
        }
        return norm_rows(&pend, nullptr, M, nullptr);  // the last layer's residual
    }

    // Tied unembed of n rows of `src` (pre-final-norm hidden) into out [n][V].
    pf_status unembed(const float* src, int n, float* out) {
        const int64_t plane = (int64_t)Mcap * d;
        PF_TRY(split_digits(src, d, d, n, nullptr, digits, plane, d, dscale, st));
        GemmParams p;
        p.A = digits; p.plane_stride = plane; p.lda = d; p.a_scale = dscale; p.M = n; p.N = V; p.K = d;
        p.W = emb_packed; p.wf = fmt_emb; p.w_scale_all = emb_gscale;
        p.epi = EPI_LOGITS3; p.out = out; p.ldo = V;
        return gemm(p, 3);
    }

    // One MTP projection over the digit planes of n rows stacked along M
    // ([3][n][d]): K split into int32 slices in rws; returns the split count.
    pf_status mtp_gemm(const void* W, int N, int n, int* parts) {
        GemmParams p;
        p.A = digits; p.lda = d; p.M = 3 * n; p.N = N; p.K = d;
        p.W = W; p.wf = WF_Q4;
        p.epi = EPI_I32; p.out_i32 = rws; p.ldo = N;
        p.splits = gemm_tc_slices(3 * n, N, d);
        p.slice_stride = (int64_t)3 * n * N;
        PF_CHECK((size_t)p.splits * 3 * n * N <= rws_elems, "projection workspace too small");
        p.pdl = true;
        PF_TRY(tbegin(1));
        PF_TRY(gemm_tc_launch(p, 1, 3 * n, st));
        PF_TRY(tend());
        *parts = p.splits;
        return PF_OK;
    }

    // MTP heads on mtp_cur (n rows): drafts[b][h] (MTPHeads::forward, src/mtp.cpp:47-129).
    // The digit planes of the rows feed each projection as 3 n stacked rows;
    // each finishing kernel applies the projection's epilogue and splits its
    // result for the next one (the head's residual output also feeds the
    // unembedding and the next head).
    pf_status mtp_chain(int n) {
        if (K == 0 || n == 0) return PF_OK;
        const int64_t plane = (int64_t)n * d;
        PF_TRY(split_digits(mtp_cur, d, d, n, nullptr, digits, plane, d, dscale, st));
        for (int h = 0; h < K; h++) {
            int parts = 0;
            PF_TRY(mtp_gemm(mtp_gu[h], 2 * d, n, &parts));
            PF_TRY(mtp_finish(true, rws, parts, (int64_t)3 * n * 2 * d, dscale, mtp_gu_s[h], d, n, nullptr, digits,
                              dscale, st));
            PF_TRY(mtp_gemm(mtp_down[h], d, n, &parts));
            PF_TRY(mtp_finish(false, rws, parts, (int64_t)3 * n * d, dscale, mtp_down_s[h], d, n, mtp_cur, digits,
                              dscale, st, mdig + (size_t)h * max_seqs * d, (int64_t)K * max_seqs * d,
                              mdscale + (size_t)h * max_seqs));
        }
        // The heads' unembeddings depend only on their own hidden states, so
        // they run as one launch over every head's rows (K * max_seqs rows,
        // rows h * max_seqs + b), not as K launches of n rows each.
        {
            const int MK = K * max_seqs;
            GemmParams p;
            p.A = mdig; p.plane_stride = (int64_t)MK * d; p.lda = d; p.a_scale = mdscale; p.M = MK; p.N = V; p.K = d;
            p.W = emb_packed; p.wf = fmt_emb; p.w_scale_all = emb_gscale;
            p.epi = EPI_LOGITS3; p.out = mtp_logits; p.ldo = V;
            p.splits = 1;
            p.pdl = true;
            PF_TRY(tbegin(1));
            PF_TRY(gemm_tc_launch(p, 3, MK, st));
            PF_TRY(tend());
            if (greedy()) {
                PF_TRY(argmax_rows(mtp_logits, V, V, MK, nullptr, mtp_tok, st));
            } else {
                for (int h = 0; h < K; h++)
                    PF_TRY(sample_rows(mtp_logits + (size_t)h * max_seqs * V, V, V, iota, n, samp, cur_u + 1 + h, R,
                                       mtp_tok + (size_t)h * max_seqs, st));
            }
            PF_TRY(put_drafts(mtp_tok, n, K, max_seqs, sb.drafts, st));
        }
        return PF_OK;
    }

    pf_status select_uniforms();

    // The device work of one decode step (capturable).
    pf_status enqueue_step() {
        kev_used = 0;
        kev_over = false;
        const int n = n_seqs, M = n * R;
        StepBufs s = sb;
        s.n_seqs = n;
        PF_TRY(verify_setup(s, st));
        if (!greedy()) PF_TRY(select_uniforms());
        PF_TRY(embed(emb_i8, emb_gscale, d, V, s.row_tok, M, nullptr, x, st));
        RowBatch rb;
        rb.nb = n; rb.M = M; rb.row0 = s.bs_row0; rb.n = s.bs_n; rb.len0 = s.bs_len0; rb.row_pos = s.row_pos;
        rb.max_rows = R;
        PF_TRY(layers(rb, M));
        PF_TRY(unembed(x, M, logits));
        PF_TRY(argmax_rows(logits, V, V, M, nullptr, s.amax, st));
        PF_TRY(accept(s, st));
        if (greedy()) PF_TRY(pick(s.amax, s.final_row, n, next, st));
        else PF_TRY(sample_rows(logits, V, V, s.final_row, n, samp, cur_u, R, next, st));
        PF_TRY(finish(s, next, st));
        PF_TRY(kv_commit(kv, rb, s.n_commit, stage, Mcap, st));
        if (skip_on)
            PF_TRY(skip_commit(n, L, d, Mcap, s.bs_row0, s.n_commit, skip_all, normed_all, skip_cache, ffn_counts, st));
        else
            PF_TRY(ffn_count(n, L, s.n_commit, ffn_counts, st));
        PF_TRY(gather_rows(x, d, s.final_row, n, mtp_in, st));
        PF_CUDA(cudaMemcpyAsync(mtp_cur, mtp_in, (size_t)n * d * sizeof(float), cudaMemcpyDeviceToDevice, st));
        PF_TRY(mtp_chain(n));
        // the step's results for the host, one copy into pinned memory
        PF_TRY(pack_step(n, R, sb.n_emitted, sb.emitted, sb.seq_len, device_error_flag(), dpack, st));
        PF_CUDA(cudaMemcpyAsync(hpin, dpack, pack_bytes(n), cudaMemcpyDeviceToHost, st));
        return PF_OK;
    }
    size_t pack_bytes(int n) const { return (size_t)(n * (R + 2) + 1) * sizeof(int); }

    pf_status fill_uniforms(int steps);
};

// Uniform draws: per sequence and step, R values in the order the reference
// would draw them — the token after the accepted prefix first, then drafts
// 0..K-1 — from the sequence's own std::mt19937 (src/engine.cpp:16,996).
__global__ void select_uniforms_kernel(const float* __restrict__ all, int n_per_step, int* __restrict__ ustep,
                                       float* __restrict__ cur) {
    const int s = *ustep;
    for (int i = threadIdx.x; i < n_per_step; i += blockDim.x) cur[i] = all[(size_t)(s % kUniformSteps) * n_per_step + i];
    __syncthreads();
    if (threadIdx.x == 0) *ustep = s + 1;
}

pf_status pf_engine::select_uniforms() {
    select_uniforms_kernel<<<1, 256, 0, st>>>(uniforms, max_seqs * R, ustep, cur_u);
    return launch_check("select_uniforms");
}

pf_status pf_engine::fill_uniforms(int steps) {
    if (greedy()) return PF_OK;
    PF_CHECK(steps <= kUniformSteps, "at most %d stochastic steps per call", kUniformSteps);
    std::vector<float> h((size_t)steps * max_seqs * R, 0.0f);
    for (int t = 0; t < steps; t++)
        for (int b = 0; b < n_seqs; b++)
            for (int r = 0; r < R; r++)
                h[((size_t)t * max_seqs + b) * R + r] = std::uniform_real_distribution<float>(0.0f, 1.0f)(rngs[b]);
    // The device consumes slot (ustep % kUniformSteps); reset the counter so
    // the next `steps` steps read slots 0..steps-1.
    PF_CUDA(cudaMemcpyAsync(uniforms, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice, st));
    PF_CUDA(cudaMemsetAsync(ustep, 0, sizeof(int), st));
    return PF_OK;
}

// ============================================================================
// C ABI
// ============================================================================
extern "C" {

pf_status pf_engine_create(const pf_model_config* c, int32_t max_seqs, int32_t max_positions, int32_t device,
                           pf_engine** out) {
    PF_CHECK(c && out, "pf_engine_create: null argument");
    *out = nullptr;
    PF_CHECK(max_seqs > 0 && max_positions > 0, "pf_engine_create: bad sizes");
    PF_CHECK(c->head_dim == 64, "head_dim must be 64 (got %d)", c->head_dim);
    PF_CHECK(c->n_heads * c->head_dim == c->n_embd, "n_heads*head_dim must equal n_embd");
    PF_CHECK(c->n_heads % c->n_kv_heads == 0 && c->n_heads / c->n_kv_heads <= 8, "n_heads/n_kv_heads must be 1..8");
    PF_CHECK(c->n_embd % 128 == 0 && c->n_ff % 128 == 0, "n_embd and n_ff must be multiples of 128");
    PF_CHECK(c->n_vocab % 64 == 0 && c->n_vocab <= 16384, "n_vocab must be a multiple of 64 and <= 16384");
    PF_CHECK(c->n_mtp_heads >= 1 && c->n_mtp_heads <= 8, "n_mtp_heads must be 1..8");
    PF_CHECK(c->sink_size >= 0 && c->sink_size <= 8, "sink_size must be 0..8");
    PF_CHECK(c->pool_block >= 1 && c->window_size >= 1, "bad window/pool");
    PF_CHECK(max_positions <= c->max_context, "max_positions must not exceed max_context");
    for (int m = 0; m < 3; m++)
        PF_CHECK(wfmt_of_qtype(c->qtype[m]) == wfmt_of_qtype(c->qtype[0]), "Q, K and V must share a weight format");
    PF_CHECK(wfmt_of_qtype(c->qtype[PF_MAT_GATE]) == wfmt_of_qtype(c->qtype[PF_MAT_UP]),
             "gate and up must share a weight format");
    PF_TRY(require_device());
    PF_CUDA(cudaSetDevice(device));
    PF_TRY(require_device());
    // The device's error latch is shared by every caller on the device;
    // flags latched before this engine existed are not its errors.
    if (uint32_t* flag = device_error_flag()) PF_CUDA(cudaMemset(flag, 0, sizeof(uint32_t)));

    auto* e = new pf_engine();
    auto fail = [&](pf_status s) {
        delete e;
        return s;
    };
#define E_TRY(x)                         \
    do {                                 \
        pf_status _s = (x);              \
        if (_s != PF_OK) return fail(_s);\
    } while (0)
    e->cfg = *c;
    e->dev = device;
    if (cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking) != cudaSuccess) return fail(PF_ERR_CUDA);
    cudaEventCreate(&e->ev0);
    cudaEventCreate(&e->ev1);
    e->max_seqs = max_seqs;
    e->max_pos = max_positions;
    e->K = c->n_mtp_heads;
    e->R = e->K + 1;
    e->Mv = max_seqs * e->R;
    e->Mcap = std::max(e->Mv, std::min(8192, max_seqs * 256));
    e->d = c->n_embd;
    e->H = c->n_heads;
    e->G = c->n_kv_heads;
    e->F = c->n_ff;
    e->V = c->n_vocab;
    e->L = c->n_layers;
    e->NQ = e->H * 64;
    e->NK = e->G * 64;
    e->NQKV = e->NQ + 2 * e->NK;
    e->fmt_qkv = wfmt_of_qtype(c->qtype[0]);
    e->fmt_o = wfmt_of_qtype(c->qtype[PF_MAT_O]);
    e->fmt_gu = wfmt_of_qtype(c->qtype[PF_MAT_GATE]);
    e->fmt_down = wfmt_of_qtype(c->qtype[PF_MAT_DOWN]);
    e->fmt_emb = wfmt_of_qtype(c->emb_qtype);
    e->skip_on = c->skip_enabled != 0;
    e->skip_thr = c->skip_threshold;
    const int L = e->L, d = e->d, F = e->F, V = e->V, G = e->G;
    auto& o = e->owned;

    // weights
    e->w_qkv.assign(L, nullptr); e->w_o.assign(L, nullptr); e->w_gu.assign(L, nullptr); e->w_down.assign(L, nullptr);
    e->s_qkv.assign(L, nullptr); e->s_o.assign(L, nullptr); e->s_gu.assign(L, nullptr); e->s_down.assign(L, nullptr);
    e->loaded.assign(L, 0);
    for (int l = 0; l < L; l++) {
        uint8_t* p;
        E_TRY(dalloc(&p, packed_bytes_tc(e->NQKV, d, e->fmt_qkv), o)); e->w_qkv[l] = p;
        E_TRY(dalloc(&p, packed_bytes_tc(d, e->NQ, e->fmt_o), o)); e->w_o[l] = p;
        E_TRY(dalloc(&p, packed_bytes_tc(2 * F, d, e->fmt_gu), o)); e->w_gu[l] = p;
        E_TRY(dalloc(&p, packed_bytes_tc(d, F, e->fmt_down), o)); e->w_down[l] = p;
        E_TRY(dalloc(&e->s_qkv[l], e->NQKV, o));
        E_TRY(dalloc(&e->s_o[l], d, o));
        E_TRY(dalloc(&e->s_gu[l], 2 * F, o));
        E_TRY(dalloc(&e->s_down[l], d, o));
    }
    E_TRY(dalloc(&e->emb_i8, (size_t)V * d, o));
    {
        uint8_t* p;
        E_TRY(dalloc(&p, packed_bytes_tc(V, d, e->fmt_emb), o));
        e->emb_packed = p;
    }
    E_TRY(dalloc(&e->attn_norm, (size_t)L * d, o));
    E_TRY(dalloc(&e->ffn_norm, (size_t)L * d, o));
    E_TRY(dalloc(&e->final_norm, (size_t)d, o));
    {
        std::vector<float> ones((size_t)L * d, 1.0f);
        PF_CUDA(cudaMemcpy(e->attn_norm, ones.data(), ones.size() * 4, cudaMemcpyHostToDevice));
        PF_CUDA(cudaMemcpy(e->ffn_norm, ones.data(), ones.size() * 4, cudaMemcpyHostToDevice));
        PF_CUDA(cudaMemcpy(e->final_norm, ones.data(), (size_t)d * 4, cudaMemcpyHostToDevice));
    }
    e->mtp_gu.assign(e->K, nullptr); e->mtp_down.assign(e->K, nullptr);
    e->mtp_gu_s.assign(e->K, nullptr); e->mtp_down_s.assign(e->K, nullptr);
    e->mtp_set.assign(e->K, false);
    for (int h = 0; h < e->K; h++) {
        uint8_t* p;
        E_TRY(dalloc(&p, packed_bytes_tc(2 * d, d, WF_Q4), o)); e->mtp_gu[h] = p;
        E_TRY(dalloc(&p, packed_bytes_tc(d, d, WF_Q4), o)); e->mtp_down[h] = p;
        E_TRY(dalloc(&e->mtp_gu_s[h], 2 * d, o));
        E_TRY(dalloc(&e->mtp_down_s[h], d, o));
    }
    // RoPE table with the reference's float library calls (src/engine.cpp:660-668).
    {
        const int half = 32;
        std::vector<float> cs((size_t)max_positions * half), sn((size_t)max_positions * half);
        for (int pos = 0; pos < max_positions; pos++)
            for (int i = 0; i < 64; i += 2) {
                const float freq = 1.0f / std::pow(c->rope_theta, (float)i / (float)64);
                cs[(size_t)pos * half + i / 2] = std::cos((float)pos * freq);
                sn[(size_t)pos * half + i / 2] = std::sin((float)pos * freq);
            }
        E_TRY(dalloc(&e->rope_cos, cs.size(), o));
        E_TRY(dalloc(&e->rope_sin, sn.size(), o));
        PF_CUDA(cudaMemcpy(e->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
        PF_CUDA(cudaMemcpy(e->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    }

    // KV cache
    KvCache& kv = e->kv;
    kv.n_seqs = max_seqs; kv.L = L; kv.G = G; kv.hd = 64;
    kv.S = c->sink_size; kv.pb = c->pool_block; kv.max_pos = max_positions;
    kv.Wr = std::min(c->window_size, c->max_context);
    kv.W_alloc = std::max(1, std::min(kv.Wr, max_positions - kv.S));
    kv.P_max = (max_positions - kv.S - kv.Wr > 0) ? (max_positions - kv.S - kv.Wr) / kv.pb + 1 : 1;
    kv.W_pad = ceil_div(kv.W_alloc, 32) * 32;
    kv.P_pad = ceil_div(kv.P_max, 32) * 32;
    e->evicting = max_positions - kv.S > kv.Wr;
    const size_t units = (size_t)max_seqs * L * G;
    E_TRY(dalloc(&kv.ring_k, units * kv.W_pad * 64, o));
    E_TRY(dalloc(&kv.ring_v, units * kv.W_pad * 64, o));
    E_TRY(dalloc(&kv.ring_ks, units * kv.W_pad, o));
    E_TRY(dalloc(&kv.ring_vs, units * kv.W_pad, o));
    E_TRY(dalloc(&kv.sink_k, units * std::max(1, kv.S) * 64, o));
    E_TRY(dalloc(&kv.sink_v, units * std::max(1, kv.S) * 64, o));
    E_TRY(dalloc(&kv.sink_ks, units * std::max(1, kv.S), o));
    E_TRY(dalloc(&kv.sink_vs, units * std::max(1, kv.S), o));
    E_TRY(dalloc(&kv.pool_k, units * kv.P_pad * 64, o));
    E_TRY(dalloc(&kv.pool_v, units * kv.P_pad * 64, o));
    E_TRY(dalloc(&kv.pool_ks, units * kv.P_pad, o));
    E_TRY(dalloc(&kv.pool_vs, units * kv.P_pad, o));
    E_TRY(dalloc(&kv.acc_k, units * 64, o));
    E_TRY(dalloc(&kv.acc_v, units * 64, o));
    // zero-filled so that padding slots read by whole-block loads hold finite values
    PF_CUDA(cudaMemset(kv.ring_k, 0, units * kv.W_pad * 64));
    PF_CUDA(cudaMemset(kv.ring_v, 0, units * kv.W_pad * 64));
    PF_CUDA(cudaMemset(kv.ring_ks, 0, units * kv.W_pad * 4));
    PF_CUDA(cudaMemset(kv.ring_vs, 0, units * kv.W_pad * 4));
    PF_CUDA(cudaMemset(kv.pool_k, 0, units * kv.P_pad * 64));
    PF_CUDA(cudaMemset(kv.pool_v, 0, units * kv.P_pad * 64));
    PF_CUDA(cudaMemset(kv.pool_ks, 0, units * kv.P_pad * 4));
    PF_CUDA(cudaMemset(kv.pool_vs, 0, units * kv.P_pad * 4));

    // activations
    const size_t Mc = e->Mcap;
    const int wide = std::max(std::max(d, e->NQ), F);
    E_TRY(dalloc(&e->x, Mc * d, o));
    E_TRY(dalloc(&e->xq, Mc * wide, o));
    E_TRY(dalloc(&e->xs, Mc, o));
    E_TRY(dalloc(&e->qkv, Mc * e->NQKV, o));
    E_TRY(dalloc(&e->att, Mc * e->NQ, o));
    E_TRY(dalloc(&e->act, Mc * F, o));
    E_TRY(dalloc(&e->stage.k, (size_t)L * Mc * G * 64, o));
    E_TRY(dalloc(&e->stage.v, (size_t)L * Mc * G * 64, o));
    E_TRY(dalloc(&e->stage.ks, (size_t)L * Mc * G, o));
    E_TRY(dalloc(&e->stage.vs, (size_t)L * Mc * G, o));
    // new pool entries one batch can finalize for a sequence (rows per sequence <= Mcap)
    e->sp.per = ceil_div((int)Mc, kv.pb) + 2;
    E_TRY(dalloc(&e->sp.k, (size_t)max_seqs * G * e->sp.per * 64, o));
    E_TRY(dalloc(&e->sp.v, (size_t)max_seqs * G * e->sp.per * 64, o));
    E_TRY(dalloc(&e->sp.ks, (size_t)max_seqs * G * e->sp.per, o));
    E_TRY(dalloc(&e->sp.vs, (size_t)max_seqs * G * e->sp.per, o));
    if (e->skip_on) {
        E_TRY(dalloc(&e->normed_all, (size_t)L * Mc * d, o));
        E_TRY(dalloc(&e->skip_all, (size_t)L * Mc, o));
        E_TRY(dalloc(&e->skip_cache, (size_t)max_seqs * L * d, o));
    }
    E_TRY(dalloc(&e->ffn_counts, 2, o));
    E_TRY(dalloc(&e->digits, 3 * Mc * d, o));
    E_TRY(dalloc(&e->dscale, Mc, o));
    E_TRY(dalloc(&e->logits, (size_t)e->Mv * V, o));
    E_TRY(dalloc(&e->mtp_in, (size_t)max_seqs * d, o));
    E_TRY(dalloc(&e->mtp_cur, (size_t)max_seqs * d, o));
    E_TRY(dalloc(&e->mtp_logits, (size_t)e->K * max_seqs * V, o));
    E_TRY(dalloc(&e->mtp_tok, (size_t)e->K * max_seqs, o));
    E_TRY(dalloc(&e->mdig, (size_t)3 * e->K * max_seqs * d, o));
    E_TRY(dalloc(&e->mdscale, (size_t)e->K * max_seqs, o));
    // rows of sequences not in a batch stay finite (zero digits and scales)
    if (cudaMemset(e->mdig, 0, (size_t)3 * e->K * max_seqs * d) != cudaSuccess ||
        cudaMemset(e->mdscale, 0, (size_t)e->K * max_seqs * sizeof(float)) != cudaSuccess)
        return fail(PF_ERR_CUDA);
    E_TRY(dalloc(&e->next, max_seqs, o));
    E_TRY(dalloc(&e->iota, max_seqs, o));
    E_TRY(dalloc(&e->last_row, max_seqs, o));
    {
        std::vector<int> io(max_seqs);
        for (int i = 0; i < max_seqs; i++) io[i] = i;
        PF_CUDA(cudaMemcpy(e->iota, io.data(), io.size() * 4, cudaMemcpyHostToDevice));
    }
    E_TRY(dalloc(&e->uniforms, (size_t)kUniformSteps * max_seqs * e->R, o));
    E_TRY(dalloc(&e->ustep, 1, o));
    E_TRY(dalloc(&e->cur_u, (size_t)max_seqs * e->R, o));
    StepBufs& sb = e->sb;
    sb.n_seqs = max_seqs; sb.K = e->K; sb.max_pos = max_positions;
    E_TRY(dalloc(&sb.pending, max_seqs, o));
    E_TRY(dalloc(&sb.drafts, (size_t)max_seqs * e->K, o));
    E_TRY(dalloc(&sb.seq_len, max_seqs, o));
    E_TRY(dalloc(&sb.row_tok, Mc, o));
    E_TRY(dalloc(&sb.row_pos, Mc, o));
    E_TRY(dalloc(&sb.bs_row0, max_seqs, o));
    E_TRY(dalloc(&sb.bs_n, max_seqs, o));
    E_TRY(dalloc(&sb.bs_len0, max_seqs, o));
    E_TRY(dalloc(&sb.amax, e->Mv, o));
    E_TRY(dalloc(&sb.n_commit, max_seqs, o));
    E_TRY(dalloc(&sb.final_row, max_seqs, o));
    E_TRY(dalloc(&sb.emitted, (size_t)max_seqs * e->R, o));
    E_TRY(dalloc(&sb.n_emitted, max_seqs, o));
    E_TRY(dalloc(&e->dpack, (size_t)max_seqs * (e->R + 2) + 1, o));
    if (cudaHostAlloc(reinterpret_cast<void**>(&e->hpin), ((size_t)max_seqs * (e->R + 2) + 1) * sizeof(int),
                      cudaHostAllocDefault) != cudaSuccess)
        return fail(PF_ERR_OOM);
    sb.log_cap = max_positions;
    E_TRY(dalloc(&sb.log, (size_t)max_seqs * max_positions, o));
    E_TRY(dalloc(&sb.n_logged, max_seqs, o));
    // split-K workspace (the largest single-plane projection of a verify batch)
    // split-K is only chosen below 2*148 output tiles of 64x64
    e->gws_elems = (size_t)3 * 296 * 64 * 64;
    E_TRY(dalloc(&e->gws, e->gws_elems, o));
    for (int m = 1; m <= e->Mcap; m++)  // slices of the K-split projections, any row count
        e->rws_elems = std::max({e->rws_elems,
                                 (size_t)std::max(gemm_tc_slices(m, d, e->NQ), gemm_tc_slices(m, d, F)) * m * d,
                                 (size_t)gemm_tc_slices(m, e->NQKV, d) * m * e->NQKV});
    for (int n = 1; n <= max_seqs; n++)  // the MTP heads' projections over 3 n stacked digit rows
        e->rws_elems = std::max({e->rws_elems, (size_t)gemm_tc_slices(3 * n, 2 * d, d) * 3 * n * 2 * d,
                                 (size_t)gemm_tc_slices(3 * n, d, d) * 3 * n * d});
    E_TRY(dalloc(&e->rws, e->rws_elems, o));
    e->attn_part_floats = attention_decode_work_floats(max_seqs, G, pf_engine::kMaxAttnSplits, 1);
    e->attn_cnt_elems = (size_t)max_seqs * G * pf_engine::kMaxAttnSplits;
    E_TRY(dalloc(&e->attn_part, e->attn_part_floats, o));
    E_TRY(dalloc(&e->attn_cnt, e->attn_cnt_elems, o));
    if (cudaMemset(e->attn_cnt, 0, e->attn_cnt_elems * sizeof(int)) != cudaSuccess) return fail(PF_ERR_CUDA);
    e->gcnt_elems = 296;
    E_TRY(dalloc(&e->gcnt, e->gcnt_elems, o));
    PF_CUDA(cudaMemset(e->gws, 0, e->gws_elems * 4));
    PF_CUDA(cudaMemset(e->gcnt, 0, e->gcnt_elems * 4));
    PF_CUDA(cudaMemset(e->ffn_counts, 0, 16));
    PF_CUDA(cudaDeviceSynchronize());
    *out = e;
    return PF_OK;
#undef E_TRY
}

void pf_engine_destroy(pf_engine* e) {
    if (!e) return;
    cudaSetDevice(e->dev);
    cudaStreamSynchronize(e->st);
    delete e;
}

static pf_status upload_scaled(float* dst, const float* src, size_t n, cudaStream_t st) {
    PF_CUDA(cudaMemcpyAsync(dst, src, n * sizeof(float), cudaMemcpyHostToDevice, st));
    return PF_OK;
}

// Packs a host int8 matrix into dst (format wf), rows [row0, row0+rows) of a
// taller packed matrix of `total_rows` rows are not supported: matrices that
// are fused (QKV, gate/up) are assembled on the host first.
static pf_status pack_host(pf_engine* e, const int8_t* w, int rows, int cols, int wf, void* dst) {
    int8_t* tmp = nullptr;
    PF_CUDA(cudaMallocAsync(&tmp, (size_t)rows * cols, e->st));
    pf_status s = PF_OK;
    if (cudaMemcpyAsync(tmp, w, (size_t)rows * cols, cudaMemcpyHostToDevice, e->st) != cudaSuccess) s = PF_ERR_CUDA;
    if (s == PF_OK) s = pack_weights_tc(tmp, rows, cols, wf, dst, e->st);
    cudaFreeAsync(tmp, e->st);
    if (s == PF_OK && cudaStreamSynchronize(e->st) != cudaSuccess) s = PF_ERR_CUDA;
    if (s != PF_OK) return s;
    uint32_t flag = 0;
    PF_CUDA(cudaMemcpy(&flag, device_error_flag(), 4, cudaMemcpyDeviceToHost));
    if (flag & ERR_WEIGHT_RANGE) {
        cudaMemset(device_error_flag(), 0, 4);
        set_error("weight values outside the range of their packed format");
        return PF_ERR_DEVICE;
    }
    return PF_OK;
}

pf_status pf_engine_set_matrix(pf_engine* e, int32_t layer, int32_t m, const int8_t* w, const float* rs) {
    PF_CHECK(e && w && rs, "pf_engine_set_matrix: null argument");
    PF_CHECK(layer >= 0 && layer < e->L && m >= 0 && m < PF_MAT_COUNT, "pf_engine_set_matrix: bad index");
    PF_CUDA(cudaSetDevice(e->dev));
    const int d = e->d, F = e->F;
    // Shapes (src/engine.cpp:702-714, 792-794, 822-843).
    int rows = 0, cols = 0;
    switch (m) {
        case PF_MAT_Q: rows = e->NQ; cols = d; break;
        case PF_MAT_K: case PF_MAT_V: rows = e->NK; cols = d; break;
        case PF_MAT_O: rows = d; cols = e->NQ; break;
        case PF_MAT_GATE: case PF_MAT_UP: rows = F; cols = d; break;
        default: rows = d; cols = F; break;
    }
    auto& held = e->loaded[layer];
    // QKV and gate/up are fused on the device: keep host copies until complete.
    auto& pend = e->pend;
    auto& pend_s = e->pend_s;
    const size_t key = (size_t)layer * PF_MAT_COUNT;
    if (pend.size() < (size_t)e->L * PF_MAT_COUNT) {
        pend.resize((size_t)e->L * PF_MAT_COUNT);
        pend_s.resize((size_t)e->L * PF_MAT_COUNT);
    }
    pend[key + m].assign(w, w + (size_t)rows * cols);
    pend_s[key + m].assign(rs, rs + rows);
    held |= 1u << m;
    if (m <= PF_MAT_V && (held & 7u) == 7u) {
        std::vector<int8_t> fused((size_t)e->NQKV * d);
        std::vector<float> fs(e->NQKV);
        size_t r0 = 0;
        for (int j = 0; j < 3; j++) {
            std::memcpy(fused.data() + r0 * d, pend[key + j].data(), pend[key + j].size());
            std::memcpy(fs.data() + r0, pend_s[key + j].data(), pend_s[key + j].size() * 4);
            r0 += pend_s[key + j].size();
        }
        PF_TRY(pack_host(e, fused.data(), e->NQKV, d, e->fmt_qkv, e->w_qkv[layer]));
        PF_TRY(upload_scaled(e->s_qkv[layer], fs.data(), fs.size(), e->st));
        for (int j = 0; j < 3; j++) pend[key + j].clear(), pend[key + j].shrink_to_fit();
    } else if (m == PF_MAT_O) {
        PF_TRY(pack_host(e, w, rows, cols, e->fmt_o, e->w_o[layer]));
        PF_TRY(upload_scaled(e->s_o[layer], rs, rows, e->st));
    } else if ((m == PF_MAT_GATE || m == PF_MAT_UP) && (held & 0x30u) == 0x30u) {
        // interleave: packed row 2j = gate row j, 2j+1 = up row j (SwiGLU pairs in one thread)
        std::vector<int8_t> fused((size_t)2 * F * d);
        std::vector<float> fs(2 * F);
        for (int j = 0; j < F; j++) {
            std::memcpy(fused.data() + (size_t)(2 * j) * d, pend[key + PF_MAT_GATE].data() + (size_t)j * d, d);
            std::memcpy(fused.data() + (size_t)(2 * j + 1) * d, pend[key + PF_MAT_UP].data() + (size_t)j * d, d);
            fs[2 * j] = pend_s[key + PF_MAT_GATE][j];
            fs[2 * j + 1] = pend_s[key + PF_MAT_UP][j];
        }
        PF_TRY(pack_host(e, fused.data(), 2 * F, d, e->fmt_gu, e->w_gu[layer]));
        PF_TRY(upload_scaled(e->s_gu[layer], fs.data(), fs.size(), e->st));
        pend[key + PF_MAT_GATE].clear();
        pend[key + PF_MAT_UP].clear();
    } else if (m == PF_MAT_DOWN) {
        PF_TRY(pack_host(e, w, rows, cols, e->fmt_down, e->w_down[layer]));
        PF_TRY(upload_scaled(e->s_down[layer], rs, rows, e->st));
    }
    PF_CUDA(cudaStreamSynchronize(e->st));
    e->graph_dirty = true;
    return PF_OK;
}

pf_status pf_engine_set_embedding(pf_engine* e, const int8_t* emb, float gscale) {
    PF_CHECK(e && emb, "pf_engine_set_embedding: null argument");
    PF_CUDA(cudaSetDevice(e->dev));
    PF_CUDA(cudaMemcpy(e->emb_i8, emb, (size_t)e->V * e->d, cudaMemcpyHostToDevice));
    PF_TRY(pack_host(e, emb, e->V, e->d, e->fmt_emb, e->emb_packed));
    e->emb_gscale = gscale;
    e->emb_set = true;
    e->graph_dirty = true;
    return PF_OK;
}

pf_status pf_engine_set_norms(pf_engine* e, const float* a, const float* f, const float* fin) {
    PF_CHECK(e, "pf_engine_set_norms: null engine");
    PF_CUDA(cudaSetDevice(e->dev));
    const size_t n = (size_t)e->L * e->d;
    if (a) PF_CUDA(cudaMemcpy(e->attn_norm, a, n * 4, cudaMemcpyHostToDevice));
    if (f) PF_CUDA(cudaMemcpy(e->ffn_norm, f, n * 4, cudaMemcpyHostToDevice));
    if (fin) PF_CUDA(cudaMemcpy(e->final_norm, fin, (size_t)e->d * 4, cudaMemcpyHostToDevice));
    return PF_OK;
}

pf_status pf_engine_set_mtp_head(pf_engine* e, int32_t h, const uint8_t* gq, const float* gs, const uint8_t* uq,
                                 const float* us, const uint8_t* dq, const float* ds) {
    PF_CHECK(e && gq && gs && uq && us && dq && ds, "pf_engine_set_mtp_head: null argument");
    PF_CHECK(h >= 0 && h < e->K, "pf_engine_set_mtp_head: bad head");
    PF_CUDA(cudaSetDevice(e->dev));
    const int d = e->d;
    // Nibbles as MTPHeads::quantize_q4 packs them (src/mtp.cpp:185-194):
    // byte c/2 of a row holds column c (low) and c+1 (high), value = nibble - 8.
    auto unpack = [&](const uint8_t* q, int8_t* out) {
        for (size_t i = 0; i < (size_t)d * d / 2; i++) {
            out[2 * i] = (int8_t)((int)(q[i] & 0xF) - 8);
            out[2 * i + 1] = (int8_t)((int)(q[i] >> 4) - 8);
        }
    };
    std::vector<int8_t> g((size_t)d * d), u((size_t)d * d), dn((size_t)d * d), gu((size_t)2 * d * d);
    unpack(gq, g.data());
    unpack(uq, u.data());
    unpack(dq, dn.data());
    std::vector<float> gus(2 * d);
    for (int j = 0; j < d; j++) {
        std::memcpy(gu.data() + (size_t)(2 * j) * d, g.data() + (size_t)j * d, d);
        std::memcpy(gu.data() + (size_t)(2 * j + 1) * d, u.data() + (size_t)j * d, d);
        gus[2 * j] = gs[j];
        gus[2 * j + 1] = us[j];
    }
    PF_TRY(pack_host(e, gu.data(), 2 * d, d, WF_Q4, e->mtp_gu[h]));
    PF_TRY(pack_host(e, dn.data(), d, d, WF_Q4, e->mtp_down[h]));
    PF_CUDA(cudaMemcpy(e->mtp_gu_s[h], gus.data(), gus.size() * 4, cudaMemcpyHostToDevice));
    PF_CUDA(cudaMemcpy(e->mtp_down_s[h], ds, (size_t)d * 4, cudaMemcpyHostToDevice));
    e->mtp_set[h] = true;
    e->graph_dirty = true;
    return PF_OK;
}

pf_status pf_engine_set_sampling(pf_engine* e, const pf_sampling_config* c) {
    PF_CHECK(e && c, "pf_engine_set_sampling: null argument");
    e->samp = *c;
    e->graph_dirty = true;
    return PF_OK;
}

pf_status pf_engine_set_skip_threshold(pf_engine* e, float t) {
    PF_CHECK(e, "pf_engine_set_skip_threshold: null engine");
    e->skip_thr = t;
    e->graph_dirty = true;
    return PF_OK;
}

static pf_status check_ready(pf_engine* e) {
    for (int l = 0; l < e->L; l++)
        if (e->loaded[l] != 0x7Fu) {
            set_error("layer %d weights incomplete", l);
            return PF_ERR_STATE;
        }
    if (!e->emb_set) {
        set_error("embedding not set");
        return PF_ERR_STATE;
    }
    for (int h = 0; h < e->K; h++)
        if (!e->mtp_set[h]) {
            set_error("MTP head %d not set", h);
            return PF_ERR_STATE;
        }
    return PF_OK;
}

static pf_status read_error_flag(pf_engine* e) {
    uint32_t flag = 0;
    PF_CUDA(cudaMemcpy(&flag, device_error_flag(), 4, cudaMemcpyDeviceToHost));
    if (flag) {
        cudaMemset(device_error_flag(), 0, 4);
        set_error("device error flag 0x%x (1 bounds, 2 weight range, 4 token, 8 context full)", flag);
        return PF_ERR_DEVICE;
    }
    return PF_OK;
}

pf_status pf_engine_prefill(pf_engine* e, int32_t n, const int32_t* tokens, const int64_t* offsets,
                            const uint32_t* seeds) {
    PF_CHECK(e && tokens && offsets, "pf_engine_prefill: null argument");
    PF_CHECK(n > 0 && n <= e->max_seqs, "pf_engine_prefill: n_seqs %d out of range", n);
    PF_CUDA(cudaSetDevice(e->dev));
    PF_TRY(check_ready(e));
    std::vector<int> len(n);
    int maxlen = 0;
    for (int b = 0; b < n; b++) {
        len[b] = (int)(offsets[b + 1] - offsets[b]);
        PF_CHECK(len[b] >= 1, "prompt %d is empty", b);
        PF_CHECK(len[b] + e->R <= e->max_pos, "prompt %d (%d tokens) leaves no room for a step", b, len[b]);
        for (int i = 0; i < len[b]; i++)
            PF_CHECK(tokens[offsets[b] + i] >= 0 && tokens[offsets[b] + i] < e->V, "token out of range in prompt %d", b);
        maxlen = std::max(maxlen, len[b]);
    }
    e->n_seqs = n;
    e->rngs.assign(n, std::mt19937());
    for (int b = 0; b < n; b++) e->rngs[b].seed(seeds ? seeds[b] : 0u);
    cudaStream_t st = e->st;
    const size_t units = (size_t)e->max_seqs * e->L * e->G;
    PF_CUDA(cudaMemsetAsync(e->kv.acc_k, 0, units * 64 * 8, st));
    PF_CUDA(cudaMemsetAsync(e->kv.acc_v, 0, units * 64 * 8, st));
    if (e->skip_on) PF_CUDA(cudaMemsetAsync(e->skip_cache, 0, (size_t)e->max_seqs * e->L * e->d * 4, st));
    PF_CUDA(cudaMemsetAsync(e->sb.n_logged, 0, e->max_seqs * 4, st));
    PF_CUDA(cudaMemsetAsync(e->ffn_counts, 0, 16, st));
    PF_CUDA(cudaMemsetAsync(e->sb.seq_len, 0, e->max_seqs * 4, st));

    // Chunked prefill: every chunk is a row batch through all layers, committed whole.
    // (at most as many rows per sequence as the tensor-core attention takes)
    int C = std::max(1, std::min(e->kv.Wr, e->Mcap / n));
    while (C > 1 && !attention_decode_supported(e->kv, e->H, C)) C--;
    {
        const int rpc = attention_decode_rows_per_cta(e->kv, e->H);  // whole row groups per chunk
        if (C > rpc) C -= C % rpc;
    }
    std::vector<int> row_tok, row_pos, row0(n), cnt(n), len0(n), last_idx(n, -1);
    std::vector<float> dummy;
    for (int c0 = 0; c0 < maxlen; c0 += C) {
        row_tok.clear();
        row_pos.clear();
        for (int b = 0; b < n; b++) {
            const int k = std::max(0, std::min(C, len[b] - c0));
            row0[b] = (int)row_tok.size();
            cnt[b] = k;
            len0[b] = std::min(c0, len[b]);
            for (int r = 0; r < k; r++) {
                row_tok.push_back(tokens[offsets[b] + c0 + r]);
                row_pos.push_back(c0 + r);
            }
            if (k > 0 && c0 + k == len[b]) last_idx[b] = row0[b] + k - 1;
        }
        const int M = (int)row_tok.size();
        PF_CUDA(cudaMemcpyAsync(e->sb.row_tok, row_tok.data(), M * 4, cudaMemcpyHostToDevice, st));
        PF_CUDA(cudaMemcpyAsync(e->sb.row_pos, row_pos.data(), M * 4, cudaMemcpyHostToDevice, st));
        PF_CUDA(cudaMemcpyAsync(e->sb.bs_row0, row0.data(), n * 4, cudaMemcpyHostToDevice, st));
        PF_CUDA(cudaMemcpyAsync(e->sb.bs_n, cnt.data(), n * 4, cudaMemcpyHostToDevice, st));
        PF_CUDA(cudaMemcpyAsync(e->sb.bs_len0, len0.data(), n * 4, cudaMemcpyHostToDevice, st));
        PF_CUDA(cudaMemcpyAsync(e->sb.n_commit, cnt.data(), n * 4, cudaMemcpyHostToDevice, st));
        PF_TRY(embed(e->emb_i8, e->emb_gscale, e->d, e->V, e->sb.row_tok, M, nullptr, e->x, st));
        RowBatch rb;
        rb.nb = n; rb.M = M; rb.row0 = e->sb.bs_row0; rb.n = e->sb.bs_n; rb.len0 = e->sb.bs_len0;
        rb.row_pos = e->sb.row_pos; rb.max_rows = C;
        PF_TRY(e->layers(rb, M));
        PF_TRY(kv_commit(e->kv, rb, e->sb.n_commit, e->stage, e->Mcap, st));
        if (e->skip_on)
            PF_TRY(skip_commit(n, e->L, e->d, e->Mcap, e->sb.bs_row0, e->sb.n_commit, e->skip_all, e->normed_all,
                               e->skip_cache, e->ffn_counts, st));
        else
            PF_TRY(ffn_count(n, e->L, e->sb.n_commit, e->ffn_counts, st));
        // Keep the hidden of every prompt's last row (MTP input, unembed row).
        std::vector<int> sel, dst;
        for (int b = 0; b < n; b++)
            if (cnt[b] > 0 && c0 + cnt[b] == len[b]) {
                sel.push_back(row0[b] + cnt[b] - 1);
                dst.push_back(b);
            }
        for (size_t i = 0; i < sel.size(); i++)
            PF_CUDA(cudaMemcpyAsync(e->mtp_in + (size_t)dst[i] * e->d, e->x + (size_t)sel[i] * e->d,
                                    (size_t)e->d * 4, cudaMemcpyDeviceToDevice, st));
        PF_CUDA(cudaStreamSynchronize(st));  // host arrays are reused by the next chunk
    }
    PF_CUDA(cudaMemcpyAsync(e->sb.seq_len, len.data(), n * 4, cudaMemcpyHostToDevice, st));
    e->host_len = len;
    // First pending token from the last prompt row, then the first drafts.
    PF_TRY(e->fill_uniforms(1));
    if (!e->greedy()) PF_TRY(e->select_uniforms());
    PF_CUDA(cudaMemcpyAsync(e->mtp_cur, e->mtp_in, (size_t)n * e->d * 4, cudaMemcpyDeviceToDevice, st));
    PF_TRY(e->unembed(e->mtp_in, n, e->logits));
    if (e->greedy()) PF_TRY(argmax_rows(e->logits, e->V, e->V, n, nullptr, e->sb.pending, st));
    else PF_TRY(sample_rows(e->logits, e->V, e->V, e->iota, n, e->samp, e->cur_u, e->R, e->sb.pending, st));
    PF_TRY(e->mtp_chain(n));
    PF_CUDA(cudaStreamSynchronize(st));
    PF_TRY(read_error_flag(e));
    e->prefilled = true;
    if (e->graph_n != n) e->graph_dirty = true;  // the step graph is specialised to n sequences
    return PF_OK;
}

static pf_status run(pf_engine* e, int steps) {
    PF_CHECK(e->prefilled, "step before prefill");
    for (int b = 0; b < e->n_seqs; b++)
        PF_CHECK(e->host_len[b] + (int64_t)steps * e->R <= e->max_pos,
                 "sequence %d would exceed max_positions=%d", b, e->max_pos);
    cudaStream_t st = e->st;
    if (e->graph_dirty) {
        if (e->graph) {
            cudaGraphExecDestroy(e->graph);
            e->graph = nullptr;
        }
        cudaGraph_t g = nullptr;
        PF_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        const pf_status s = e->enqueue_step();
        const cudaError_t ce = cudaStreamEndCapture(st, &g);
        if (s != PF_OK) {
            if (g) cudaGraphDestroy(g);
            return s;
        }
        if (ce != cudaSuccess) {
            set_error("graph capture failed: %s", cudaGetErrorString(ce));
            return PF_ERR_CUDA;
        }
        size_t nn = 0;
        cudaGraphGetNodes(g, nullptr, &nn);
        std::vector<cudaGraphNode_t> nodes(nn);
        cudaGraphGetNodes(g, nodes.data(), &nn);
        e->graph_kernels = 0;
        for (auto nd : nodes) {
            cudaGraphNodeType t;
            if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) e->graph_kernels++;
        }
        const cudaError_t ie = cudaGraphInstantiate(&e->graph, g, 0);
        cudaGraphDestroy(g);
        if (ie != cudaSuccess) {
            set_error("graph instantiate failed: %s", cudaGetErrorString(ie));
            return PF_ERR_CUDA;
        }
        e->graph_dirty = false;
        e->graph_n = e->n_seqs;
    }
    for (int done = 0; done < steps;) {
        const int chunk = std::min(steps - done, kUniformSteps);
        PF_TRY(e->fill_uniforms(chunk));
        if (done == 0) PF_CUDA(cudaEventRecord(e->ev0, st));
        for (int i = 0; i < chunk; i++) PF_CUDA(cudaGraphLaunch(e->graph, st));
        done += chunk;
    }
    PF_CUDA(cudaEventRecord(e->ev1, st));
    for (int b = 0; b < e->n_seqs; b++) e->host_len[b] += steps * e->R;  // upper bound
    return PF_OK;
}

// After a step graph: the step's packed results from pinned memory (the
// lengths tighten the host's bound; a latched device error is reported once).
static pf_status read_pack(pf_engine* e, int32_t* n_emitted, int32_t* emitted) {
    const int n = e->n_seqs, R = e->R;
    const int* h = e->hpin;
    if (n_emitted) std::memcpy(n_emitted, h, (size_t)n * 4);
    if (emitted) std::memcpy(emitted, h + n, (size_t)n * R * 4);
    e->host_len.assign(h + n * (R + 1), h + n * (R + 2));
    const uint32_t flag = (uint32_t)h[n * (R + 2)];
    if (flag) {
        cudaMemset(device_error_flag(), 0, 4);
        set_error("device error flag 0x%x (1 bounds, 2 weight range, 4 token, 8 context full)", flag);
        return PF_ERR_DEVICE;
    }
    return PF_OK;
}

pf_status pf_engine_step(pf_engine* e, int32_t* n_emitted, int32_t* emitted) {
    PF_CHECK(e, "pf_engine_step: null engine");
    PF_CUDA(cudaSetDevice(e->dev));
    PF_TRY(run(e, 1));
    PF_CUDA(cudaStreamSynchronize(e->st));
    PF_CUDA(cudaEventElapsedTime(&e->last_ms, e->ev0, e->ev1));
    return read_pack(e, n_emitted, emitted);
}

pf_status pf_engine_set_drafts(pf_engine* e, const int32_t* drafts) {
    PF_CHECK(e && drafts, "pf_engine_set_drafts: null argument");
    PF_CHECK(e->prefilled, "pf_engine_set_drafts before prefill");
    PF_CUDA(cudaSetDevice(e->dev));
    for (int i = 0; i < e->n_seqs * e->K; i++)
        PF_CHECK(drafts[i] >= 0 && drafts[i] < e->V, "draft token out of range");
    PF_CUDA(cudaMemcpyAsync(e->sb.drafts, drafts, (size_t)e->n_seqs * e->K * 4, cudaMemcpyHostToDevice, e->st));
    PF_CUDA(cudaStreamSynchronize(e->st));
    return PF_OK;
}

pf_status pf_engine_run_steps(pf_engine* e, int32_t steps) {
    PF_CHECK(e && steps >= 0, "pf_engine_run_steps: bad arguments");
    if (steps == 0) return PF_OK;
    PF_CUDA(cudaSetDevice(e->dev));
    PF_TRY(run(e, steps));
    PF_CUDA(cudaStreamSynchronize(e->st));
    PF_CUDA(cudaEventElapsedTime(&e->last_ms, e->ev0, e->ev1));
    return read_pack(e, nullptr, nullptr);
}

static pf_status d2h(pf_engine* e, void* dst, const void* src, size_t bytes) {
    PF_CHECK(e && dst, "read: null argument");
    PF_CUDA(cudaSetDevice(e->dev));
    PF_CUDA(cudaStreamSynchronize(e->st));
    PF_CUDA(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost));
    return PF_OK;
}

pf_status pf_engine_read_logits(pf_engine* e, float* out) {
    return d2h(e, out, e->logits, (size_t)e->n_seqs * e->R * e->V * 4);
}
pf_status pf_engine_read_drafts(pf_engine* e, int32_t* out) {
    return d2h(e, out, e->sb.drafts, (size_t)e->n_seqs * e->K * 4);
}
pf_status pf_engine_read_pending(pf_engine* e, int32_t* out) { return d2h(e, out, e->sb.pending, e->n_seqs * 4); }
pf_status pf_engine_read_positions(pf_engine* e, int32_t* out) { return d2h(e, out, e->sb.seq_len, e->n_seqs * 4); }
pf_status pf_engine_read_hidden(pf_engine* e, float* out) {
    return d2h(e, out, e->mtp_in, (size_t)e->n_seqs * e->d * 4);
}
pf_status pf_engine_read_mtp_logits(pf_engine* e, float* out) {
    PF_CHECK(e && out, "read: null argument");
    PF_CUDA(cudaSetDevice(e->dev));
    PF_CUDA(cudaStreamSynchronize(e->st));
    const size_t row = (size_t)e->V;
    for (int b = 0; b < e->n_seqs; b++)
        for (int h = 0; h < e->K; h++)
            PF_CUDA(cudaMemcpy(out + ((size_t)b * e->K + h) * row, e->mtp_logits + ((size_t)h * e->max_seqs + b) * row,
                               row * 4, cudaMemcpyDeviceToHost));
    return PF_OK;
}
pf_status pf_engine_read_skip_counts(pf_engine* e, int64_t* computed, int64_t* skipped) {
    long long c[2];
    PF_TRY(d2h(e, c, e->ffn_counts, 16));
    if (computed) *computed = c[0];
    if (skipped) *skipped = c[1];
    return PF_OK;
}
pf_status pf_engine_read_log(pf_engine* e, int32_t* counts, int32_t* tokens, int32_t cap) {
    PF_CHECK(e && counts, "read: null argument");
    PF_TRY(d2h(e, counts, e->sb.n_logged, e->n_seqs * 4));
    if (tokens)
        for (int b = 0; b < e->n_seqs; b++)
            PF_CUDA(cudaMemcpy(tokens + (size_t)b * cap, e->sb.log + (size_t)b * e->sb.log_cap,
                               (size_t)std::min(cap, counts[b]) * 4, cudaMemcpyDeviceToHost));
    return PF_OK;
}

pf_status pf_engine_read_kv(pf_engine* e, int32_t b, int32_t l, int32_t g, int8_t* k, float* ks, int8_t* v, float* vs,
                            int32_t max_entries, int32_t* count) {
    PF_CHECK(e && k && ks && v && vs && count, "pf_engine_read_kv: null argument");
    PF_CHECK(b >= 0 && b < e->n_seqs && l >= 0 && l < e->L && g >= 0 && g < e->G, "pf_engine_read_kv: bad index");
    PF_CUDA(cudaSetDevice(e->dev));
    PF_CUDA(cudaStreamSynchronize(e->st));
    int len = 0;
    PF_CUDA(cudaMemcpy(&len, e->sb.seq_len + b, 4, cudaMemcpyDeviceToHost));
    const KvCache& kv = e->kv;
    const size_t u = kv.unit(b, l, g);
    const int cs = std::min(len, kv.S), np = kv_pool_count(len, kv.S, kv.Wr, kv.pb);
    const int qlo = std::max(kv.S, len - kv.Wr), nw = std::max(0, len - qlo);
    int n = 0;
    auto put = [&](const int8_t* kp, const float* ksp, const int8_t* vp, const float* vsp) -> pf_status {
        if (n >= max_entries) return PF_OK;
        PF_CUDA(cudaMemcpy(k + (size_t)n * 64, kp, 64, cudaMemcpyDeviceToHost));
        PF_CUDA(cudaMemcpy(v + (size_t)n * 64, vp, 64, cudaMemcpyDeviceToHost));
        PF_CUDA(cudaMemcpy(ks + n, ksp, 4, cudaMemcpyDeviceToHost));
        PF_CUDA(cudaMemcpy(vs + n, vsp, 4, cudaMemcpyDeviceToHost));
        n++;
        return PF_OK;
    };
    for (int p = 0; p < cs; p++)
        PF_TRY(put(kv.sink_k + (u * kv.S + p) * 64, kv.sink_ks + u * kv.S + p, kv.sink_v + (u * kv.S + p) * 64,
                   kv.sink_vs + u * kv.S + p));
    std::vector<int8_t> vblk(64 * 32);
    auto put_blocked = [&](const int8_t* kp, const float* ksp, const int8_t* vbase, size_t e, const float* vsp)
        -> pf_status {
        if (n >= max_entries) return PF_OK;
        PF_CUDA(cudaMemcpy(k + (size_t)n * 64, kp, 64, cudaMemcpyDeviceToHost));
        PF_CUDA(cudaMemcpy(vblk.data(), vbase + (e >> 5) * 2048, 2048, cudaMemcpyDeviceToHost));
        for (int d = 0; d < 64; d++) v[(size_t)n * 64 + d] = vblk[(size_t)d * 32 + kv_vpos((int)(e & 31))];
        PF_CUDA(cudaMemcpy(ks + n, ksp, 4, cudaMemcpyDeviceToHost));
        PF_CUDA(cudaMemcpy(vs + n, vsp, 4, cudaMemcpyDeviceToHost));
        n++;
        return PF_OK;
    };
    for (int j = 0; j < np; j++)
        PF_TRY(put_blocked(kv.pool_k + (u * kv.P_pad + j) * 64, kv.pool_ks + u * kv.P_pad + j,
                           kv.pool_v + u * kv.P_pad * 64, (size_t)j, kv.pool_vs + u * kv.P_pad + j));
    for (int i = 0; i < nw; i++) {
        const int slot = (qlo + i - kv.S) % kv.Wr;
        const size_t o = u * kv.W_pad + slot;
        PF_TRY(put_blocked(kv.ring_k + o * 64, kv.ring_ks + o, kv.ring_v + u * kv.W_pad * 64, (size_t)slot,
                           kv.ring_vs + o));
    }
    *count = n;
    return PF_OK;
}

pf_status pf_engine_launches_per_step(pf_engine* e, int32_t* kernels) {
    PF_CHECK(e && kernels, "pf_engine_launches_per_step: null argument");
    *kernels = e->graph_kernels;
    return PF_OK;
}

pf_status pf_engine_last_ms(pf_engine* e, float* ms) {
    PF_CHECK(e && ms, "pf_engine_last_ms: null argument");
    *ms = e->last_ms;
    return PF_OK;
}

pf_status pf_engine_set_attention_splits(pf_engine* e, int32_t n) {
    PF_CHECK(e, "pf_engine_set_attention_splits: null engine");
    PF_CHECK(n >= 0 && n <= pf_engine::kMaxAttnSplits, "attention splits must be 0..%d", pf_engine::kMaxAttnSplits);
    if (n != e->attn_splits) e->graph_dirty = true;
    e->attn_splits = n;
    return PF_OK;
}

pf_status pf_engine_set_kernel_timing(pf_engine* e, int32_t on) {
    PF_CHECK(e, "pf_engine_set_kernel_timing: null engine");
    PF_CUDA(cudaSetDevice(e->dev));
    if (on && e->kev.empty()) {
        e->kev.resize(2 * pf_engine::kTimedLaunches);
        e->kev_cat.resize(pf_engine::kTimedLaunches);
        for (cudaEvent_t& v : e->kev) PF_CUDA(cudaEventCreate(&v));
    }
    if ((on != 0) != e->ktiming) e->graph_dirty = true;
    e->ktiming = on != 0;
    return PF_OK;
}

pf_status pf_engine_kernel_times(pf_engine* e, float* ms, int32_t* launches) {
    PF_CHECK(e && ms && launches, "pf_engine_kernel_times: null argument");
    PF_CHECK(e->ktiming && !e->graph_dirty, "pf_engine_kernel_times: no step ran with kernel timing on");
    PF_CHECK(!e->kev_over, "pf_engine_kernel_times: more than %d timed launches in a step", pf_engine::kTimedLaunches);
    PF_CUDA(cudaSetDevice(e->dev));
    PF_CUDA(cudaStreamSynchronize(e->st));
    ms[0] = ms[1] = 0.0f;
    launches[0] = launches[1] = 0;
    for (int i = 0; i < e->kev_used; i++) {
        float t = 0.0f;
        PF_CUDA(cudaEventElapsedTime(&t, e->kev[2 * i], e->kev[2 * i + 1]));
        ms[e->kev_cat[i]] += t;
        launches[e->kev_cat[i]]++;
    }
    return PF_OK;
}

}  // extern "C"

// attention.cu — attention over the 3-tier int8 KV cache for a batch of rows,
// the staging of new K/V, speculative pool entries, and the commit.
//
// Semantics (KVCache::attention_scores / attention_weighted_sum and
// Engine::compute_attention, src/kv_cache.cpp:129-198, src/engine.cpp:753-779):
// row r of a sequence, at position p = len0 + r, attends to the cache as it
// would be after positions [0, p) were stored one by one:
//   sink positions [0, min(p, S)),
//   pool entries [0, floor(max(0, p - S - Wr) / pb)),
//   window positions [max(S, p - Wr), p),
// all as int8 rows times their scale, plus itself in float (the self term),
// with scores scaled by 1/sqrt(head_dim) and one softmax over all of them.
// Positions >= len0 are this batch's own earlier rows (staged, already
// quantized exactly as KVCache::store would), so a K+1-row verification
// sees what K+1 sequential forwards would see.
#include <cfloat>

#include "kv.cuh"

namespace pf {

namespace {

__device__ __forceinline__ float wmax(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float wsum(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// KVCache::quantize_row (src/kv_cache.cpp:19-28) for 64 values held two per lane.
__device__ __forceinline__ void quant64_warp(float a, float b, int8_t& qa, int8_t& qb, float& scale) {
    const float amax = wmax(fmaxf(fabsf(a), fabsf(b)));
    scale = (amax == 0.0f) ? 1.0f : __fdiv_rn(amax, 127.0f);
    const float mul = (amax == 0.0f) ? 1.0f : __fdiv_rn(127.0f, amax);
    qa = (int8_t)(int)roundf(__fmul_rn(a, mul));
    qb = (int8_t)(int)roundf(__fmul_rn(b, mul));
}

}  // namespace

// ---------------------------------------------------------------------------
// Staging: quantize each row's K and V per kv head.
// ---------------------------------------------------------------------------
__global__ void kv_quant_kernel(const float* __restrict__ qkv, int ld, int k_col, int v_col, int M,
                                const int* m_dev, int G, Staged st) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the attention may start streaming the cache
    const int wid = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int m_act = m_dev ? min(M, *m_dev) : M;
    if (wid >= m_act * G) return;
    const int m = wid / G, g = wid % G;
    const float* kr = qkv + (size_t)m * ld + k_col + g * 64;
    const float* vr = qkv + (size_t)m * ld + v_col + g * 64;
    int8_t a, b;
    float s;
    quant64_warp(kr[lane], kr[lane + 32], a, b, s);
    st.k[(size_t)wid * 64 + lane] = a;
    st.k[(size_t)wid * 64 + lane + 32] = b;
    if (lane == 0) st.ks[wid] = s;
    quant64_warp(vr[lane], vr[lane + 32], a, b, s);
    st.v[(size_t)wid * 64 + lane] = a;
    st.v[(size_t)wid * 64 + lane + 32] = b;
    if (lane == 0) st.vs[wid] = s;
}

pf_status kv_quant_rows(const float* qkv, int ldqkv, int k_col, int v_col, int M, const int* m_dev, int G, int hd,
                        Staged st, cudaStream_t stream) {
    PF_CHECK(hd == 64, "kv_quant_rows: head_dim must be 64");
    kv_quant_kernel<<<ceil_div(M * G, 4), 128, 0, stream>>>(qkv, ldqkv, k_col, v_col, M, m_dev, G, st);
    return launch_check("kv_quant");
}

// ---------------------------------------------------------------------------
// The QKV projection's epilogue for a K-split launch, fused with the staging:
// per row, sum the int32 slices exactly, v = ((float)acc * a_s[m]) * w_s[n]
// (matmul_quantized's roundings, src/matmul_neon.cpp:176-180), rotate the q
// and k columns by adjacent pairs at the row's position (src/engine.cpp:737-748,
// the same arithmetic as the GEMM's EPI_QKV), write the fp32 row, and quantize
// each kv head's K and V as kv_quant_kernel does.  One CTA of 8 warps per row;
// warp w takes the 64-column groups w, w + 8, ..., lane l columns 2l, 2l + 1.
// ---------------------------------------------------------------------------
constexpr int kQkvMaxParts = 4;
constexpr int kQkvGroups = 8;  // 64-column groups per warp (n <= 4096)

__global__ void __launch_bounds__(256) qkv_finish_kernel(const int32_t* __restrict__ parts, int n_parts,
                                                         int64_t part_stride, const float* __restrict__ a_s,
                                                         const float* __restrict__ w_s, int N, int M,
                                                         const float* __restrict__ rope_cos,
                                                         const float* __restrict__ rope_sin,
                                                         const int* __restrict__ row_pos, int rope_cols, int hd,
                                                         float* __restrict__ qkv, int k_col, int v_col, int G,
                                                         Staged st) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the attention may start streaming the cache
    const int m = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (m >= M) return;
    const float as = a_s[m];
    const int pos = row_pos[m];
    const int ngroups = N / 64;
    // every load of the row first
    int2 acc[kQkvGroups];
    float2 ws[kQkvGroups], cs[kQkvGroups];
#pragma unroll
    for (int k = 0; k < kQkvGroups; k++) {
        const int grp = warp + 8 * k;
        const bool in = grp < ngroups;
        const int c0 = grp * 64 + 2 * lane;
        acc[k] = make_int2(0, 0);
#pragma unroll
        for (int s2 = 0; s2 < kQkvMaxParts; s2++) {
            const int2 v = (in && s2 < n_parts)
                               ? __ldcg(reinterpret_cast<const int2*>(parts + s2 * part_stride + (size_t)m * N + c0))
                               : make_int2(0, 0);
            acc[k].x += v.x;
            acc[k].y += v.y;
        }
        ws[k] = in ? *reinterpret_cast<const float2*>(w_s + c0) : make_float2(0.f, 0.f);
        const bool rot = in && c0 < rope_cols;
        const size_t o = (size_t)pos * (hd >> 1) + ((c0 % hd) >> 1);
        cs[k] = rot ? make_float2(rope_cos[o], rope_sin[o]) : make_float2(1.f, 0.f);
    }
#pragma unroll
    for (int k = 0; k < kQkvGroups; k++) {
        const int grp = warp + 8 * k;
        if (grp >= ngroups) break;  // uniform over the warp
        const int c0 = grp * 64 + 2 * lane;
        float v0 = __fmul_rn(__fmul_rn(__int2float_rn(acc[k].x), as), ws[k].x);
        float v1 = __fmul_rn(__fmul_rn(__int2float_rn(acc[k].y), as), ws[k].y);
        if (c0 < rope_cols) {
            const float r0 = __fsub_rn(__fmul_rn(v0, cs[k].x), __fmul_rn(v1, cs[k].y));
            const float r1 = __fadd_rn(__fmul_rn(v0, cs[k].y), __fmul_rn(v1, cs[k].x));
            v0 = r0;
            v1 = r1;
        }
        *reinterpret_cast<float2*>(qkv + (size_t)m * N + c0) = make_float2(v0, v1);
        if (grp * 64 >= k_col) {  // a K or V head: stage it (the group is one head)
            const bool is_k = grp * 64 < v_col;
            const int g = (grp * 64 - (is_k ? k_col : v_col)) / 64;
            int8_t a, b;
            float sc;
            quant64_warp(v0, v1, a, b, sc);
            const size_t wid = (size_t)m * G + g;
            int8_t* dst = (is_k ? st.k : st.v) + wid * 64 + 2 * lane;
            dst[0] = a;
            dst[1] = b;
            if (lane == 0) (is_k ? st.ks : st.vs)[wid] = sc;
        }
    }
}

pf_status qkv_finish(const int32_t* parts, int n_parts, int64_t part_stride, const float* a_s, const float* w_s,
                     int N, int M, const float* rope_cos, const float* rope_sin, const int* row_pos, int rope_cols,
                     int hd, float* qkv, int k_col, int v_col, int G, Staged st, cudaStream_t stream) {
    PF_CHECK(hd == 64, "qkv_finish: head_dim must be 64");
    PF_CHECK(n_parts >= 1 && n_parts <= kQkvMaxParts && part_stride >= (int64_t)M * N, "qkv_finish: bad slices");
    PF_CHECK(N % 64 == 0 && N / 64 <= 8 * kQkvGroups, "qkv_finish: N=%d must be a multiple of 64, at most %d", N,
             512 * kQkvGroups);
    PF_CHECK(k_col % 64 == 0 && v_col % 64 == 0 && k_col <= v_col && v_col + G * 64 <= N && rope_cols <= v_col,
             "qkv_finish: bad column layout");
    qkv_finish_kernel<<<M, 256, 0, stream>>>(parts, n_parts, part_stride, a_s, w_s, N, M, rope_cos, rope_sin,
                                             row_pos, rope_cols, hd, qkv, k_col, v_col, G, st);
    return launch_check("qkv_finish");
}

// ---------------------------------------------------------------------------
// Pool entries a batch finalizes between its first and last row
// (src/kv_cache.cpp:77-109): the committed fp64 accumulator plus the evicted
// ring entries, added in eviction order, mean = (float)(acc * (1.0f/pb)),
// requantized.  All evicted entries involved are committed ring entries.
// ---------------------------------------------------------------------------
__global__ void kv_pool_spec_kernel(KvCache kv, int layer, RowBatch rb, SpecPool sp) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the attention may start streaming the cache
    const int b = blockIdx.x, g = blockIdx.y, d = threadIdx.x;  // 64 threads
    const int n = rb.n[b];
    if (n == 0) return;
    const int L0 = rb.len0[b], plast = L0 + n - 1;
    const int nb0 = kv_pool_count(L0, kv.S, kv.Wr, kv.pb), nb1 = kv_pool_count(plast, kv.S, kv.Wr, kv.pb);
    if (nb1 <= nb0) return;
    const size_t u = kv.unit(b, layer, g);
    const int E0 = max(0, L0 - kv.S - kv.Wr);
    __shared__ float red[2][64];
    for (int j = nb0; j < nb1 && j - nb0 < sp.per; j++) {
        double sk = (j == nb0) ? kv.acc_k[u * 64 + d] : 0.0;
        double sv = (j == nb0) ? kv.acc_v[u * 64 + d] : 0.0;
        const int q0 = kv.S + max(j * kv.pb, E0), q1 = kv.S + (j + 1) * kv.pb;
        for (int q = q0; q < q1; q++) {
            const int slot = (q - kv.S) % kv.Wr;
            const size_t e = u * kv.W_pad + slot;
            sk += (double)kv.ring_k[e * 64 + d] * (double)kv.ring_ks[e];
            sv += (double)kv.ring_v[u * kv.W_pad * 64 + kv_voff(slot, d)] * (double)kv.ring_vs[e];
        }
        const float inv = 1.0f / (float)kv.pb;
        const float mk = (float)(sk * (double)inv), mv = (float)(sv * (double)inv);
        red[0][d] = fabsf(mk);
        red[1][d] = fabsf(mv);
        __syncthreads();
        for (int s = 32; s >= 1; s >>= 1) {
            if (d < s) {
                red[0][d] = fmaxf(red[0][d], red[0][d + s]);
                red[1][d] = fmaxf(red[1][d], red[1][d + s]);
            }
            __syncthreads();
        }
        const float ak = red[0][0], av = red[1][0];
        __syncthreads();
        const size_t o = (((size_t)b * kv.G + g) * sp.per + (j - nb0));
        const float mulk = ak == 0.0f ? 1.0f : __fdiv_rn(127.0f, ak), mulv = av == 0.0f ? 1.0f : __fdiv_rn(127.0f, av);
        sp.k[o * 64 + d] = (int8_t)(int)roundf(__fmul_rn(mk, mulk));
        sp.v[o * 64 + d] = (int8_t)(int)roundf(__fmul_rn(mv, mulv));
        if (d == 0) {
            sp.ks[o] = ak == 0.0f ? 1.0f : __fdiv_rn(ak, 127.0f);
            sp.vs[o] = av == 0.0f ? 1.0f : __fdiv_rn(av, 127.0f);
        }
    }
}

pf_status kv_pool_spec(const KvCache& kv, int layer, const RowBatch& rb, SpecPool sp, cudaStream_t stream) {
    PF_CHECK(kv.hd == 64, "kv_pool_spec: head_dim must be 64");
    dim3 grid(rb.nb, kv.G);
    kv_pool_spec_kernel<<<grid, 64, 0, stream>>>(kv, layer, rb, sp);
    return launch_check("kv_pool_spec");
}

// ---------------------------------------------------------------------------
// Attention.  One CTA per (sequence, kv head); warp w serves q head
// g + w*G (the reference's GQA map kv = h % n_kv_heads).  Entries stream
// through shared memory 32 at a time; each lane scores one entry against up
// to RG query rows, then an online softmax (running max / sum, rescaled)
// accumulates p * v.  The self term and the 1e-10 of softmax
// (src/matmul_neon.cpp:222) are applied at the end.
// ---------------------------------------------------------------------------
namespace {
constexpr int RG = 8;        // query rows per pass
constexpr int KROW = 80;     // smem bytes per K row (conflict-free 16 B reads)

struct EntryDesc {
    const int8_t* k;
    const int8_t* v;       // entry-major row, or the unit's blocked V array
    int vblock;            // >= 0: entry index inside the blocked V array
    float ks, vs;
    int rlo, rhi;  // visible to rows rlo..rhi
};

__device__ EntryDesc entry_at(const KvCache& kv, int layer, int b, int g, int L0, int n, int row0, int e,
                              int cs, int npool, int nb0, int qlo, int nwin, const Staged& st, const SpecPool& sp) {
    EntryDesc d;
    d.vblock = -1;
    const size_t u = kv.unit(b, layer, g);
    if (e < cs) {  // committed sink position e
        d.k = kv.sink_k + (u * kv.S + e) * 64;
        d.v = kv.sink_v + (u * kv.S + e) * 64;
        d.ks = kv.sink_ks[u * kv.S + e];
        d.vs = kv.sink_vs[u * kv.S + e];
        d.rlo = 0;
        d.rhi = 1 << 30;
        return d;
    }
    e -= cs;
    if (e < npool) {  // pool entry e
        if (e < nb0) {
            d.k = kv.pool_k + (u * kv.P_pad + e) * 64;
            d.v = kv.pool_v + u * kv.P_pad * 64;
            d.vblock = e;
            d.ks = kv.pool_ks[u * kv.P_pad + e];
            d.vs = kv.pool_vs[u * kv.P_pad + e];
        } else {
            const size_t o = ((size_t)b * kv.G + g) * sp.per + (e - nb0);
            d.k = sp.k + o * 64;
            d.v = sp.v + o * 64;
            d.ks = sp.ks[o];
            d.vs = sp.vs[o];
        }
        d.rlo = max(0, kv.S + kv.Wr + (e + 1) * kv.pb - L0);
        d.rhi = 1 << 30;
        return d;
    }
    e -= npool;
    if (e < nwin) {  // committed window position q
        const int q = qlo + e;
        const int slot = (q - kv.S) % kv.Wr;
        const size_t o = u * kv.W_pad + slot;
        d.k = kv.ring_k + o * 64;
        d.v = kv.ring_v + u * kv.W_pad * 64;
        d.vblock = slot;
        d.ks = kv.ring_ks[o];
        d.vs = kv.ring_vs[o];
        d.rlo = 0;
        d.rhi = q + kv.Wr - L0;
        return d;
    }
    e -= nwin;  // staged row e of this batch
    const size_t o = (size_t)(row0 + e) * kv.G + g;
    d.k = st.k + o * 64;
    d.v = st.v + o * 64;
    d.ks = st.ks[o];
    d.vs = st.vs[o];
    d.rlo = e + 1;
    d.rhi = 1 << 30;
    return d;
}
}  // namespace

__global__ void __launch_bounds__(256) attention_kernel(KvCache kv, int layer, RowBatch rb, const float* __restrict__ qkv,
                                                        int ld, int k_col, int v_col, int H, Staged st, SpecPool sp,
                                                        float* __restrict__ out, int ldo) {
    const int b = blockIdx.x, g = blockIdx.y;
    const int n = rb.n[b];
    if (n == 0) return;
    const int nwarps = blockDim.x >> 5;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = g + warp * kv.G;
    const int L0 = rb.len0[b], row0 = rb.row0[b];
    const int plast = L0 + n - 1;
    const int cs = min(L0, kv.S);
    const int nb0 = kv_pool_count(L0, kv.S, kv.Wr, kv.pb);
    const int npool = kv_pool_count(plast, kv.S, kv.Wr, kv.pb);
    const int qlo = max(kv.S, L0 - kv.Wr);
    const int nwin = max(0, L0 - qlo);
    const int T = cs + npool + nwin + (n - 1);
    const float scale = 1.0f / sqrtf(64.0f);

    __shared__ __align__(16) int8_t Kt[32 * KROW];
    __shared__ __align__(16) int8_t Vt[32 * 64];
    __shared__ float kst[32], vst[32];
    __shared__ int rlo_s[32], rhi_s[32];
    __shared__ float qsh[8][RG][64];
    __shared__ float psh[8][RG][32];

    for (int rg0 = 0; rg0 < n; rg0 += RG) {
        const int nr = min(RG, n - rg0);
        // Queries of this pass.
        for (int r = 0; r < nr; r++) {
            const float* qr = qkv + (size_t)(row0 + rg0 + r) * ld + h * 64;
            qsh[warp][r][lane] = qr[lane];
            qsh[warp][r][lane + 32] = qr[lane + 32];
        }
        float m_run[RG], l_run[RG], acc0[RG], acc1[RG];
#pragma unroll
        for (int r = 0; r < RG; r++) {
            m_run[r] = -INFINITY;
            l_run[r] = 0.0f;
            acc0[r] = 0.0f;
            acc1[r] = 0.0f;
        }
        for (int t0 = 0; t0 < T; t0 += 32) {
            __syncthreads();  // previous tile fully consumed
            for (int task = threadIdx.x; task < 32 * 4; task += blockDim.x) {
                const int i = task & 31, c = task >> 5;
                const int e = t0 + i;
                if (e < T) {
                    const EntryDesc d = entry_at(kv, layer, b, g, L0, n, row0, e, cs, npool, nb0, qlo, nwin, st, sp);
                    *reinterpret_cast<uint4*>(Kt + i * KROW + c * 16) = *reinterpret_cast<const uint4*>(d.k + c * 16);
                    if (d.vblock < 0) {
                        *reinterpret_cast<uint4*>(Vt + i * 64 + c * 16) = *reinterpret_cast<const uint4*>(d.v + c * 16);
                    } else {
                        for (int dd = c * 16; dd < c * 16 + 16; dd++) Vt[i * 64 + dd] = d.v[kv_voff(d.vblock, dd)];
                    }
                    if (c == 0) {
                        kst[i] = d.ks;
                        vst[i] = d.vs;
                        rlo_s[i] = d.rlo;
                        rhi_s[i] = d.rhi;
                    }
                } else if (c == 0) {
                    kst[i] = 0.0f;
                    vst[i] = 0.0f;
                    rlo_s[i] = 1 << 30;
                    rhi_s[i] = -1;
                }
            }
            __syncthreads();
            if (warp >= H / kv.G) continue;
            // Scores: lane = entry.
            float kf[64];
            {
                const int8_t* kr = Kt + lane * KROW;
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const uint4 w4 = *reinterpret_cast<const uint4*>(kr + c * 16);
                    const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                    for (int q = 0; q < 4; q++)
#pragma unroll
                        for (int j = 0; j < 4; j++) kf[c * 16 + q * 4 + j] = (float)(int8_t)(ws[q] >> (8 * j));
                }
            }
            const float ksl = kst[lane];
            const int lo = rlo_s[lane], hi = rhi_s[lane];
#pragma unroll
            for (int r = 0; r < RG; r++) {
                if (r >= nr) break;
                const int rr = rg0 + r;
                float s = 0.0f;
#pragma unroll
                for (int dd = 0; dd < 64; dd++) s = fmaf(qsh[warp][r][dd], kf[dd], s);
                s = (rr >= lo && rr <= hi) ? s * ksl * scale : -INFINITY;
                const float tmax = wmax(s);
                const float m_new = fmaxf(m_run[r], tmax);
                float p = 0.0f, corr = 1.0f;
                if (m_new != -INFINITY) {
                    corr = (m_run[r] == -INFINITY) ? 0.0f : expf(m_run[r] - m_new);
                    p = (s == -INFINITY) ? 0.0f : expf(s - m_new);
                }
                l_run[r] = l_run[r] * corr + wsum(p);
                acc0[r] *= corr;
                acc1[r] *= corr;
                m_run[r] = m_new;
                psh[warp][r][lane] = p * vst[lane];
            }
            __syncwarp();
            for (int i = 0; i < 32; i++) {
                const float va = (float)Vt[i * 64 + lane], vb = (float)Vt[i * 64 + lane + 32];
#pragma unroll
                for (int r = 0; r < RG; r++) {
                    if (r >= nr) break;
                    const float pv = psh[warp][r][i];
                    acc0[r] = fmaf(pv, va, acc0[r]);
                    acc1[r] = fmaf(pv, vb, acc1[r]);
                }
            }
            __syncwarp();
        }
        // Self term and output.
        if (warp < H / kv.G) {
            for (int r = 0; r < nr; r++) {
                const int row = row0 + rg0 + r;
                const float* kself = qkv + (size_t)row * ld + k_col + g * 64;
                const float* vself = qkv + (size_t)row * ld + v_col + g * 64;
                const float s =
                    wsum(qsh[warp][r][lane] * kself[lane] + qsh[warp][r][lane + 32] * kself[lane + 32]) * scale;
                const float m_new = fmaxf(m_run[r], s);
                const float corr = (m_run[r] == -INFINITY) ? 0.0f : expf(m_run[r] - m_new);
                const float p = expf(s - m_new);
                const float l = l_run[r] * corr + p;
                const float inv = 1.0f / (l + 1e-10f);
                float* o = out + (size_t)row * ldo + h * 64;
                o[lane] = (acc0[r] * corr + p * vself[lane]) * inv;
                o[lane + 32] = (acc1[r] * corr + p * vself[lane + 32]) * inv;
            }
        }
    }
}

pf_status attention(const KvCache& kv, int layer, const RowBatch& rb, const float* qkv, int ldqkv, int k_col,
                    int v_col, int H, Staged st, SpecPool sp, float* out, int ldo, cudaStream_t stream) {
    PF_CHECK(kv.hd == 64, "attention: head_dim must be 64");
    PF_CHECK(H % kv.G == 0 && H / kv.G <= 8, "attention: n_heads/n_kv_heads must be 1..8");
    dim3 grid(rb.nb, kv.G);
    const int warps = H / kv.G;
    attention_kernel<<<grid, 32 * warps, 0, stream>>>(kv, layer, rb, qkv, ldqkv, k_col, v_col, H, st, sp, out, ldo);
    return launch_check("attention");
}

// ---------------------------------------------------------------------------
// Commit (KVCache::store, src/kv_cache.cpp:59-127) of the accepted rows of
// every sequence, every layer and kv head: sink or ring slot, eviction of
// the slot's old entry into the fp64 accumulator in position order, pool
// finalization every pb evictions.  One CTA of 64 threads (one per dim)
// per (sequence, layer, kv head).
// ---------------------------------------------------------------------------
__global__ void kv_commit_kernel(KvCache kv, RowBatch rb, const int* __restrict__ n_commit, Staged st, int Mst) {
    const int b = blockIdx.x, l = blockIdx.y, g = blockIdx.z, d = threadIdx.x;
    const int nc = n_commit[b];
    if (nc <= 0) return;
    const int L0 = rb.len0[b], row0 = rb.row0[b];
    const size_t u = kv.unit(b, l, g);
    double ak = kv.acc_k[u * 64 + d], av = kv.acc_v[u * 64 + d];
    __shared__ float red[2][64];
    const size_t lbase = (size_t)l * Mst * kv.G;
    for (int r = 0; r < nc; r++) {
        const int p = L0 + r;
        if (p >= kv.max_pos) break;
        const size_t src = lbase + (size_t)(row0 + r) * kv.G + g;
        const int8_t nk = st.k[src * 64 + d], nv = st.v[src * 64 + d];
        const float nks = st.ks[src], nvs = st.vs[src];
        if (p < kv.S) {
            kv.sink_k[(u * kv.S + p) * 64 + d] = nk;
            kv.sink_v[(u * kv.S + p) * 64 + d] = nv;
            if (d == 0) {
                kv.sink_ks[u * kv.S + p] = nks;
                kv.sink_vs[u * kv.S + p] = nvs;
            }
            continue;
        }
        const int slot = (p - kv.S) % kv.Wr;
        const size_t e = u * kv.W_pad + slot;
        const size_t ve = u * kv.W_pad * 64 + kv_voff(slot, d);
        if (p - kv.S >= kv.Wr) {  // window full: evict position p - Wr from this slot
            ak += (double)kv.ring_k[e * 64 + d] * (double)kv.ring_ks[e];
            av += (double)kv.ring_v[ve] * (double)kv.ring_vs[e];
            const int E = p - kv.S - kv.Wr + 1;  // evictions so far
            if (E % kv.pb == 0) {
                const int blk = E / kv.pb - 1;
                const float inv = 1.0f / (float)kv.pb;
                const float mk = (float)(ak * (double)inv), mv = (float)(av * (double)inv);
                red[0][d] = fabsf(mk);
                red[1][d] = fabsf(mv);
                __syncthreads();
                for (int s = 32; s >= 1; s >>= 1) {
                    if (d < s) {
                        red[0][d] = fmaxf(red[0][d], red[0][d + s]);
                        red[1][d] = fmaxf(red[1][d], red[1][d + s]);
                    }
                    __syncthreads();
                }
                const float amk = red[0][0], amv = red[1][0];
                const float mulk = amk == 0.0f ? 1.0f : __fdiv_rn(127.0f, amk);
                const float mulv = amv == 0.0f ? 1.0f : __fdiv_rn(127.0f, amv);
                if (blk < kv.P_max) {
                    const size_t po = u * kv.P_pad + blk;
                    kv.pool_k[po * 64 + d] = (int8_t)(int)roundf(__fmul_rn(mk, mulk));
                    kv.pool_v[u * kv.P_pad * 64 + kv_voff(blk, d)] = (int8_t)(int)roundf(__fmul_rn(mv, mulv));
                    if (d == 0) {
                        kv.pool_ks[po] = amk == 0.0f ? 1.0f : __fdiv_rn(amk, 127.0f);
                        kv.pool_vs[po] = amv == 0.0f ? 1.0f : __fdiv_rn(amv, 127.0f);
                    }
                }
                ak = 0.0;
                av = 0.0;
            }
        }
        __syncthreads();  // every lane has read the old slot
        kv.ring_k[e * 64 + d] = nk;
        kv.ring_v[ve] = nv;
        if (d == 0) {
            kv.ring_ks[e] = nks;
            kv.ring_vs[e] = nvs;
        }
        __syncthreads();
    }
    kv.acc_k[u * 64 + d] = ak;
    kv.acc_v[u * 64 + d] = av;
}

pf_status kv_commit(const KvCache& kv, const RowBatch& rb, const int* n_commit, Staged staged, int M_stride,
                    cudaStream_t stream) {
    dim3 grid(rb.nb, kv.L, kv.G);
    kv_commit_kernel<<<grid, 64, 0, stream>>>(kv, rb, n_commit, staged, M_stride);
    return launch_check("kv_commit");
}

}  // namespace pf

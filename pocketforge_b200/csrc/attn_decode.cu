// attn_decode.cu — tensor-core attention for verify batches (up to 32 query
// rows per kv head: q heads sharing the kv head x rows of the sequence).
//
// Same semantics as attention() in attention.cu (KVCache::attention_scores /
// attention_weighted_sum + Engine::compute_attention, src/kv_cache.cpp:129-198,
// src/engine.cpp:753-779).  The committed pool and window entries — all but a
// handful — go through int8 tensor-core MMAs:
//   scores  S = Q . K^T : Q (fp32 after RoPE) split into three int8 digit
//           planes per row (x = s(q1 + q2/254 + q3/254^2)); K is the stored
//           int8; int32 products are exact, recombined in fp32 (~1e-7 rel.).
//   output  O = P . V   : per 32-entry block, w = p * v_scale split into three
//           int8 digit planes relative to the row's block maximum; V int8.
// An online softmax (running max / sum, rescaled per block) joins the blocks.
// Sink entries, pool entries finalized inside this batch, the batch's own
// earlier rows (staged) and the float self term are added in fp32 at the end,
// after the four warps' partial states are merged.
//
// Fragment layouts (mma.m16n8k32.s8): the k index of an MMA can be any
// permutation of the reduced dimension as long as A and B agree.
//   QK: thread (g, t) loads 16 contiguous bytes [16t, 16t+16) of K row g and
//       of Q rows g, g+8; k-step 0 uses bytes 0-7, k-step 1 bytes 8-15.
//   PV: the QK accumulator of thread (g, t) holds entries 8j + 2t + {0,1}
//       (j = n8 tile); those 8 values become its A fragment directly, so V is
//       stored dim-major per 32-entry block with the matching entry order
//       (kv_vpos in kv.cuh) and every B fragment is one 8-byte load.
#include "kv.cuh"

namespace pf {

namespace {

constexpr int QR = 32;  // padded query rows per CTA

__device__ __forceinline__ void mma_s8(int32_t (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float comb(int32_t a, int32_t b, int32_t c) {
    const float r = 1.0f / 254.0f;
    return (float)a + ((float)b + (float)c * r) * r;
}

__device__ __forceinline__ void digits3(float x, float mul, int& d1, int& d2, int& d3) {
    const float r0 = x * mul;
    const float f1 = rintf(r0);
    const float r1 = (r0 - f1) * 254.0f;
    const float f2 = rintf(r1);
    const float r2 = (r1 - f2) * 254.0f;
    d1 = (int)f1;
    d2 = (int)f2;
    d3 = (int)fminf(127.0f, fmaxf(-127.0f, rintf(r2)));
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return (uint32_t)(a & 0xFF) | ((uint32_t)(b & 0xFF) << 8) | ((uint32_t)(c & 0xFF) << 16) | ((uint32_t)(d & 0xFF) << 24);
}

__device__ __forceinline__ float quad_max(float v) {
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
    return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}
__device__ __forceinline__ float quad_sum(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    return v + __shfl_xor_sync(0xffffffffu, v, 2);
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

struct Online {  // running softmax state of one query row held by a lane pair
    float m, l;
};

}  // namespace

__global__ void __launch_bounds__(128) attn_decode_kernel(KvCache kv, int layer, RowBatch rb, const float* __restrict__ qkv,
                                                          int ld, int k_col, int v_col, int H, Staged st, SpecPool sp,
                                                          float* __restrict__ out, int ldo) {
    const int b = blockIdx.x, g = blockIdx.y;
    const int n = rb.n[b];
    if (n == 0) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
    const int qpk = H / kv.G;
    const int rows = qpk * n;  // <= QR (checked on the host)
    const int L0 = rb.len0[b], row0 = rb.row0[b];
    const int plast = L0 + n - 1;
    const int cs = min(L0, kv.S);
    const int nb0 = kv_pool_count(L0, kv.S, kv.Wr, kv.pb);
    const int npool = kv_pool_count(plast, kv.S, kv.Wr, kv.pb);
    const int qlo = max(kv.S, L0 - kv.Wr);
    const int nwin = max(0, L0 - qlo);
    const int s0 = (qlo - kv.S) % kv.Wr;  // ring slot of the oldest window position
    const size_t u = kv.unit(b, layer, g);
    const float scale = 0.125f;           // 1/sqrt(64)

    __shared__ __align__(16) int8_t qd[3][QR][64];
    __shared__ float qsc[QR];
    __shared__ float mw[4][QR], lw[4][QR];
    __shared__ float accw[4][QR][64];

    // ---- queries -> three digit planes (row ri = hh*n + r, head g + hh*G) ----
    for (int ri = warp; ri < QR; ri += 4) {
        float x0 = 0.0f, x1 = 0.0f;
        if (ri < rows) {
            const int hh = ri / n, r = ri % n;
            const float* q = qkv + (size_t)(row0 + r) * ld + (size_t)(g + hh * kv.G) * 64;
            x0 = q[lane];
            x1 = q[lane + 32];
        }
        const float amax = warp_max(fmaxf(fabsf(x0), fabsf(x1)));
        const float mul = (amax == 0.0f || !isfinite(amax)) ? 0.0f : 127.0f / amax;
        int a1, a2, a3, b1, b2, b3;
        digits3(x0, mul, a1, a2, a3);
        digits3(x1, mul, b1, b2, b3);
        qd[0][ri][lane] = (int8_t)a1;
        qd[1][ri][lane] = (int8_t)a2;
        qd[2][ri][lane] = (int8_t)a3;
        qd[0][ri][lane + 32] = (int8_t)b1;
        qd[1][ri][lane + 32] = (int8_t)b2;
        qd[2][ri][lane + 32] = (int8_t)b3;
        if (lane == 0) qsc[ri] = !isfinite(amax) ? __int_as_float(0x7fc00000) : amax / 127.0f;
    }
    __syncthreads();

    // ---- per-warp online softmax over the committed pool and window blocks ----
    Online st4[4];  // rows gid, gid+8, 16+gid, 24+gid  (index mb*2 + h)
    float acc[2][8][4];
#pragma unroll
    for (int i = 0; i < 4; i++) st4[i] = {-INFINITY, 0.0f};
#pragma unroll
    for (int mb = 0; mb < 2; mb++)
#pragma unroll
        for (int nt = 0; nt < 8; nt++)
#pragma unroll
            for (int c = 0; c < 4; c++) acc[mb][nt][c] = 0.0f;
    float qs_r[4];
#pragma unroll
    for (int i = 0; i < 4; i++) qs_r[i] = qsc[(i >> 1) * 16 + (i & 1) * 8 + gid];

    const int pool_blocks = (nb0 + 31) / 32;
    const int ring_blocks = (nwin + 31) / 32;
    const int nblk = pool_blocks + ring_blocks;
    for (int blk = warp; blk < nblk; blk += 4) {
        const bool is_pool = blk < pool_blocks;
        const int bi = is_pool ? blk : blk - pool_blocks;
        const int8_t* kbase;
        const int8_t* vbase;
        const float* ksb;
        const float* vsb;
        if (is_pool) {
            kbase = kv.pool_k + ((u * kv.P_pad) + (size_t)bi * 32) * 64;
            vbase = kv.pool_v + ((u * kv.P_pad) + (size_t)bi * 32) * 64;
            ksb = kv.pool_ks + u * kv.P_pad + (size_t)bi * 32;
            vsb = kv.pool_vs + u * kv.P_pad + (size_t)bi * 32;
        } else {
            kbase = kv.ring_k + ((u * kv.W_pad) + (size_t)bi * 32) * 64;
            vbase = kv.ring_v + ((u * kv.W_pad) + (size_t)bi * 32) * 64;
            ksb = kv.ring_ks + u * kv.W_pad + (size_t)bi * 32;
            vsb = kv.ring_vs + u * kv.W_pad + (size_t)bi * 32;
        }
        // Entries of this thread's accumulator columns: e = 8j + 2*tig + c.
        // Validity and the last row that may see the entry.
        int rhi[8];
        float ksv[8], vsv[8];
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int c = 0; c < 2; c++) {
                const int e = 8 * j + 2 * tig + c;
                int hi = -1;
                if (is_pool) {
                    if (bi * 32 + e < nb0) hi = 1 << 30;
                } else {
                    const int slot = bi * 32 + e;
                    if (slot < kv.Wr) {
                        const int off = (slot - s0 + kv.Wr) % kv.Wr;
                        if (off < nwin) hi = qlo + off + kv.Wr - L0;
                    }
                }
                rhi[j * 2 + c] = hi;
                ksv[j * 2 + c] = hi >= 0 ? ksb[e] : 0.0f;
                vsv[j * 2 + c] = hi >= 0 ? vsb[e] : 0.0f;
            }
        // K fragments: entry 8j + gid, bytes [16*tig, 16*tig+16)
        uint4 kf[4];
#pragma unroll
        for (int j = 0; j < 4; j++) kf[j] = *reinterpret_cast<const uint4*>(kbase + (size_t)(8 * j + gid) * 64 + 16 * tig);
        // ---- scores ----
        float s[2][4][4];
#pragma unroll
        for (int mb = 0; mb < 2; mb++) {
            int32_t ac[3][4][4];
#pragma unroll
            for (int p = 0; p < 3; p++)
#pragma unroll
                for (int j = 0; j < 4; j++)
#pragma unroll
                    for (int c = 0; c < 4; c++) ac[p][j][c] = 0;
#pragma unroll
            for (int p = 0; p < 3; p++) {
                const uint4 qa = *reinterpret_cast<const uint4*>(&qd[p][mb * 16 + gid][16 * tig]);
                const uint4 qb = *reinterpret_cast<const uint4*>(&qd[p][mb * 16 + gid + 8][16 * tig]);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    mma_s8(ac[p][j], qa.x, qb.x, qa.y, qb.y, kf[j].x, kf[j].y);
                    mma_s8(ac[p][j], qa.z, qb.z, qa.w, qb.w, kf[j].z, kf[j].w);
                }
            }
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int r = mb * 16 + gid + (c >> 1) * 8;
                    const int e2 = j * 2 + (c & 1);
                    const float v = comb(ac[0][j][c], ac[1][j][c], ac[2][j][c]) * qs_r[mb * 2 + (c >> 1)] * ksv[e2] * scale;
                    const int rr = r % max(n, 1);  // row of the sequence for query row r
                    s[mb][j][c] = (r < rows && rr <= rhi[e2]) ? v : -INFINITY;
                }
        }
        // ---- online softmax update, weights w = p * v_scale ----
        uint32_t wa[2][3][4];  // A fragments of the three digit planes
        float wscale[4];
#pragma unroll
        for (int mb = 0; mb < 2; mb++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int si = mb * 2 + h;
                float bm = -INFINITY;
#pragma unroll
                for (int j = 0; j < 4; j++)
#pragma unroll
                    for (int c = 0; c < 2; c++) bm = fmaxf(bm, s[mb][j][h * 2 + c]);
                bm = quad_max(bm);
                const float m_new = fmaxf(st4[si].m, bm);
                float corr = 1.0f;
                float pw[8];
                float psum = 0.0f, wmax = 0.0f;
                if (m_new == -INFINITY) {
#pragma unroll
                    for (int k = 0; k < 8; k++) pw[k] = 0.0f;
                } else {
                    corr = (st4[si].m == -INFINITY) ? 0.0f : __expf(st4[si].m - m_new);
#pragma unroll
                    for (int j = 0; j < 4; j++)
#pragma unroll
                        for (int c = 0; c < 2; c++) {
                            const float sv = s[mb][j][h * 2 + c];
                            const float p = (sv == -INFINITY) ? 0.0f : __expf(sv - m_new);
                            psum += p;
                            pw[j * 2 + c] = p * vsv[j * 2 + c];
                            wmax = fmaxf(wmax, fabsf(pw[j * 2 + c]));
                        }
                }
                psum = quad_sum(psum);
                wmax = quad_max(wmax);
                st4[si].l = st4[si].l * corr + psum;
                st4[si].m = m_new;
#pragma unroll
                for (int nt = 0; nt < 8; nt++) {
                    acc[mb][nt][h * 2] *= corr;
                    acc[mb][nt][h * 2 + 1] *= corr;
                }
                const float mul = (wmax == 0.0f || !isfinite(wmax)) ? 0.0f : 127.0f / wmax;
                wscale[si] = wmax / 127.0f;
                int d[3][8];
#pragma unroll
                for (int k = 0; k < 8; k++) digits3(pw[k], mul, d[0][k], d[1][k], d[2][k]);
                // a0/a1 (k = 4*tig + 0..3): tiles 0,1; a2/a3 (k = 16 + 4*tig + 0..3): tiles 2,3
#pragma unroll
                for (int p = 0; p < 3; p++) {
                    wa[mb][p][h] = pack4(d[p][0], d[p][1], d[p][2], d[p][3]);
                    wa[mb][p][2 + h] = pack4(d[p][4], d[p][5], d[p][6], d[p][7]);
                }
            }
        // ---- O += W . V ----
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
            const uint2 vf = *reinterpret_cast<const uint2*>(vbase + (size_t)(nt * 8 + gid) * 32 + 8 * tig);
#pragma unroll
            for (int mb = 0; mb < 2; mb++) {
                int32_t o[3][4];
#pragma unroll
                for (int p = 0; p < 3; p++) {
                    o[p][0] = o[p][1] = o[p][2] = o[p][3] = 0;
                    // A regs: a0 row g (k low), a1 row g+8 (k low), a2 row g (k high), a3 row g+8 (k high)
                    mma_s8(o[p], wa[mb][p][0], wa[mb][p][1], wa[mb][p][2], wa[mb][p][3], vf.x, vf.y);
                }
#pragma unroll
                for (int c = 0; c < 4; c++)
                    acc[mb][nt][c] += comb(o[0][c], o[1][c], o[2][c]) * wscale[mb * 2 + (c >> 1)];
            }
        }
    }

    // ---- merge the four warps ----
#pragma unroll
    for (int mb = 0; mb < 2; mb++)
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int r = mb * 16 + h * 8 + gid;
            if (tig == 0) {
                mw[warp][r] = st4[mb * 2 + h].m;
                lw[warp][r] = st4[mb * 2 + h].l;
            }
#pragma unroll
            for (int nt = 0; nt < 8; nt++) {
                accw[warp][r][nt * 8 + 2 * tig] = acc[mb][nt][h * 2];
                accw[warp][r][nt * 8 + 2 * tig + 1] = acc[mb][nt][h * 2 + 1];
            }
        }
    __syncthreads();

    // ---- per query row: merged state + sink, pool entries finalized in this
    // batch, staged rows, self term; then the output ----
    for (int ri = warp; ri < rows; ri += 4) {
        const int hh = ri / n, r = ri % n;
        const int h = g + hh * kv.G;
        const int row = row0 + r;
        const float* q = qkv + (size_t)row * ld + (size_t)h * 64;
        const float q0 = q[lane], q1 = q[lane + 32];
        float m = -INFINITY;
        for (int w = 0; w < 4; w++) m = fmaxf(m, mw[w][ri]);
        float l = 0.0f, o0 = 0.0f, o1 = 0.0f;
        if (m != -INFINITY)
            for (int w = 0; w < 4; w++) {
                const float f = (mw[w][ri] == -INFINITY) ? 0.0f : __expf(mw[w][ri] - m);
                l += lw[w][ri] * f;
                o0 += accw[w][ri][lane] * f;
                o1 += accw[w][ri][lane + 32] * f;
            }
        auto add = [&](const int8_t* kk, float ks, const int8_t* vv, float vs) {
            const float sc = warp_sum(q0 * ((float)kk[lane] * ks) + q1 * ((float)kk[lane + 32] * ks)) * scale;
            const float mn = fmaxf(m, sc);
            const float corr = (m == -INFINITY) ? 0.0f : __expf(m - mn);
            const float p = __expf(sc - mn);
            l = l * corr + p;
            o0 = o0 * corr + p * ((float)vv[lane] * vs);
            o1 = o1 * corr + p * ((float)vv[lane + 32] * vs);
            m = mn;
        };
        for (int e = 0; e < cs; e++)
            add(kv.sink_k + (u * kv.S + e) * 64, kv.sink_ks[u * kv.S + e], kv.sink_v + (u * kv.S + e) * 64,
                kv.sink_vs[u * kv.S + e]);
        for (int j = nb0; j < npool; j++) {
            if (r < kv.S + kv.Wr + (j + 1) * kv.pb - L0) continue;  // finalized by a later row
            const size_t o = ((size_t)b * kv.G + g) * sp.per + (j - nb0);
            add(sp.k + o * 64, sp.ks[o], sp.v + o * 64, sp.vs[o]);
        }
        for (int j = 0; j < r; j++) {
            const size_t o = (size_t)(row0 + j) * kv.G + g;
            add(st.k + o * 64, st.ks[o], st.v + o * 64, st.vs[o]);
        }
        {  // self term with the float k and v (src/engine.cpp:760-778)
            const float* ks = qkv + (size_t)row * ld + k_col + (size_t)g * 64;
            const float* vs = qkv + (size_t)row * ld + v_col + (size_t)g * 64;
            const float sc = warp_sum(q0 * ks[lane] + q1 * ks[lane + 32]) * scale;
            const float mn = fmaxf(m, sc);
            const float corr = (m == -INFINITY) ? 0.0f : __expf(m - mn);
            const float p = __expf(sc - mn);
            l = l * corr + p;
            o0 = o0 * corr + p * vs[lane];
            o1 = o1 * corr + p * vs[lane + 32];
        }
        const float inv = 1.0f / (l + 1e-10f);
        out[(size_t)row * ldo + (size_t)h * 64 + lane] = o0 * inv;
        out[(size_t)row * ldo + (size_t)h * 64 + lane + 32] = o1 * inv;
    }
}

bool attention_decode_supported(int H, int G, int max_rows) { return (H / G) * max_rows <= QR; }

pf_status attention_decode(const KvCache& kv, int layer, const RowBatch& rb, const float* qkv, int ldqkv, int k_col,
                           int v_col, int H, Staged st, SpecPool sp, float* out, int ldo, cudaStream_t stream) {
    PF_CHECK(kv.hd == 64, "attention_decode: head_dim must be 64");
    PF_CHECK(attention_decode_supported(H, kv.G, rb.max_rows), "attention_decode: too many query rows");
    dim3 grid(rb.nb, kv.G);
    attn_decode_kernel<<<grid, 128, 0, stream>>>(kv, layer, rb, qkv, ldqkv, k_col, v_col, H, st, sp, out, ldo);
    return launch_check("attention_decode");
}

}  // namespace pf

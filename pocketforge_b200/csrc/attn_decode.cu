// attn_decode.cu — tensor-core attention for verify batches (up to 32 query
// rows per kv head: q heads sharing the kv head x rows of the sequence).
//
// Same semantics as attention() in attention.cu (KVCache::attention_scores /
// attention_weighted_sum + Engine::compute_attention, src/kv_cache.cpp:129-198,
// src/engine.cpp:753-779).  Every int8 entry a row can see goes through int8
// tensor-core MMAs, 32 entries (one block) at a time:
//   scores  S = Q . K^T : Q (fp32 after RoPE) split into three int8 digit
//           planes per row (x = s(q1 + q2/254 + q3/254^2)); K is the stored
//           int8; int32 products are exact, recombined in fp32 (~1e-7 rel.).
//   output  O = P . V   : per block, w = p * v_scale split into three int8
//           digit planes relative to the row's block maximum; V int8.
// Blocks are the committed pool blocks, the window-ring blocks, and one
// extra block assembled in shared memory from the sink entries, the pool
// entries finalized inside this batch and the batch's own earlier rows
// (staged), each with the range of query rows that may see it.  The float
// self term of each row is added when the partial softmax states are merged.
//
// One CTA per (sequence, kv head), four warps.  The query rows form MT
// m-tiles of 16; the warps of an m-tile take the blocks of a chunk in turn
// (4/MT blocks per chunk) and keep their own online-softmax state.  Pool and
// ring blocks stream through a 4-stage cp.async ring in shared memory.
//
// Fragment layouts (mma.m16n8k32.s8): the k index of an MMA can be any
// permutation of the reduced dimension as long as A and B agree.
//   QK: thread (g, t) uses bytes [16t, 16t+16) of K row g and of Q rows g,
//       g+8; k-step 0 takes bytes 0-7, k-step 1 bytes 8-15.
//   PV: the QK accumulator of thread (g, t) holds entries 8j + 2t + {0,1}
//       (j = n8 tile); those 8 values become its A fragment directly, so V is
//       stored dim-major per 32-entry block with the matching entry order
//       (kv_vpos in kv.cuh) and every B fragment is one 8-byte load.
#include "kv.cuh"

namespace pf {

namespace {

constexpr int QR = 32;  // padded query rows per CTA
constexpr int NS = 4;   // cp.async stages
constexpr int BIG = 1 << 30;

__device__ __forceinline__ void mma_s8(int32_t (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Integer <-> float conversions and round-to-nearest-even of values below
// 2^22 in magnitude on the FMA / integer pipes: adding 1.5 * 2^23 leaves the
// value's nearest integer (ties to even, as rintf) in the low mantissa bits.
// Every value converted here is below 2^22: digit-plane products sum at most
// 64 * 127 * 127 terms, and the digits themselves lie in [-127, 127].
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
constexpr int kMagicBits = 0x4B400000;
__device__ __forceinline__ float i2f_small(int32_t a) { return __fsub_rn(__int_as_float(a + kMagicBits), kMagic); }

__device__ __forceinline__ float comb(int32_t a, int32_t b, int32_t c) {
    const float r = 1.0f / 254.0f;
    return i2f_small(a) + (i2f_small(b) + i2f_small(c) * r) * r;
}

__device__ __forceinline__ void digits3(float x, float mul, int& d1, int& d2, int& d3) {
    const float r0 = x * mul;
    const float t1 = __fadd_rn(r0, kMagic);  // rint(r0) + magic
    const float r1 = (r0 - __fsub_rn(t1, kMagic)) * 254.0f;
    const float t2 = __fadd_rn(r1, kMagic);
    const float r2 = (r1 - __fsub_rn(t2, kMagic)) * 254.0f;
    const float t3 = __fadd_rn(r2, kMagic);
    d1 = __float_as_int(t1) - kMagicBits;
    d2 = __float_as_int(t2) - kMagicBits;
    d3 = min(127, max(-127, __float_as_int(t3) - kMagicBits));
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

__device__ __forceinline__ void cp16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One 32-entry block in shared memory, in the global layouts of kv.cuh.
struct __align__(16) BlockBuf {
    int8_t k[32][64];  // entry-major
    int8_t v[2048];    // [64 dims][32 entries in kv_vpos order]
    float ks[32], vs[32];
};

template <int MT>
struct __align__(16) AttnSmem {
    static constexpr int WPM = 4 / MT;  // warps (= blocks per chunk) per m-tile
    int8_t qd[3][QR][64];               // query digit planes
    float qsc[QR];                      // query scales
    float s_self[QR];                   // self-term scores (scaled)
    float v_self[QR][64];               // self-term values
    BlockBuf ex;                        // the extra block
    int ex_lo[32], ex_hi[32];           // rows of the sequence that see each extra entry
    union {
        BlockBuf stage[NS][WPM];
        struct {
            float m[4][QR], l[4][QR];
            float acc[4][QR][64];
        } merge;
    } u;
};

struct Online {  // running softmax state of one query row held by a lane quad
    float m, l;
};

}  // namespace

template <int MT>
__global__ void __launch_bounds__(128, 3) attn_decode_kernel(KvCache kv, int layer, RowBatch rb, const float* __restrict__ qkv,
                                                          int ld, int k_col, int v_col, int H, Staged st, SpecPool sp,
                                                          float* __restrict__ out, int ldo, uint32_t* err) {
    constexpr int WPM = 4 / MT;
    extern __shared__ __align__(16) uint8_t attn_smem_raw[];
    AttnSmem<MT>& sm = *reinterpret_cast<AttnSmem<MT>*>(attn_smem_raw);
    const int b = blockIdx.x, g = blockIdx.y;
    const int n = rb.n[b];
    if (n == 0) return;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, tig = lane & 3;
    const int qpk = H / kv.G;
    const int rows = qpk * n;  // <= 16 * MT (checked on the host)
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
    const int n_spec = npool - nb0;
    const int n_ex = cs + n_spec + (n - 1);
    if (n_ex > 32 || rows > 16 * MT) {  // excluded by the host; never index past the tiles
        if (tid == 0 && err) atomicOr(err, ERR_BOUNDS);
        return;
    }
    const int pool_blocks = (nb0 + 31) / 32;
    const int ring_blocks = (nwin + 31) / 32;
    const int nkv = pool_blocks + ring_blocks;  // blocks that stream from memory
    const int nblk = nkv + (n_ex > 0 ? 1 : 0);
    const int nchunk = (nblk + WPM - 1) / WPM;

    // ---- cp.async of chunk c (its pool / ring blocks) into stage c % NS ----
    auto load_chunk = [&](int c) {
        BlockBuf* sb = sm.u.stage[c % NS];
#pragma unroll
        for (int j = 0; j < WPM; j++) {
            const int blk = c * WPM + j;
            if (blk >= nkv) break;
            const bool is_pool = blk < pool_blocks;
            const int bi = is_pool ? blk : blk - pool_blocks;
            const size_t e0 = (is_pool ? u * kv.P_pad : u * kv.W_pad) + (size_t)bi * 32;
            cp16(&sb[j].k[0][0] + tid * 16, (is_pool ? kv.pool_k : kv.ring_k) + e0 * 64 + tid * 16);
            cp16(sb[j].v + tid * 16, (is_pool ? kv.pool_v : kv.ring_v) + e0 * 64 + tid * 16);
            if (tid < 8)
                cp16(sb[j].ks + tid * 4, (is_pool ? kv.pool_ks : kv.ring_ks) + e0 + tid * 4);
            else if (tid < 16)
                cp16(sb[j].vs + (tid - 8) * 4, (is_pool ? kv.pool_vs : kv.ring_vs) + e0 + (tid - 8) * 4);
        }
    };
#pragma unroll
    for (int c = 0; c < NS - 1; c++) {
        if (c < nchunk) load_chunk(c);
        cp_commit();
    }

    // ---- queries -> digit planes; self-term score and value ----
#pragma unroll 2
    for (int ri = warp; ri < QR; ri += 4) {
        float x0 = 0.0f, x1 = 0.0f, k0 = 0.0f, k1 = 0.0f, v0 = 0.0f, v1 = 0.0f;
        if (ri < rows) {
            const int hh = ri / n, r = ri % n;
            const float* row = qkv + (size_t)(row0 + r) * ld;
            const float* q = row + (size_t)(g + hh * kv.G) * 64;
            x0 = q[lane];
            x1 = q[lane + 32];
            k0 = row[k_col + g * 64 + lane];
            k1 = row[k_col + g * 64 + lane + 32];
            v0 = row[v_col + g * 64 + lane];
            v1 = row[v_col + g * 64 + lane + 32];
        }
        const float amax = warp_max(fmaxf(fabsf(x0), fabsf(x1)));
        const float mul = (amax == 0.0f || !isfinite(amax)) ? 0.0f : 127.0f / amax;
        int a1, a2, a3, b1, b2, b3;
        digits3(x0, mul, a1, a2, a3);
        digits3(x1, mul, b1, b2, b3);
        sm.qd[0][ri][lane] = (int8_t)a1;
        sm.qd[1][ri][lane] = (int8_t)a2;
        sm.qd[2][ri][lane] = (int8_t)a3;
        sm.qd[0][ri][lane + 32] = (int8_t)b1;
        sm.qd[1][ri][lane + 32] = (int8_t)b2;
        sm.qd[2][ri][lane + 32] = (int8_t)b3;
        // self term with the float k and v (src/engine.cpp:760-778)
        const float sc = warp_sum(x0 * k0 + x1 * k1) * scale;
        if (lane == 0) {
            sm.qsc[ri] = !isfinite(amax) ? __int_as_float(0x7fc00000) : amax / 127.0f;
            sm.s_self[ri] = sc;
        }
        sm.v_self[ri][lane] = v0;
        sm.v_self[ri][lane + 32] = v1;
    }

    // ---- the extra block: sink entries, pool entries finalized inside the
    // batch (visible from the row that finalizes them), staged earlier rows ----
    auto ex_src = [&](int e, const int8_t*& kp, const int8_t*& vp, float& ks, float& vs, int& lo) {
        if (e < cs) {
            const size_t o = u * kv.S + e;
            kp = kv.sink_k + o * 64;
            vp = kv.sink_v + o * 64;
            ks = kv.sink_ks[o];
            vs = kv.sink_vs[o];
            lo = 0;
        } else if (e < cs + n_spec) {
            const int j = nb0 + (e - cs);
            const size_t o = ((size_t)b * kv.G + g) * sp.per + (j - nb0);
            kp = sp.k + o * 64;
            vp = sp.v + o * 64;
            ks = sp.ks[o];
            vs = sp.vs[o];
            lo = kv.S + kv.Wr + (j + 1) * kv.pb - L0;
        } else {
            const int j = e - cs - n_spec;
            const size_t o = (size_t)(row0 + j) * kv.G + g;
            kp = st.k + o * 64;
            vp = st.v + o * 64;
            ks = st.ks[o];
            vs = st.vs[o];
            lo = j + 1;
        }
    };
    {
        const int e = tid >> 2, q4 = tid & 3;  // entry e, dims [16*q4, 16*q4 + 16)
        uint4 kk = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
        float ks = 0.0f, vs = 0.0f;
        int lo = BIG, hi = -1;
        if (e < n_ex) {
            const int8_t *kp, *vp;
            ex_src(e, kp, vp, ks, vs, lo);
            hi = BIG;
            kk = *reinterpret_cast<const uint4*>(kp + 16 * q4);
            vv = *reinterpret_cast<const uint4*>(vp + 16 * q4);
        }
        *reinterpret_cast<uint4*>(&sm.ex.k[e][16 * q4]) = kk;
        const uint8_t* vb = reinterpret_cast<const uint8_t*>(&vv);
        const int pos = kv_vpos(e);
#pragma unroll
        for (int i = 0; i < 16; i++) sm.ex.v[(16 * q4 + i) * 32 + pos] = (int8_t)vb[i];
        if (q4 == 0) {
            sm.ex.ks[e] = ks;
            sm.ex.vs[e] = vs;
            sm.ex_lo[e] = lo;
            sm.ex_hi[e] = hi;
        }
    }
    __syncthreads();

    // ---- this warp's m-tile: query fragments and row bookkeeping ----
    const int mt = warp / WPM, jw = warp % WPM;
    uint4 qa[3], qb[3];
#pragma unroll
    for (int p = 0; p < 3; p++) {
        qa[p] = *reinterpret_cast<const uint4*>(&sm.qd[p][mt * 16 + gid][16 * tig]);
        qb[p] = *reinterpret_cast<const uint4*>(&sm.qd[p][mt * 16 + gid + 8][16 * tig]);
    }
    int ri2[2], rr2[2];
    float qs2[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        ri2[h] = mt * 16 + gid + 8 * h;
        rr2[h] = ri2[h] < rows ? ri2[h] % n : -1;  // padding row: every entry has lo >= 0
        qs2[h] = sm.qsc[ri2[h]];
    }
    Online st2[2] = {{-INFINITY, 0.0f}, {-INFINITY, 0.0f}};
    float acc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; nt++)
#pragma unroll
        for (int c = 0; c < 4; c++) acc[nt][c] = 0.0f;

    for (int c = 0; c < nchunk; c++) {
        cp_wait<NS - 2>();
        __syncthreads();  // chunk c landed; stage (c - 1) % NS is free again
        if (c + NS - 1 < nchunk) load_chunk(c + NS - 1);
        cp_commit();
        const int blk = c * WPM + jw;
        if (blk >= nblk) continue;
        const bool is_ex = blk == nkv;
        const BlockBuf& bb = is_ex ? sm.ex : sm.u.stage[c % NS][jw];
        // Entries of this thread's accumulator columns: e = 8j + 2*tig + cc,
        // with the rows [lo, hi] of the sequence that may see them.
        int lo8[8], hi8[8];
        float ksv[8], vsv[8];
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int cc = 0; cc < 2; cc++) {
                const int e = 8 * j + 2 * tig + cc;
                int lo = BIG, hi = -1;
                if (is_ex) {
                    lo = sm.ex_lo[e];
                    hi = sm.ex_hi[e];
                } else if (blk < pool_blocks) {
                    if (blk * 32 + e < nb0) lo = 0, hi = BIG;
                } else {
                    const int slot = (blk - pool_blocks) * 32 + e;
                    if (slot < kv.Wr) {
                        const int off = slot >= s0 ? slot - s0 : slot - s0 + kv.Wr;  // (slot - s0) mod Wr
                        if (off < nwin) lo = 0, hi = qlo + off + kv.Wr - L0;
                    }
                }
                const bool valid = hi >= 0 && lo < BIG;
                lo8[j * 2 + cc] = lo;
                hi8[j * 2 + cc] = hi;
                ksv[j * 2 + cc] = valid ? bb.ks[e] : 0.0f;
                vsv[j * 2 + cc] = valid ? bb.vs[e] : 0.0f;  // a masked entry must not bring a NaN scale in
            }
        // ---- scores ----
        float s[4][4];  // [n8 tile j][accumulator c]: rows gid (c < 2), gid + 8 (c >= 2)
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint4 kf = *reinterpret_cast<const uint4*>(&bb.k[8 * j + gid][16 * tig]);
            int32_t ac[3][4];
#pragma unroll
            for (int p = 0; p < 3; p++) {
                ac[p][0] = ac[p][1] = ac[p][2] = ac[p][3] = 0;
                mma_s8(ac[p], qa[p].x, qb[p].x, qa[p].y, qb[p].y, kf.x, kf.y);
                mma_s8(ac[p], qa[p].z, qb[p].z, qa[p].w, qb[p].w, kf.z, kf.w);
            }
#pragma unroll
            for (int cc = 0; cc < 4; cc++) {
                const int h = cc >> 1, e2 = j * 2 + (cc & 1);
                const float v = comb(ac[0][cc], ac[1][cc], ac[2][cc]) * qs2[h] * ksv[e2] * scale;
                s[j][cc] = (rr2[h] >= lo8[e2] && rr2[h] <= hi8[e2]) ? v : -INFINITY;
            }
        }
        // ---- online softmax update, weights w = p * v_scale ----
        uint32_t wa[3][4];  // A fragments of the three digit planes
        float wscale[2];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            float bm = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int cc = 0; cc < 2; cc++) bm = fmaxf(bm, s[j][h * 2 + cc]);
            bm = quad_max(bm);
            const float m_new = fmaxf(st2[h].m, bm);
            float corr = 1.0f;
            float pw[8];
            float psum = 0.0f, wmax = 0.0f;
            if (m_new == -INFINITY) {
#pragma unroll
                for (int k = 0; k < 8; k++) pw[k] = 0.0f;
            } else {
                corr = (st2[h].m == -INFINITY) ? 0.0f : __expf(st2[h].m - m_new);
#pragma unroll
                for (int j = 0; j < 4; j++)
#pragma unroll
                    for (int cc = 0; cc < 2; cc++) {
                        const float sv = s[j][h * 2 + cc];
                        const float p = (sv == -INFINITY) ? 0.0f : __expf(sv - m_new);
                        psum += p;
                        pw[j * 2 + cc] = p * vsv[j * 2 + cc];
                        wmax = fmaxf(wmax, fabsf(pw[j * 2 + cc]));
                    }
            }
            psum = quad_sum(psum);
            wmax = quad_max(wmax);
            st2[h].l = st2[h].l * corr + psum;
            st2[h].m = m_new;
#pragma unroll
            for (int nt = 0; nt < 8; nt++) {
                acc[nt][h * 2] *= corr;
                acc[nt][h * 2 + 1] *= corr;
            }
            const float mul = (wmax == 0.0f || !isfinite(wmax)) ? 0.0f : 127.0f / wmax;
            wscale[h] = wmax / 127.0f;
            int d[3][8];
#pragma unroll
            for (int k = 0; k < 8; k++) digits3(pw[k], mul, d[0][k], d[1][k], d[2][k]);
            // a0/a1 (k = 4*tig + 0..3): tiles 0,1; a2/a3 (k = 16 + 4*tig + 0..3): tiles 2,3
#pragma unroll
            for (int p = 0; p < 3; p++) {
                wa[p][h] = pack4(d[p][0], d[p][1], d[p][2], d[p][3]);
                wa[p][2 + h] = pack4(d[p][4], d[p][5], d[p][6], d[p][7]);
            }
        }
        // ---- O += W . V ----
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
            const uint2 vf = *reinterpret_cast<const uint2*>(&bb.v[(nt * 8 + gid) * 32 + 8 * tig]);
            int32_t o[3][4];
#pragma unroll
            for (int p = 0; p < 3; p++) {
                o[p][0] = o[p][1] = o[p][2] = o[p][3] = 0;
                // A regs: a0 row g (k low), a1 row g+8 (k low), a2 row g (k high), a3 row g+8 (k high)
                mma_s8(o[p], wa[p][0], wa[p][1], wa[p][2], wa[p][3], vf.x, vf.y);
            }
#pragma unroll
            for (int cc = 0; cc < 4; cc++) acc[nt][cc] += comb(o[0][cc], o[1][cc], o[2][cc]) * wscale[cc >> 1];
        }
    }
    cp_wait<0>();
    __syncthreads();  // the stage ring becomes the merge area

    // ---- partial states of the warps -> shared memory ----
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int r = ri2[h];
        if (tig == 0) {
            sm.u.merge.m[warp][r] = st2[h].m;
            sm.u.merge.l[warp][r] = st2[h].l;
        }
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
            sm.u.merge.acc[warp][r][nt * 8 + 2 * tig] = acc[nt][h * 2];
            sm.u.merge.acc[warp][r][nt * 8 + 2 * tig + 1] = acc[nt][h * 2 + 1];
        }
    }
    __syncthreads();

    // ---- per query row: merge the m-tile's warps and the self term ----
    for (int ri = warp; ri < rows; ri += 4) {
        const int hh = ri / n, r = ri % n;
        const int h = g + hh * kv.G;
        const int w0 = (ri / 16) * WPM;
        const float ss = sm.s_self[ri];
        float m = ss;
#pragma unroll
        for (int w = 0; w < WPM; w++) m = fmaxf(m, sm.u.merge.m[w0 + w][ri]);
        float l = 0.0f, o0 = 0.0f, o1 = 0.0f;
#pragma unroll
        for (int w = 0; w < WPM; w++) {
            const float mw = sm.u.merge.m[w0 + w][ri];
            const float f = (mw == -INFINITY) ? 0.0f : __expf(mw - m);
            l += sm.u.merge.l[w0 + w][ri] * f;
            o0 += sm.u.merge.acc[w0 + w][ri][lane] * f;
            o1 += sm.u.merge.acc[w0 + w][ri][lane + 32] * f;
        }
        const float ps = __expf(ss - m);
        l += ps;
        o0 += ps * sm.v_self[ri][lane];
        o1 += ps * sm.v_self[ri][lane + 32];
        const float inv = 1.0f / (l + 1e-10f);
        const int row = row0 + r;
        out[(size_t)row * ldo + (size_t)h * 64 + lane] = o0 * inv;
        out[(size_t)row * ldo + (size_t)h * 64 + lane + 32] = o1 * inv;
    }
}

bool attention_decode_supported(const KvCache& kv, int H, int max_rows) {
    const int rows = (H / kv.G) * max_rows;
    const int spec = max_rows > 1 ? ceil_div(max_rows - 1, kv.pb) + 1 : 1;  // pool entries a batch can finalize
    return rows <= QR && kv.S + spec + max_rows - 1 <= 32;
}

template <int MT>
static pf_status launch_decode(const KvCache& kv, int layer, const RowBatch& rb, const float* qkv, int ldqkv, int k_col,
                               int v_col, int H, Staged st, SpecPool sp, float* out, int ldo, cudaStream_t stream) {
    const int smem = (int)sizeof(AttnSmem<MT>);
    static bool attr = false;
    if (!attr) {
        PF_CUDA(cudaFuncSetAttribute(attn_decode_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr = true;
    }
    dim3 grid(rb.nb, kv.G);
    attn_decode_kernel<MT><<<grid, 128, smem, stream>>>(kv, layer, rb, qkv, ldqkv, k_col, v_col, H, st, sp, out, ldo,
                                                         device_error_flag());
    return launch_check("attention_decode");
}

pf_status attention_decode(const KvCache& kv, int layer, const RowBatch& rb, const float* qkv, int ldqkv, int k_col,
                           int v_col, int H, Staged st, SpecPool sp, float* out, int ldo, cudaStream_t stream) {
    PF_CHECK(kv.hd == 64, "attention_decode: head_dim must be 64");
    PF_CHECK(attention_decode_supported(kv, H, rb.max_rows), "attention_decode: too many query rows");
    if ((H / kv.G) * rb.max_rows <= 16)
        return launch_decode<1>(kv, layer, rb, qkv, ldqkv, k_col, v_col, H, st, sp, out, ldo, stream);
    return launch_decode<2>(kv, layer, rb, qkv, ldqkv, k_col, v_col, H, st, sp, out, ldo, stream);
}

}  // namespace pf

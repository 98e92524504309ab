// attn_decode.cu — tensor-core attention for verify batches (up to 32 query
// rows per kv head: q heads sharing the kv head x rows of the sequence).
//
// Same semantics as attention() in attention.cu (KVCache::attention_scores /
// attention_weighted_sum + Engine::compute_attention, src/kv_cache.cpp:129-198,
// src/engine.cpp:753-779).  Every int8 entry a row can see goes through
// tensor-core MMAs, 32 entries (one block) at a time, with the entries as the
// MMAs' M dimension and the query rows as N (8-row tiles: 20 rows of a
// K = 4 verify batch pad to 24, not to 32):
//   scores  S^T = K . Q^T : Q (fp32 after RoPE) split into three int8 digit
//           planes per row (x = s(q1 + q2/254 + q3/254^2)), K the stored int8,
//           mma.sync m16n8k32.s8: the int32 products are exact and are
//           recombined in fp32 (~1e-7 relative, unbiased);
//           s_raw = S * k_scale, and the score in log2 units is f * s_raw with
//           f = s * log2(e) / sqrt(64).
//   output  O^T = V^T . W^T : w = p * v_scale / 2^E (E = a power-of-two
//           reference for the v scales, per warp) split into two fp16 planes,
//           w = hi + lo (hi truncated to 11 significant bits, lo the
//           fp16-rounded remainder: ~22 bits), V the stored int8, exact in
//           fp16; mma.sync m16n8k16 with fp32 accumulators.  The score
//           accumulator of a thread (entry e, rows 2t, 2t+1) is one row of an
//           8 x 8 fp16 tile; movmatrix.trans turns it into the B fragment of
//           the value MMA.  Each block's products start from a zero
//           accumulator (the small plane first) and are added to the running
//           sums with a rounded fp32 add, so the tensor cores' accumulation
//           rounding does not build up over the context.
// Online softmax per row with a lazily raised maximum: the reference point
// moves only when a block's maximum exceeds it by more than 8 (log2 units),
// so p = 2^((s_raw - m) f) stays <= 2^8 and the fp16 planes stay in range.
// A thread checks its own entries; only when some thread sees a score past
// the limit does the warp reduce the rows' maxima (shuffles over the 8
// threads sharing a row).  The row sums are per-thread partial sums, reduced
// once at the end.  Maxima stay in the raw units of the scores, and every
// exponent is an exact difference of two raw scores times f (as exp(s - max)
// in the reference): a product f * m, rounded, would cost an ulp of a large
// number.
//
// Blocks are the committed pool blocks, the window-ring blocks, and one extra
// block assembled in shared memory from the sink entries, the pool entries
// finalized inside this batch and the batch's own earlier rows (staged), each
// with the range of query rows that may see it.  The float self term of each
// row is added when the partial softmax states are merged.
//
// Grid (sequence, kv head, split).  A split takes a contiguous range of the
// (sequence, kv head)'s blocks; its three warps take the blocks of the range
// in turn, each with all query rows (NT tiles of 8) and its own cp.async
// ring, so the block loop has no CTA-wide barrier.  Three warps and 168
// registers a thread let four CTAs share an SM, so the 512 (sequence, kv
// head) units of a 64-sequence batch run as one wave (with four warps per
// CTA, three CTAs fit and the last 68 units formed a second wave that took
// ~40% of the launch).  The warps' states are merged in shared memory; with
// more than one split each split writes its state to a workspace and the last
// split to arrive (a counter per (sequence, kv head), reset by that split)
// merges them, adds the self term and writes the output.
//
// Fragment layouts: the k index of an MMA can be any permutation of the
// reduced dimension as long as A and B agree.
//   QK (m16n8k32): thread (g, t) uses bytes [16t, 16t+16) of K rows g, g+8
//       (A) and of query row g of the tile (B); k-step 0 takes bytes 0-7,
//       k-step 1 bytes 8-15, so the digit planes are stored in natural order.
//   PV (m16n8k16): A = V^T, thread (g, t) needs entries 16 ks + {2t, 2t+1,
//       2t+8, 2t+9} of dims g, g+8; V is stored dim-major per 32-entry block
//       in that entry order (kv_vpos in kv.cuh): one 8-byte load per dim row
//       gives both k-steps.
#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

#include "kv.cuh"

namespace pf {

namespace {

constexpr int QR = 32;   // query rows per CTA at most
// Query rows a CTA takes: 24 (three 8-row tiles) while the q heads sharing a
// kv head fit, so that wide batches (prefill chunks) also run the 168-register
// kernel at four CTAs per SM; 32 otherwise.
__host__ __device__ inline int cta_query_rows(int qpk) { return qpk <= 24 ? 24 : QR; }
constexpr int ACC_STRIDE = 68;  // floats per row of the warps' merge sums
constexpr int NW = 3;    // warps per CTA (3: four CTAs fit an SM, one wave for 512 units)
constexpr int NT_THREADS = 32 * NW;
constexpr int NSW = 3;   // cp.async stages per warp (two blocks of lookahead)
constexpr int BIG = 1 << 30;
constexpr int PART = 68; // floats per (split, row) partial state: m, l, pad, pad, o[64]
constexpr int kMaxSplits = 8;  // context splits per (sequence, kv head, row group)
constexpr int NEXMAX = 4; // extra blocks (sinks, in-batch pool entries, earlier rows of the batch)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kMaxLead = 8.0f;  // log2 units a block max may exceed the reference before it moves

// The MMAs below are plain (non-volatile) asm: they only read and write
// registers, so the compiler may interleave independent accumulator chains.
__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_s8(int32_t (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm(
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

// a + b/254 + c/254^2 from the three planes' exact sums: b*254 + c is exact
// in int32 (|b| <= 64*127*127); its conversion rounds only the second-order
// part, and one fused multiply-add rounds the result.
__device__ __forceinline__ float comb(int32_t a, int32_t b, int32_t c) {
    const float r2 = 1.0f / (254.0f * 254.0f);
    return __fmaf_rn(__int2float_rn(b * 254 + c), r2, i2f_small(a));
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

// Four int8 (one 32-bit word) -> two fp16x2, exactly: byte u = x ^ 0x80 under
// the fp16 exponent of 1024 is 1024 + u; subtracting 1152 leaves x.
__device__ __forceinline__ void i8x4_to_h2(uint32_t x, uint32_t& lo, uint32_t& hi) {
    x ^= 0x80808080u;
    const uint32_t a = __byte_perm(x, 0x64646464u, 0x4140);
    const uint32_t b = __byte_perm(x, 0x64646464u, 0x4342);
    asm("sub.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(a), "r"(0x64806480u));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(b), "r"(0x64806480u));
}

__device__ __forceinline__ uint32_t pack_h2(float lo_half, float hi_half) {
    const __half2 h = __floats2half2_rn(lo_half, hi_half);
    return *reinterpret_cast<const uint32_t*>(&h);
}
// Transpose of an 8 x 8 tile of 16-bit values held one row pair per thread
// (thread (g, t): row g, columns 2t, 2t + 1).
__device__ __forceinline__ uint32_t movm_trans(uint32_t x) {
    uint32_t y;
    asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
// x = hi + lo: hi keeps 11 significant bits (exact in fp16 for |x| >= 2^-14).
__device__ __forceinline__ float trunc11(float x) { return __int_as_float(__float_as_int(x) & (int)0xFFFFE000u); }

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// 2^k for |k| <= 126.
__device__ __forceinline__ float pow2i(int k) { return __int_as_float((127 + k) << 23); }
// Exponent e with x in [2^(e-1), 2^e), for finite x > 0.
__device__ __forceinline__ int exp_of(float x) { return ((__float_as_int(x) >> 23) & 0xFF) - 126; }

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

template <int NT, int NEX>
struct __align__(16) AttnSmem {
    int8_t qd[3][8 * NT][64];  // query digit planes [plane][row][dim] (B fragments of the score MMA)
    float fr[QR];            // per row: f = s * log2(e) / 8 (0 for padding rows)
    float s_self[QR];        // self-term score, raw units
    BlockBuf ex[NEX];        // the extra blocks
    int ex_lo[32 * NEX], ex_hi[32 * NEX];  // rows of the sequence that see each extra entry
    union {
        BlockBuf ring[NW][NSW];
        struct {
            float m[NW][QR], l[NW][QR];  // raw-unit maxima, sums
            float acc[NW][QR][ACC_STRIDE];  // true-scale weighted sums (padded rows: no bank conflicts)
        } merge;
    } u;
    float cm[QR], cl[QR];    // the CTA's merged state (with acc in u.merge.acc[0])
    int last;
};

}  // namespace

template <int NT, int NEX>
__global__ void __launch_bounds__(NT_THREADS, NT <= 3 ? 4 : 2) attn_decode_kernel(KvCache kv, int layer, RowBatch rb, const float* __restrict__ qkv,
                                                          int ld, int k_col, int v_col, int H, Staged st, SpecPool sp,
                                                          AttnWork aw, int nsplit, float* __restrict__ out, int ldo,
                                                          uint32_t* err) {
    extern __shared__ __align__(16) uint8_t attn_smem_raw[];
    AttnSmem<NT, NEX>& sm = *reinterpret_cast<AttnSmem<NT, NEX>*>(attn_smem_raw);
    constexpr int QP = 8 * NT;  // query rows padded to whole 8-row tiles
    const int b = blockIdx.x, g = blockIdx.y;
    const int split = (int)blockIdx.z % nsplit, rg = (int)blockIdx.z / nsplit;
    const int n = rb.n[b];
    const int qpk = H / kv.G;
    const int rpc = cta_query_rows(qpk) / qpk;  // sequence rows per CTA
    const int r0 = rg * rpc;       // this CTA's sequence rows [r0, r0 + nr)
    if (r0 >= n) {
        // (every CTA waits for the previous kernel, so that this grid's
        // completion implies that kernel's, for the kernels launched after it)
        asm volatile("griddepcontrol.wait;" ::: "memory");
        return;
    }
    const int nr = min(rpc, n - r0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, tig = lane & 3;
    const int rows = qpk * nr;  // <= QP (checked on the host)
    const int L0 = rb.len0[b], row0 = rb.row0[b];
    const int plast = L0 + n - 1;
    const int cs = min(L0, kv.S);
    const int nb0 = kv_pool_count(L0, kv.S, kv.Wr, kv.pb);
    const int npool = kv_pool_count(plast, kv.S, kv.Wr, kv.pb);
    const int qlo = max(kv.S, L0 - kv.Wr);
    const int nwin = max(0, L0 - qlo);
    const int s0 = (qlo - kv.S) % kv.Wr;  // ring slot of the oldest window position
    const size_t u = kv.unit(b, layer, g);
    const int n_spec = npool - nb0;
    // earlier rows of the batch: row r sees staged rows j < r, and this CTA's
    // last row is r0 + nr - 1
    const int n_ex = cs + n_spec + (r0 + nr - 1);
    if (n_ex > 32 * NEX || rows > QP) {  // excluded by the host; never index past the tiles
        if (tid == 0 && err) atomicOr(err, ERR_BOUNDS);
        asm volatile("griddepcontrol.wait;" ::: "memory");
        return;
    }
    const int pool_blocks = (nb0 + 31) / 32;
    const int ring_blocks = (nwin + 31) / 32;
    const int nkv = pool_blocks + ring_blocks;  // blocks that stream from memory
    const int nex = (n_ex + 31) / 32;
    const int nblk = nkv + nex;
    const int b_begin = (int)((int64_t)nblk * split / nsplit);
    const int b_end = (int)((int64_t)nblk * (split + 1) / nsplit);

    // ---- this warp's cp.async ring: block of iteration i is b_begin + warp + NW * i ----
    auto load_block = [&](int i, int slot) {
        const int blk = b_begin + warp + NW * i;
        if (blk >= b_end || blk >= nkv) return;
        BlockBuf& bb = sm.u.ring[warp][slot];
        const bool is_pool = blk < pool_blocks;
        const int bi = is_pool ? blk : blk - pool_blocks;
        const size_t e0 = (is_pool ? u * kv.P_pad : u * kv.W_pad) + (size_t)bi * 32;
        const int8_t* ksrc = (is_pool ? kv.pool_k : kv.ring_k) + e0 * 64;
        const int8_t* vsrc = (is_pool ? kv.pool_v : kv.ring_v) + e0 * 64;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            cp16(&bb.k[0][0] + (lane + 32 * c) * 16, ksrc + (lane + 32 * c) * 16);
            cp16(bb.v + (lane + 32 * c) * 16, vsrc + (lane + 32 * c) * 16);
        }
        if (lane < 8)
            cp16(bb.ks + lane * 4, (is_pool ? kv.pool_ks : kv.ring_ks) + e0 + lane * 4);
        else if (lane < 16)
            cp16(bb.vs + (lane - 8) * 4, (is_pool ? kv.pool_vs : kv.ring_vs) + e0 + (lane - 8) * 4);
    };
#pragma unroll
    for (int i = 0; i < NSW - 1; i++) {
        load_block(i, i);
        cp_commit();
    }
    // The committed cache streamed above was written by earlier steps; the
    // queries, staged rows and in-batch pool entries below come from the
    // kernels just before this one (programmatic dependent launch).
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // ---- the extra block: sink entries, pool entries finalized inside the
    // batch (visible from the row that finalizes them), staged earlier rows.
    // Its loads, and the query rows' below, are all issued before first use. ----
    auto ex_src = [&](int e, const int8_t*& kp, const int8_t*& vp, const float*& ksp, const float*& vsp, int& lo) {
        if (e < cs) {
            const size_t o = u * kv.S + e;
            kp = kv.sink_k + o * 64;
            vp = kv.sink_v + o * 64;
            ksp = kv.sink_ks + o;
            vsp = kv.sink_vs + o;
            lo = 0;
        } else if (e < cs + n_spec) {
            const int j = nb0 + (e - cs);
            const size_t o = ((size_t)b * kv.G + g) * sp.per + (j - nb0);
            kp = sp.k + o * 64;
            vp = sp.v + o * 64;
            ksp = sp.ks + o;
            vsp = sp.vs + o;
            lo = kv.S + kv.Wr + (j + 1) * kv.pb - L0;
        } else {
            const int j = e - cs - n_spec;
            const size_t o = (size_t)(row0 + j) * kv.G + g;
            kp = st.k + o * 64;
            vp = st.v + o * 64;
            ksp = st.ks + o;
            vsp = st.vs + o;
            lo = j + 1;
        }
    };
    // this split owns some extra block: it assembles all of them
    const bool own_ex = nex > 0 && b_end > nkv && b_begin < nblk;
    // task t (< nex * 128, strided over the CTA's threads): entry t >> 2,
    // dims [16*(t&3), +16)
    constexpr int EXT = (128 * NEX + NT_THREADS - 1) / NT_THREADS;  // tasks per thread
    uint4 ex_k[EXT], ex_v[EXT];
    float ex_ks[EXT], ex_vs[EXT];
    int ex_lo[EXT];
#pragma unroll
    for (int x = 0; x < EXT; x++) {
        const int task = tid + NT_THREADS * x;
        const int e = task >> 2, q4 = task & 3;
        ex_k[x] = make_uint4(0, 0, 0, 0);
        ex_v[x] = make_uint4(0, 0, 0, 0);
        ex_ks[x] = 0.0f;
        ex_vs[x] = 0.0f;
        ex_lo[x] = BIG;
        if (own_ex && task < 128 * NEX && e < n_ex) {
            const int8_t *kp, *vp;
            const float *ksp, *vsp;
            ex_src(e, kp, vp, ksp, vsp, ex_lo[x]);
            ex_k[x] = *reinterpret_cast<const uint4*>(kp + 16 * q4);
            ex_v[x] = *reinterpret_cast<const uint4*>(vp + 16 * q4);
            ex_ks[x] = *ksp;
            ex_vs[x] = *vsp;
        }
    }

    // ---- queries -> int8 digit planes; self-term score ----
    constexpr int RPW = (QP + NW - 1) / NW;  // query rows per warp: warp + NW * k (< QP)
    float qx[RPW][2], kx[RPW][2];
#pragma unroll
    for (int k = 0; k < RPW; k++) {
        const int ri = warp + NW * k;
        const bool in = ri < rows;
        const int hh = in ? ri / nr : 0, r = in ? r0 + ri % nr : 0;
        const float* row = qkv + (size_t)(row0 + r) * ld;
        const float* q = row + (size_t)(g + hh * kv.G) * 64;
        qx[k][0] = in ? q[lane] : 0.0f;
        qx[k][1] = in ? q[lane + 32] : 0.0f;
        kx[k][0] = in ? row[k_col + g * 64 + lane] : 0.0f;
        kx[k][1] = in ? row[k_col + g * 64 + lane + 32] : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < RPW; k++) {
        const int ri = warp + NW * k;
        if (ri >= QP) break;  // (warp-uniform)
        const float x0 = qx[k][0], x1 = qx[k][1];
        const float amax = warp_max(fmaxf(fabsf(x0), fabsf(x1)));
        const bool fin = amax <= 3.0e38f;  // inf / NaN query: every score NaN, as in the reference
        const float mul = (amax == 0.0f || !fin) ? 0.0f : 127.0f / amax;
        const float f = !fin ? __int_as_float(0x7fc00000) : (amax / 127.0f) * (0.125f * kLog2e);
        int a1, a2, a3, b1, b2, b3;
        digits3(x0, mul, a1, a2, a3);
        digits3(x1, mul, b1, b2, b3);
        // planes in natural dim order: the score MMA's B fragment of thread
        // (g, t) is bytes [16t, 16t + 16) of row g of an 8-row tile
        sm.qd[0][ri][lane] = (int8_t)a1;
        sm.qd[1][ri][lane] = (int8_t)a2;
        sm.qd[2][ri][lane] = (int8_t)a3;
        sm.qd[0][ri][lane + 32] = (int8_t)b1;
        sm.qd[1][ri][lane + 32] = (int8_t)b2;
        sm.qd[2][ri][lane + 32] = (int8_t)b3;
        // self term with the float k and v (src/engine.cpp:760-778), in raw
        // units: (q . k) / sqrt(64) / (s / sqrt(64))
        const float sc = warp_sum(x0 * kx[k][0] + x1 * kx[k][1]) * mul;
        if (lane == 0) {
            sm.fr[ri] = f;
            sm.s_self[ri] = sc;
        }
    }

    if (own_ex) {
#pragma unroll
        for (int x = 0; x < EXT; x++) {
            const int task = tid + NT_THREADS * x;
            const int e = task >> 2, q4 = task & 3;
            if (task >= 128 * NEX || e >= 32 * nex) break;
            BlockBuf& xb = sm.ex[e >> 5];
            const int el = e & 31;
            *reinterpret_cast<uint4*>(&xb.k[el][16 * q4]) = ex_k[x];
            const uint8_t* vb = reinterpret_cast<const uint8_t*>(&ex_v[x]);
            const int pos = kv_vpos(el);
#pragma unroll
            for (int i = 0; i < 16; i++) xb.v[(16 * q4 + i) * 32 + pos] = (int8_t)vb[i];
            if (q4 == 0) {
                xb.ks[el] = ex_ks[x];
                xb.vs[el] = ex_vs[x];
                sm.ex_lo[e] = ex_lo[x];
                sm.ex_hi[e] = e < n_ex ? BIG : -1;
            }
        }
    }
    __syncthreads();

    // ---- per-thread rows: thread (g, t) holds query rows 8 nt + 2t + c of every
    // tile nt (c = 0, 1) and entries 8 j + g (j = 0..3) of each block ----
    float fr[NT][2], mref[NT][2], lsum[NT][2];
    int rr[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int c = 0; c < 2; c++) {
            const int ri = nt * 8 + 2 * tig + c;
            fr[nt][c] = sm.fr[ri];
            rr[nt][c] = ri < rows ? r0 + ri % nr : -1;  // padding row: every entry has lo >= 0
            mref[nt][c] = -INFINITY;
            lsum[nt][c] = 0.0f;  // this thread's entries only (summed over g at the end)
        }
    float acc[4][NT][4];  // O^T: dims 16 dt + gid (+8 for c >= 2), rows 8 nt + 2 tig + (c & 1)
#pragma unroll
    for (int dt = 0; dt < 4; dt++)
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int c = 0; c < 4; c++) acc[dt][nt][c] = 0.0f;
    int eref = 0;
    bool have_ref = false;

    int slot = 0;  // ring slot of block i (i % NSW)
    for (int i = 0;; i++) {
        const int blk = b_begin + warp + NW * i;
        if (blk >= b_end) break;
        cp_wait<NSW - 2>();
        __syncwarp();  // every lane's copies of block i landed; slot (i - 1) % NSW is free
        load_block(i + NSW - 1, slot == 0 ? NSW - 1 : slot - 1);
        cp_commit();
        const bool is_ex = blk >= nkv;
        const BlockBuf& bb = is_ex ? sm.ex[blk - nkv] : sm.u.ring[warp][slot];
        slot = (slot + 1 == NSW) ? 0 : slot + 1;

        // ---- visibility of entry `lane`: query rows [lo, hi] of the sequence ----
        int lo = BIG, hi = -1;
        if (is_ex) {
            lo = sm.ex_lo[(blk - nkv) * 32 + lane];
            hi = sm.ex_hi[(blk - nkv) * 32 + lane];
        } else if (blk < pool_blocks) {
            if (blk * 32 + lane < nb0) lo = 0, hi = BIG;
        } else {
            const int slot = (blk - pool_blocks) * 32 + lane;
            if (slot < kv.Wr) {
                const int off = slot >= s0 ? slot - s0 : slot - s0 + kv.Wr;  // (slot - s0) mod Wr
                if (off < nwin) lo = 0, hi = qlo + off + kv.Wr - L0;
            }
        }
        const bool valid = hi >= 0 && lo < BIG;
        const bool full = __all_sync(0xffffffffu, valid && lo <= r0 && hi >= r0 + nr - 1);  // every row of this CTA

        // ---- v-scale reference: a power of two per warp, raised when a block's
        // scales outgrow it (the accumulators are rescaled exactly) ----
        const float vl = valid ? bb.vs[lane] : 0.0f;
        // (a warp-wide maximum only for the first block and when some scale
        // leaves the range of the reference)
        if (__any_sync(0xffffffffu, have_ref ? !(vl < pow2i(min(126, eref + 4))) : vl > 0.0f)) {
            const float vmax = warp_max(vl);
            const int ev = (vmax > 0.0f && vmax <= 3.0e38f) ? exp_of(vmax) : (have_ref ? eref : 0);
            if (!have_ref) {
                eref = ev;
                have_ref = vmax > 0.0f && vmax <= 3.0e38f;
            } else if (ev > eref + 4) {
                const float c = pow2i(max(eref - ev, -126));
#pragma unroll
                for (int dt = 0; dt < 4; dt++)
#pragma unroll
                    for (int nt = 0; nt < NT; nt++)
#pragma unroll
                        for (int c4 = 0; c4 < 4; c4++) acc[dt][nt][c4] *= c;
                eref = ev;
            }
        }
        const float vmul = pow2i(-max(-126, min(126, eref)));

        // The rest of the block's work, specialised for blocks whose entries
        // every row sees (no masks) and for the others.
        auto body = [&](auto full_tag) {
            constexpr bool FULL = decltype(full_tag)::value;
            // ---- this thread's entries e = 8 j + gid: scales (and masks) ----
            float ksv[4], vsn[4];
            int lo4[4], hi4[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                ksv[j] = bb.ks[8 * j + gid];
                vsn[j] = bb.vs[8 * j + gid] * vmul;
                if (!FULL) {
                    lo4[j] = __shfl_sync(0xffffffffu, lo, 8 * j + gid);
                    hi4[j] = __shfl_sync(0xffffffffu, hi, 8 * j + gid);
                    if (!(hi4[j] >= 0 && lo4[j] < BIG)) vsn[j] = 0.0f;  // a masked entry must not bring a NaN scale in
                }
            }

            // ---- scores S^T = K . Q^T (three digit planes, exact int32), s_raw = S * k_scale ----
            // Per 16-entry m-tile: its A fragments (both k-steps) are K rows gid,
            // gid + 8, bytes [16 tig, 16 tig + 16); the B fragments of row
            // tile nt and plane p are bytes [16 tig, 16 tig + 16) of query row
            // 8 nt + gid.
            float s[2][NT][4];  // [m-tile][row tile][c]: entry 16 mt + gid + 8 (c >> 1), row 8 nt + 2 tig + (c & 1)
#pragma unroll
            for (int mt = 0; mt < 2; mt++) {
                const uint4 ka = *reinterpret_cast<const uint4*>(&bb.k[16 * mt + gid][16 * tig]);
                const uint4 kb = *reinterpret_cast<const uint4*>(&bb.k[16 * mt + gid + 8][16 * tig]);
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    int32_t ac[3][4];
#pragma unroll
                    for (int p = 0; p < 3; p++) {
                        const uint4 qb = *reinterpret_cast<const uint4*>(&sm.qd[p][8 * nt + gid][16 * tig]);
                        ac[p][0] = ac[p][1] = ac[p][2] = ac[p][3] = 0;
                        mma_s8(ac[p], ka.x, kb.x, ka.y, kb.y, qb.x, qb.y);
                        mma_s8(ac[p], ka.z, kb.z, ka.w, kb.w, qb.z, qb.w);
                    }
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        const int j = 2 * mt + (c >> 1);
                        float v = comb(ac[0][c], ac[1][c], ac[2][c]) * ksv[j];
                        if (!FULL) {
                            const int r = rr[nt][c & 1];
                            if (!(r >= lo4[j] && r <= hi4[j])) v = -INFINITY;
                        }
                        s[mt][nt][c] = v;
                    }
                }
            }

            // ---- online softmax with a lazily raised reference maximum: this
            // thread's entries decide whether any row's maximum must move ----
            float bmax[NT][2];
            bool need = false;
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const float bm = fmaxf(fmaxf(s[0][nt][c], s[0][nt][c + 2]), fmaxf(s[1][nt][c], s[1][nt][c + 2]));
                    bmax[nt][c] = bm;
                    const float m = mref[nt][c];
                    need |= (bm > -INFINITY) && (m == -INFINITY || (bm - m) * fr[nt][c] > kMaxLead);
                }
            if (__any_sync(0xffffffffu, need)) {
#pragma unroll
                for (int nt = 0; nt < NT; nt++)
#pragma unroll
                    for (int c = 0; c < 2; c++) {
                        float bm = bmax[nt][c];  // the block's maximum of the row: over gid
                        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 4));
                        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 8));
                        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 16));
                        const float m = mref[nt][c];
                        const float mn = fmaxf(m, bm);
                        if (mn > m) {
                            const float corr = (m == -INFINITY) ? 0.0f : ex2((m - mn) * fr[nt][c]);
                            lsum[nt][c] *= corr;
#pragma unroll
                            for (int dt = 0; dt < 4; dt++) {
                                acc[dt][nt][c] *= corr;
                                acc[dt][nt][c + 2] *= corr;
                            }
                            mref[nt][c] = mn;
                        }
                    }
            }
            // p = 2^((s_raw - m) f), w = p * v_scale / 2^E -> two fp16 planes.
            // The pair (rows 2 tig, 2 tig + 1) of entry e is row e of an 8 x 8
            // fp16 tile (entries x rows); movmatrix.trans turns it into the
            // P.V MMA's B fragment (entries 2 tig, 2 tig + 1 of row gid).
            uint32_t wb[2][NT][2][2];  // [k-step = m-tile][row tile][entry half][plane: 0 hi, 1 lo]
#pragma unroll
            for (int mt = 0; mt < 2; mt++)
#pragma unroll
                for (int nt = 0; nt < NT; nt++)
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        float w[2];
#pragma unroll
                        for (int c = 0; c < 2; c++) {
                            const float sv = s[mt][nt][2 * h + c];
                            // every entry of a FULL block is visible and finite
                            const float p = (!FULL && sv == -INFINITY) ? 0.0f : ex2((sv - mref[nt][c]) * fr[nt][c]);
                            lsum[nt][c] += p;
                            w[c] = p * vsn[2 * mt + h];
                        }
                        const float h0 = trunc11(w[0]), h1 = trunc11(w[1]);
                        wb[mt][nt][h][0] = movm_trans(pack_h2(h0, h1));
                        wb[mt][nt][h][1] = movm_trans(pack_h2(w[0] - h0, w[1] - h1));
                    }

            // ---- O^T += V^T . W^T: A = V^T (dims x entries), exact in fp16 ----
#pragma unroll
            for (int dt = 0; dt < 4; dt++) {
                const uint2 va = *reinterpret_cast<const uint2*>(&bb.v[(16 * dt + gid) * 32 + 8 * tig]);
                const uint2 vb = *reinterpret_cast<const uint2*>(&bb.v[(16 * dt + gid + 8) * 32 + 8 * tig]);
                uint32_t a[2][4];  // [k-step][reg]: entries 16 ks + {2t, 2t+1} (a0 a1), + 8 (a2 a3)
                i8x4_to_h2(va.x, a[0][0], a[0][2]);
                i8x4_to_h2(vb.x, a[0][1], a[0][3]);
                i8x4_to_h2(va.y, a[1][0], a[1][2]);
                i8x4_to_h2(vb.y, a[1][1], a[1][3]);
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                    for (int pl = 1; pl >= 0; pl--)  // the remainder plane first
#pragma unroll
                        for (int ks = 0; ks < 2; ks++)
                            mma_f16(o, a[ks][0], a[ks][1], a[ks][2], a[ks][3], wb[ks][nt][0][pl], wb[ks][nt][1][pl]);
#pragma unroll
                    for (int c = 0; c < 4; c++) acc[dt][nt][c] += o[c];
                }
            }
        };
        if (full)
            body(std::true_type{});
        else
            body(std::false_type{});
    }
    cp_wait<0>();
    __syncthreads();  // every warp left its ring: the ring area becomes the merge area

    // ---- warp states -> shared memory (raw-unit maxima, true-scale sums) ----
    {
        const float vs_scale = pow2i(max(-126, min(126, eref)));
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int c = 0; c < 2; c++) {
                const int r = nt * 8 + 2 * tig + c;
                float l = lsum[nt][c];  // over the block entries of every gid
                l += __shfl_xor_sync(0xffffffffu, l, 4);
                l += __shfl_xor_sync(0xffffffffu, l, 8);
                l += __shfl_xor_sync(0xffffffffu, l, 16);
                if (gid == 0) {
                    sm.u.merge.m[warp][r] = mref[nt][c];
                    sm.u.merge.l[warp][r] = l;
                }
#pragma unroll
                for (int dt = 0; dt < 4; dt++) {
                    sm.u.merge.acc[warp][r][16 * dt + gid] = acc[dt][nt][c] * vs_scale;
                    sm.u.merge.acc[warp][r][16 * dt + gid + 8] = acc[dt][nt][c + 2] * vs_scale;
                }
            }
    }
    __syncthreads();

    // ---- merge the warps: the CTA's state per row into cm / cl / acc[0] ----
    for (int ri = warp; ri < rows; ri += NW) {
        const float fq = sm.fr[ri];
        float m = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; w++) m = fmaxf(m, sm.u.merge.m[w][ri]);
        float l = 0.0f, o0 = 0.0f, o1 = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; w++) {
            const float mw = sm.u.merge.m[w][ri];
            const float f = (mw == -INFINITY) ? 0.0f : ex2((mw - m) * fq);
            l += sm.u.merge.l[w][ri] * f;
            o0 += sm.u.merge.acc[w][ri][lane] * f;
            o1 += sm.u.merge.acc[w][ri][lane + 32] * f;
        }
        __syncwarp();
        if (lane == 0) {
            sm.cm[ri] = m;
            sm.cl[ri] = l;
        }
        sm.u.merge.acc[0][ri][lane] = o0;  // this warp alone reads and writes row ri
        sm.u.merge.acc[0][ri][lane + 32] = o1;
    }

    // ---- more than one split: publish, and let the last split merge ----
    const size_t item = ((size_t)b * kv.G + g) * (gridDim.z / nsplit) + rg;  // (sequence, kv head, row group)
    if (nsplit > 1) {
        float* part = aw.part + (item * nsplit + split) * QR * PART;
        for (int ri = warp; ri < rows; ri += NW) {
            float* pr = part + (size_t)ri * PART;
            if (lane == 0) {
                pr[0] = sm.cm[ri];
                pr[1] = sm.cl[ri];
            }
            pr[4 + lane] = sm.u.merge.acc[0][ri][lane];
            pr[4 + lane + 32] = sm.u.merge.acc[0][ri][lane + 32];
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const int prev = atomicAdd(aw.cnt + item, 1);
            sm.last = prev == nsplit - 1;
            if (sm.last) aw.cnt[item] = 0;  // ready for the next launch
        }
        __syncthreads();
        if (!sm.last) return;
        __threadfence();
    }

    // ---- final: all splits' states + the self term -> output rows ----
    __syncwarp();  // (one split) this warp's rows of cm / cl / acc[0] are written
    for (int ri = warp; ri < rows; ri += NW) {
        const int hh = ri / nr, r = r0 + ri % nr;
        const int h = g + hh * kv.G;
        const float ss = sm.s_self[ri], fq = sm.fr[ri];
        float m = ss, l, o0, o1;
        if (nsplit == 1) {
            const float mc = sm.cm[ri];
            m = fmaxf(m, mc);
            const float f = (mc == -INFINITY) ? 0.0f : ex2((mc - m) * fq);
            l = sm.cl[ri] * f;
            o0 = sm.u.merge.acc[0][ri][lane] * f;
            o1 = sm.u.merge.acc[0][ri][lane + 32] * f;
        } else {
            // every split's state of the row is loaded before any is used
            const float* part = aw.part + item * nsplit * QR * PART + (size_t)ri * PART;
            float mc[kMaxSplits], lc[kMaxSplits], oa[kMaxSplits], ob[kMaxSplits];
#pragma unroll
            for (int sp2 = 0; sp2 < kMaxSplits; sp2++) {
                mc[sp2] = -INFINITY;
                lc[sp2] = oa[sp2] = ob[sp2] = 0.0f;
                if (sp2 < nsplit) {
                    const float* pr = part + (size_t)sp2 * QR * PART;
                    mc[sp2] = __ldcg(pr);
                    lc[sp2] = __ldcg(pr + 1);
                    oa[sp2] = __ldcg(pr + 4 + lane);
                    ob[sp2] = __ldcg(pr + 4 + lane + 32);
                }
            }
#pragma unroll
            for (int sp2 = 0; sp2 < kMaxSplits; sp2++) m = fmaxf(m, mc[sp2]);
            l = 0.0f, o0 = 0.0f, o1 = 0.0f;
#pragma unroll
            for (int sp2 = 0; sp2 < kMaxSplits; sp2++) {
                const float f = (mc[sp2] == -INFINITY) ? 0.0f : ex2((mc[sp2] - m) * fq);
                l += lc[sp2] * f;
                o0 += oa[sp2] * f;
                o1 += ob[sp2] * f;
            }
        }
        const float ps = ex2((ss - m) * fq);
        l += ps;
        const float* vrow = qkv + (size_t)(row0 + r) * ld + v_col + g * 64;  // the row's own float v
        o0 += ps * vrow[lane];
        o1 += ps * vrow[lane + 32];
        const float inv = 1.0f / (l + 1e-10f);
        const int row = row0 + r;
        out[(size_t)row * ldo + (size_t)h * 64 + lane] = o0 * inv;
        out[(size_t)row * ldo + (size_t)h * 64 + lane + 32] = o1 * inv;
    }
}

bool attention_decode_supported(const KvCache& kv, int H, int max_rows) {
    const int spec = max_rows > 1 ? ceil_div(max_rows - 1, kv.pb) + 1 : 1;  // pool entries a batch can finalize
    return H / kv.G <= QR && kv.S + spec + max_rows - 1 <= 32 * NEXMAX;
}

// Sequence rows per CTA and row groups per (sequence, kv head).
static int attn_rows_per_cta(const KvCache& kv, int H) { return cta_query_rows(H / kv.G) / (H / kv.G); }
int attention_decode_rows_per_cta(const KvCache& kv, int H) { return attn_rows_per_cta(kv, H); }
int attention_decode_row_groups(const KvCache& kv, int H, int max_rows) {
    return ceil_div(std::max(1, max_rows), attn_rows_per_cta(kv, H));
}

int attention_decode_splits(int nb, int G, int max_splits) {
    // Split only while the (sequence, kv head) items leave CTA slots (four per
    // SM) empty: each split repeats the query setup and adds a merge.
    const int items = std::max(1, nb * G);
    return std::max(1, std::min(max_splits, (4 * 148) / items));
}

size_t attention_decode_work_floats(int nb, int G, int nsplit, int nrg) {
    return (size_t)nb * G * nrg * nsplit * QR * PART;
}

template <int NT, int NEX>
static pf_status launch_decode(const KvCache& kv, int layer, const RowBatch& rb, const float* qkv, int ldqkv, int k_col,
                               int v_col, int H, Staged st, SpecPool sp, const AttnWork& aw, float* out, int ldo,
                               cudaStream_t stream) {
    const int smem = (int)sizeof(AttnSmem<NT, NEX>);
    static std::atomic<uint64_t> attr{0};
    PF_TRY(raise_smem_limit(attn_decode_kernel<NT, NEX>, smem, attr));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rb.nb, kv.G, aw.nsplit * attention_decode_row_groups(kv, H, rb.max_rows));
    cfg.blockDim = dim3(NT_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    PF_CUDA(cudaLaunchKernelEx(&cfg, attn_decode_kernel<NT, NEX>, kv, layer, rb, qkv, ldqkv, k_col, v_col, H, st, sp, aw,
                               aw.nsplit, out, ldo, device_error_flag()));
    return launch_check("attention_decode");
}

pf_status attention_decode(const KvCache& kv, int layer, const RowBatch& rb, const float* qkv, int ldqkv, int k_col,
                           int v_col, int H, Staged st, SpecPool sp, const AttnWork& aw, float* out, int ldo,
                           cudaStream_t stream) {
    PF_CHECK(kv.hd == 64, "attention_decode: head_dim must be 64");
    PF_CHECK(attention_decode_supported(kv, H, rb.max_rows), "attention_decode: too many query rows");
    const int nrg = attention_decode_row_groups(kv, H, rb.max_rows);
    PF_CHECK(aw.nsplit >= 1 && aw.nsplit <= kMaxSplits && aw.nsplit * nrg <= 65535,
             "attention_decode: %d context splits (1..%d)", aw.nsplit, kMaxSplits);
    PF_CHECK(aw.nsplit == 1 ||
                 (aw.part && aw.cnt && aw.part_floats >= attention_decode_work_floats(rb.nb, kv.G, aw.nsplit, nrg) &&
                  aw.cnt_elems >= (size_t)rb.nb * kv.G * nrg),
             "attention_decode: workspace too small for %d splits", aw.nsplit);
    // one extra block for verify batches, up to NEXMAX for prefill chunks
    const int spec = rb.max_rows > 1 ? ceil_div(rb.max_rows - 1, kv.pb) + 1 : 1;
    const bool one_ex = kv.S + spec + rb.max_rows - 1 <= 32;
    // query rows of a CTA in 8-row tiles (the N of the score MMA)
    const int nt = ceil_div((H / kv.G) * std::min(rb.max_rows, attn_rows_per_cta(kv, H)), 8);
#define PF_ATTN_LAUNCH(NT_, NEX_) \
    launch_decode<NT_, NEX_>(kv, layer, rb, qkv, ldqkv, k_col, v_col, H, st, sp, aw, out, ldo, stream)
    if (one_ex) {
        switch (nt) {
            case 1: return PF_ATTN_LAUNCH(1, 1);
            case 2: return PF_ATTN_LAUNCH(2, 1);
            case 3: return PF_ATTN_LAUNCH(3, 1);
            default: return PF_ATTN_LAUNCH(4, 1);
        }
    }
    switch (nt) {
        case 1: return PF_ATTN_LAUNCH(1, NEXMAX);
        case 2: return PF_ATTN_LAUNCH(2, NEXMAX);
        case 3: return PF_ATTN_LAUNCH(3, NEXMAX);
        default: return PF_ATTN_LAUNCH(4, NEXMAX);
    }
#undef PF_ATTN_LAUNCH
}

}  // namespace pf

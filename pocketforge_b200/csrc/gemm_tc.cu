// gemm_tc.cu — the projection GEMM on the 5th-generation tensor cores:
// int8 activations x packed Q4 / Q2 / int8 weights -> int32 in TMEM
// (tcgen05.mma.kind::i8), with the epilogues of gemm.cuh.
//
// One CTA computes a 128-row x BN-column output tile (BN = 64, 128 or 256;
// optionally one split of K), or TM = 2 such tiles stacked in M that share
// every unpacked weight stage (prefill-sized SwiGLU launches).  Per 128-wide
// K stage:
//   warp 0: lane s*(P+1)+c issues copy c of every stage that uses load slot
//     s — the activation tile of digit plane c (128 x 128 B, 128-byte
//     swizzle) or, for c == P, the packed weight block (BN rows x RB bytes)
//     — and arrives with its byte count on full_raw[s];
//   warps 2..9: unpack the weight block into unpacked-weight buffer b
//     (= stage % 2) in the tensor core's K-major 128-byte-swizzled layout
//     (the layout the TMA produces for the activations), each weight in the
//     top bits of its byte; fence the generic->async proxy; one arrival per
//     warp on b_full[b] (256 single-thread arrivals on one barrier word
//     serialised the hand-off);
//   warp 1, one thread: four tcgen05.mma (K = 32 each) per activation plane
//     into TMEM, then tcgen05.commit -> empty[s] and b_empty[b].
// The K loop is bound by shared-memory bandwidth: per stage the TMA writes,
// the unpack's loads and stores and the tensor core's operand reads (at
// BN = 256, 128 KB, ~0.5 us at 128 B per clock).  Loading the packed weights
// into registers instead of through the TMA saved nothing (global loads fill
// the same on-chip array) and lengthened the K loop.  The load ring has more
// slots than the two unpacked buffers, so more copies are in flight per
// shared-memory byte.
// After the last stage a commit on `done` releases warps 2..9 to read the
// accumulators (tcgen05.ld 32x32b: warp w reads TMEM lanes 32*(w%4)..+31,
// i.e. output rows, and one half of the columns), shift the sums back to the
// weights' scale, and run the epilogue through a shared staging tile so that
// every global store is a whole-row run.  Split-K partial sums go to an int32
// workspace laid out [plane][n][m]; the CTA that retires a tile last applies
// the epilogue and re-zeroes the workspace.  Every TMA load fills only this
// CTA's own shared memory.
//
// Under programmatic dependent launch the weight copies start before the
// previous kernel has finished; the activation copies and the epilogue wait
// for it (griddepcontrol.wait).
//
// Every mbarrier wait is bounded (about one second of spinning); a timeout
// latches ERR_TIMEOUT in the device error flag and the CTA drains and frees
// its TMEM instead of hanging.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "gemm.cuh"
#include "gemm_tc.cuh"
#include "numerics.cuh"

namespace pf {

namespace {

constexpr int BM = 128, BK = 128;
constexpr int NUM_UNPACK = 256;                 // warps 2..9: weight unpack, then epilogue
constexpr int NUM_THREADS = 64 + NUM_UNPACK;  // + warp 0 (TMA) and warp 1 (MMA)
constexpr uint32_t ERR_TIMEOUT = 16u;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait: false when ~1 s passed without the phase completing.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 0;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 1023u) == 1023u && globaltimer() - t0 > 1000000000ull) return false;
    }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    // K-major, 128-byte swizzle: 8-row groups 1024 B apart (SBO), LBO unused,
    // version 1 (sm_100), layout type 2 (SWIZZLE_128B).
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}
__host__ __device__ constexpr uint32_t idesc_i8(int n) {
    // D s32 (2 << 4), A s8 (1 << 7), B s8 (1 << 10), K-major A and B,
    // N >> 3 at bit 17, M >> 4 at bit 24 (M = 128).
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// 16 columns of this warp's 32 TMEM lanes; the registers are valid only
// after tmem_wait_ld().
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    tmem_ld16_nowait(taddr, r);
    tmem_wait_ld();
}
// The tensor maps live in kernel parameter space; fetching them ahead of the
// first copy takes the descriptor fetch off that copy's latency.
__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Barrier of the epilogue warps only (named barrier 1).
__device__ __forceinline__ void named_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NUM_UNPACK) : "memory"); }

// Packed bytes per (row, 128-wide K block) of each format.
template <int WF>
__host__ __device__ constexpr int row_bytes() {
    return WF == WF_Q4 ? 64 : (WF == WF_Q2 ? 32 : 128);
}

template <int BN, int P, int WF, int TM = 1>
struct Layout {
    static constexpr int A_BYTES = BM * BK;             // one plane of one 128-row M tile
    static constexpr int RAW_BYTES = BN * row_bytes<WF>();
    static constexpr int B_BYTES = BN * BK;
    // Load ring: STAGES slots of activation planes + packed weights (what the
    // TMA has in flight); the unpacked weights get NB buffers of their own,
    // so the ring can be deeper than the unpack -> MMA hand-off needs.
    static constexpr int SLOT_BYTES = TM * P * A_BYTES + ((RAW_BYTES + 1023) / 1024) * 1024;
    static constexpr int NB = 2;
    static constexpr int STAGES_MAX = (P * TM == 1) ? 8 : 4;
    static constexpr int BUDGET = 220 * 1024;
    static constexpr int FIT = (BUDGET - NB * B_BYTES) / SLOT_BYTES;
    static constexpr int STAGES = STAGES_MAX < FIT ? STAGES_MAX : FIT;
    static constexpr int B_OFF = STAGES * SLOT_BYTES;
    static constexpr int BAR_OFF = B_OFF + NB * B_BYTES;
    static constexpr int WSC_OFF = BAR_OFF + 256;        // BN column scales (fp32)
    static constexpr int SMEM = WSC_OFF + BN * 4 + 1024;  // + alignment slack
    // Epilogue staging (reuses the rings): 8 warps x 32 rows x (BN/2 + 4) fp32.
    static constexpr int SROW = BN / 2 + 4;
    static_assert(8 * 32 * SROW * 4 <= BAR_OFF, "staging does not fit the rings");
    static constexpr int TMEM_COLS = (TM * P * BN <= 32) ? 32 : (TM * P * BN <= 64) ? 64
                                    : (TM * P * BN <= 128) ? 128 : (TM * P * BN <= 256) ? 256 : 512;
    static_assert(TM * P * BN <= 512, "accumulators exceed TMEM");
};

template <int P>
__device__ __forceinline__ float comb3(const int32_t (&a)[P]) {
    if constexpr (P == 3) {
        const float r = 1.0f / 254.0f;
        return __fadd_rn(__int2float_rn(a[0]),
                         __fmul_rn(__fadd_rn(__int2float_rn(a[1]), __fmul_rn(__int2float_rn(a[2]), r)), r));
    } else {
        return __int2float_rn(a[0]);
    }
}
// Value of one output column of row m before the column-pair step:
// v = ((float)acc * a_scale[m]) * w_scale[n] (matmul_quantized's two
// roundings, src/matmul_neon.cpp:176-180), comb * (a_scale[m] * w_scale_all)
// for the tied unembedding, comb * a_scale[m] * w_scale[n] for the MTP forms,
// or the raw int32 bits for EPI_I32.
template <int P, int EPI>
__device__ __forceinline__ float col_value(const int32_t (&a)[P], float a_s, float w_s, float s_all) {
    if constexpr (EPI == EPI_I32) {
        return __int_as_float(a[0]);
    } else if constexpr (EPI == EPI_LOGITS3) {
        return __fmul_rn(comb3<P>(a), s_all);
    } else if constexpr (EPI == EPI_MTP_SWIGLU3 || EPI == EPI_MTP_RESID3) {
        // scales first: a_s * w_s stays finite where comb * a_s may not
        return __fmul_rn(comb3<P>(a), __fmul_rn(a_s, w_s));
    } else {
        return __fmul_rn(__fmul_rn(__int2float_rn(a[0]), a_s), w_s);
    }
}

__device__ __forceinline__ float engine_swiglu(float g, float u) { return engine_swiglu_rn(g, u); }  // engine FFN form
__device__ __forceinline__ float mtp_swiglu(float g, float u) {  // MTP head FFN form
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}
__device__ __forceinline__ void rope_pair(float& x0, float& x1, float c, float s) {
    // adjacent-pair rotation (src/engine.cpp:737-748)
    const float r0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    const float r1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    x0 = r0;
    x1 = r1;
}

// Pass 2 of the epilogue: one warp writes its 32 staged rows of BN values
// (row stride SROW floats).  Lane l owns columns 4*(l % CPR) .. +3 of row
// l / CPR of each group, so every store (and every residual load) is a
// contiguous run of a row.  Row-dependent inputs (residual rows, RoPE angles)
// are fetched for U groups before any of them is written, keeping several
// loads in flight.  The SwiGLU forms stage their outputs (pass 1 applies the
// activation), so for them BN counts output columns and n0 is an output
// column.
template <int BN, int SROW, int EPI>
__device__ __forceinline__ void store_rows(const GemmParams& p, const float* stg, int rbase, int n0, int lane,
                                           int32_t* out_i32) {
    constexpr int CPR = BN / 4, RPI = 32 / CPR, ITERS = 32 / RPI, U = 4;
    static_assert(ITERS % U == 0, "row groups");
    const int cg = lane % CPR, ro = lane / CPR;
    const int n = n0 + 4 * cg;
    const int m_act = p.m_dev ? min(p.M, *p.m_dev) : p.M;
    constexpr bool RESID = EPI == EPI_RESID || EPI == EPI_MTP_RESID3;
    for (int g0 = 0; g0 < ITERS; g0 += U) {
        int rr[U];
        bool act[U];
        float4 pre[U];  // residual row segment, or (cos0, sin0, cos1, sin1)
#pragma unroll
        for (int u = 0; u < U; u++) {
            rr[u] = (g0 + u) * RPI + ro;
            const int m = rbase + rr[u];
            act[u] = m < m_act;
            if constexpr (EPI == EPI_RESID) act[u] = act[u] && !(p.row_skip && p.row_skip[m]);
            pre[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (!act[u]) continue;
            if constexpr (RESID) {
                pre[u] = *reinterpret_cast<const float4*>(p.resid + (size_t)m * p.ldo + n);
            } else if constexpr (EPI == EPI_QKV) {
                if (n < p.rope_cols) {
                    const int i2 = (n % p.head_dim) >> 1;  // even: pairs i2, i2 + 1
                    const size_t o = (size_t)p.row_pos[m] * (p.head_dim >> 1) + i2;
                    const float2 c = *reinterpret_cast<const float2*>(p.rope_cos + o);
                    const float2 s = *reinterpret_cast<const float2*>(p.rope_sin + o);
                    pre[u] = make_float4(c.x, s.x, c.y, s.y);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            if (!act[u]) continue;
            const int m = rbase + rr[u];
            float4 x = *reinterpret_cast<const float4*>(stg + rr[u] * SROW + 4 * cg);
            if constexpr (EPI == EPI_I32) {
                *reinterpret_cast<int4*>(out_i32 + (size_t)m * p.ldo + n) =
                    make_int4(__float_as_int(x.x), __float_as_int(x.y), __float_as_int(x.z), __float_as_int(x.w));
            } else if constexpr (EPI == EPI_F32 || EPI == EPI_LOGITS3) {
                *reinterpret_cast<float4*>(p.out + (size_t)m * p.ldo + n) = x;
            } else if constexpr (EPI == EPI_QKV) {
                if (n < p.rope_cols) {
                    rope_pair(x.x, x.y, pre[u].x, pre[u].y);
                    rope_pair(x.z, x.w, pre[u].z, pre[u].w);
                }
                *reinterpret_cast<float4*>(p.out + (size_t)m * p.ldo + n) = x;
            } else if constexpr (RESID) {
                float4 r = pre[u];
                r.x = __fadd_rn(r.x, x.x);
                r.y = __fadd_rn(r.y, x.y);
                r.z = __fadd_rn(r.z, x.z);
                r.w = __fadd_rn(r.w, x.w);
                *reinterpret_cast<float4*>(p.resid + (size_t)m * p.ldo + n) = r;
            } else if constexpr (EPI == EPI_SWIGLU || EPI == EPI_MTP_SWIGLU3) {
                *reinterpret_cast<float4*>(p.out + (size_t)m * p.ldo + n) = x;  // activations of pass 1
            }
        }
    }
}

template <int BN, int P, int WF, int EPI, int TM = 1>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmParams p,
                   int plane_rows, uint32_t* err) {
    using Ly = Layout<BN, P, WF, TM>;
    constexpr int STAGES = Ly::STAGES;
    constexpr int RB = row_bytes<WF>();
    constexpr int SHIFT = WF == WF_Q4 ? 4 : (WF == WF_Q2 ? 6 : 0);  // weight position inside its byte
    constexpr int HALF = BN / 2;                                      // columns per epilogue warp
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bars = sbase + Ly::BAR_OFF;
    constexpr int NB = Ly::NB;
    auto full_raw = [&](int s) { return bars + 8u * s; };       // slot s loaded
    auto empty = [&](int s) { return bars + 8u * (STAGES + s); };  // slot s consumed by the MMAs
    auto b_full = [&](int b) { return bars + 8u * (2 * STAGES + b); };       // buffer b unpacked
    auto b_empty = [&](int b) { return bars + 8u * (2 * STAGES + NB + b); };  // buffer b read by the MMAs
    const uint32_t done = bars + 8u * (2 * STAGES + 2 * NB);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Ly::BAR_OFF + 8 * (2 * STAGES + 2 * NB + 1));
    volatile int* abort_flag =
        reinterpret_cast<volatile int*>(smem + Ly::BAR_OFF + 8 * (2 * STAGES + 2 * NB + 1) + 8);
    // slot s: activation tiles (M tile t, plane pl) at index t * P + pl, then the packed weights
    auto a_addr = [&](int s, int pl, int t = 0) {
        return sbase + (uint32_t)(s * Ly::SLOT_BYTES + (t * P + pl) * Ly::A_BYTES);
    };
    auto raw_addr = [&](int s) { return sbase + (uint32_t)(s * Ly::SLOT_BYTES + TM * P * Ly::A_BYTES); };
    auto b_addr = [&](int b) { return sbase + (uint32_t)(Ly::B_OFF + b * Ly::B_BYTES); };

    // The next kernel may start its prologue now; it waits for this grid's
    // completion before it reads anything this grid writes.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) {
        prefetch_map(&tmA);
        prefetch_map(&tmB);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM * TM;  // TM tiles of 128 rows share each weight stage
    const int nkt = p.K / BK;
    const int per = (nkt + p.splits - 1) / p.splits;
    const int kt0 = blockIdx.z * per, kt1 = min(nkt, kt0 + per);
    const int nst = max(0, kt1 - kt0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full_raw(s), TM * P + 1);  // one arrival per issuing lane
            mbar_init(empty(s), 1);
        }
        for (int b = 0; b < NB; b++) {
            mbar_init(b_full(b), NUM_UNPACK / 32);  // one arrival per unpack warp
            mbar_init(b_empty(b), 1);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(Ly::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tmem_slot;

    auto fail = [&]() {
        *abort_flag = 1;
        if (err) atomicOr(err, ERR_TIMEOUT);
    };

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        // Copies issued by one thread are processed one after another, so
        // each (slot, copy) pair has its own lane: lane s*(P+1)+c issues copy
        // c (activation plane c, or the packed weights for c == P) of every
        // stage that uses slot s, and arrives on full_raw[s] with its bytes.
        constexpr int COPIES = TM * P + 1;  // activation tiles of every (M tile, plane), then the weights
        static_assert(STAGES * COPIES <= 32, "one lane per (slot, copy)");
        if (lane < STAGES * COPIES) {
            const int s = lane / COPIES, c = lane % COPIES;
            const uint32_t bytes = (uint32_t)(c < TM * P ? Ly::A_BYTES : Ly::RAW_BYTES);
            // Activations come from the previous kernel: under programmatic
            // dependent launch, wait for it.  Weights do not, so their
            // copies may start while it finishes.
            if (c < TM * P) asm volatile("griddepcontrol.wait;" ::: "memory");
            int last = -1;
            for (int i = s; i < nst && !*abort_flag; i += STAGES) {
                if (!mbar_wait(empty(s), ((i / STAGES) & 1) ^ 1)) {
                    fail();
                    break;
                }
                const int kt = kt0 + i;
                mbar_expect_tx(full_raw(s), bytes);
                if (c < TM * P)  // tile c / P, plane c % P (rows past M read as zeros)
                    tma_load_2d(a_addr(s, c % P, c / P), &tmA, kt * BK, (c % P) * plane_rows + m0 + (c / P) * BM,
                                full_raw(s));
                else
                    tma_load_2d(raw_addr(s), &tmB, 0, kt * p.N + n0, full_raw(s));
                last = i;
            }
            // On abort, let this lane's copy still in flight land (bounded)
            // before the CTA's shared memory is released.
            if (*abort_flag && last >= 0) (void)mbar_wait(full_raw(s), (last / STAGES) & 1);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_i8(BN);
            for (int i = 0; i < nst && !*abort_flag; i++) {
                const int s = i % STAGES, ph = (i / STAGES) & 1;
                // b_full completes only after every unpack warp saw
                // full_raw (activation and weight copies landed) and
                // arrived, so it orders the MMAs after both.
                const int b = i % NB;
                if (!mbar_wait(b_full(b), (i / NB) & 1)) {
                    fail();
                    break;
                }
                (void)ph;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint64_t bd = sw128_desc(b_addr(b));
#pragma unroll
                for (int tt = 0; tt < TM; tt++)  // every M tile against the one unpacked weight stage
#pragma unroll
                    for (int pl = 0; pl < P; pl++) {
                        const uint64_t ad = sw128_desc(a_addr(s, pl, tt));
#pragma unroll
                        for (int kk = 0; kk < BK / 32; kk++)  // K = 32 bytes per MMA: +2 in 16-byte units
                            umma_i8(tmem + (uint32_t)((tt * P + pl) * BN), ad + 2 * kk, bd + 2 * kk, idesc,
                                    (i > 0 || kk > 0) ? 1u : 0u);
                    }
                umma_commit(empty(s));
                umma_commit(b_empty(b));
            }
            umma_commit(done);  // fires once every issued MMA has completed
        }
    } else {
        // ---------------- weight unpack (warps 2..9), then epilogue ----------------
        const int t = threadIdx.x - 64;  // 0 .. NUM_UNPACK-1
        float* s_wsc = reinterpret_cast<float*>(smem + Ly::WSC_OFF);
        for (int c = t; c < BN; c += NUM_UNPACK) s_wsc[c] = p.w_scale ? p.w_scale[n0 + c] : 1.0f;
        constexpr int CH_IN = BN * RB / 16;  // 16-byte packed chunks per stage
        constexpr int PER = (CH_IN + NUM_UNPACK - 1) / NUM_UNPACK;
        static_assert(CH_IN % NUM_UNPACK == 0 || PER == 1, "partial rounds only with one chunk per thread");
        for (int i = 0; i < nst; i++) {
            // Exits are warp-uniform: the warp arrives on b_full as one below.
            if (__shfl_sync(0xffffffffu, *abort_flag, 0)) break;
            const int s = i % STAGES, ph = (i / STAGES) & 1;
            const int b = i % NB;
            const bool got = mbar_wait(full_raw(s), ph) && mbar_wait(b_empty(b), ((i / NB) & 1) ^ 1);
            if (!__all_sync(0xffffffffu, got)) {
                fail();
                break;
            }
            const uint8_t* raw = smem + (raw_addr(s) - sbase);
            uint8_t* bt = smem + (b_addr(b) - sbase);
            uint4 wv[PER];
#pragma unroll
            for (int u = 0; u < PER; u++)
                if (CH_IN >= NUM_UNPACK || t < CH_IN) wv[u] = reinterpret_cast<const uint4*>(raw)[t + NUM_UNPACK * u];
#pragma unroll
            for (int u = 0; u < PER; u++) {
                const int q = t + NUM_UNPACK * u;
                if (CH_IN < NUM_UNPACK && q >= CH_IN) break;
                const int row = q / (RB / 16), c = q % (RB / 16);
                const uint4 w = wv[u];
                const int r7 = row & 7;
                uint8_t* rb = bt + (row >> 3) * 1024 + r7 * 128;
                // Each weight lands in the top bits of its byte (v * 2^SHIFT, exact
                // in int8); the epilogue shifts the int32 sums back down.
                if constexpr (WF == WF_Q4) {
                    constexpr uint32_t HI = 0xF0F0F0F0u;  // k [32c, 32c+16): low nibbles; [32c+16, 32c+32): high
                    const uint4 lo = make_uint4((w.x << 4) & HI, (w.y << 4) & HI, (w.z << 4) & HI, (w.w << 4) & HI);
                    const uint4 hi = make_uint4(w.x & HI, w.y & HI, w.z & HI, w.w & HI);
                    *reinterpret_cast<uint4*>(rb + (((2 * c) ^ r7) << 4)) = lo;
                    *reinterpret_cast<uint4*>(rb + (((2 * c + 1) ^ r7) << 4)) = hi;
                } else if constexpr (WF == WF_Q2) {
                    constexpr uint32_t HI = 0xC0C0C0C0u;
#pragma unroll
                    for (int sft = 0; sft < 4; sft++) {  // k [64c + 16 sft, +16): bits [2 sft, 2 sft + 2)
                        const int sh = 6 - 2 * sft;
                        const uint4 o = make_uint4((w.x << sh) & HI, (w.y << sh) & HI, (w.z << sh) & HI, (w.w << sh) & HI);
                        *reinterpret_cast<uint4*>(rb + (((4 * c + sft) ^ r7) << 4)) = o;
                    }
                } else {
                    *reinterpret_cast<uint4*>(rb + ((c ^ r7) << 4)) = w;
                }
            }
            // Every thread makes its generic-proxy writes visible to the
            // tensor core's async proxy; the warp then arrives once.
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(b_full(b));
        }
        // ---------------- epilogue ----------------
        asm volatile("griddepcontrol.wait;" ::: "memory");  // resid, scales, workspace of earlier kernels
        // `ok` must be the same for all epilogue threads: the TMEM loads below
        // are warp-collective and the split-K path uses a named barrier.
        __shared__ int s_ok, s_last;
        const bool okl = !*abort_flag && mbar_wait(done, 0);
        if (!okl) fail();
        named_sync();
        if (t == 0) s_ok = !*abort_flag;
        named_sync();
        const bool ok = s_ok != 0;
        asm volatile("tcgen05.fence::after_thread_sync;");
        // Warp w reads TMEM lanes 32*(w%4) .. +31 (tile rows) and one half of
        // the tile's columns.
        const int sub = warp & 3;
        const int c0 = ((warp - 2) >> 2) * HALF;
        for (int tt = 0; tt < TM; tt++) {  // the CTA's M tiles, one after another (TM > 1: no split K)
        const int m0t = m0 + tt * BM;
        const int m = m0t + sub * 32 + lane;
        const bool in_m = m < p.M;
        const uint32_t tbase = tmem + ((uint32_t)(sub * 32) << 16) + (uint32_t)(tt * P * BN);
        bool write_tile = ok;
        if (ok && p.splits > 1 && p.slice_stride == 0) {
            // Split-K: every split adds its partial sums into the workspace,
            // laid out [plane][n][m] so that a warp's 32 rows are 32 adjacent
            // words; the split that retires the tile last reads the totals
            // back, re-zeroes them and runs the epilogue.
            if (nst > 0) {
                for (int j = 0; j < HALF / 16; j++) {
                    uint32_t r[P][16];
#pragma unroll
                    for (int pl = 0; pl < P; pl++) tmem_ld16(tbase + (uint32_t)(pl * BN + c0 + j * 16), r[pl]);
                    if (!in_m) continue;
#pragma unroll
                    for (int pl = 0; pl < P; pl++)
#pragma unroll
                        for (int c = 0; c < 16; c++)
                            if (r[pl][c] != 0)
                                atomicAdd(p.ws + ((size_t)pl * p.N + n0 + c0 + j * 16 + c) * p.M + m, (int32_t)r[pl][c]);
                }
            }
            __threadfence();
            named_sync();
            const int tile = blockIdx.y * gridDim.x + blockIdx.x;
            if (t == 0) s_last = (atomicAdd(p.counters + tile, 1) == p.splits - 1);
            named_sync();
            write_tile = s_last != 0;
            if (write_tile) {
                __threadfence();
                if (t == 0) p.counters[tile] = 0;
            }
        }
        if (write_tile) {
            // Pass 1: per-column values of this thread's row -> its warp's
            // staging rows (row stride HALF + 4 words: conflict-free).
            float* stg = reinterpret_cast<float*>(smem) + (warp - 2) * 32 * Ly::SROW;
            const float a_s = (in_m && EPI != EPI_I32) ? p.a_scale[m] : 0.0f;  // (int32 slices: no scales)
            const float s_all = __fmul_rn(a_s, p.w_scale_all);
            constexpr bool SWI = EPI == EPI_SWIGLU || EPI == EPI_MTP_SWIGLU3;
            // TMEM chunks loaded per wait: one round trip covers up to 64 columns.
            constexpr int JB = (P == 1) ? (HALF / 16 < 4 ? HALF / 16 : 4) : 1;
            static_assert((HALF / 16) % JB == 0, "chunk batches");
            for (int j0 = 0; j0 < HALF / 16; j0 += JB) {
                uint32_t r[JB][P][16];
                if (p.splits > 1 && p.slice_stride == 0) {
                    // All loads of the chunk are issued before anything is
                    // written; the workspace is re-zeroed after the tile.
#pragma unroll
                    for (int jj = 0; jj < JB; jj++)
#pragma unroll
                        for (int pl = 0; pl < P; pl++)
#pragma unroll
                            for (int c = 0; c < 16; c++)
                                r[jj][pl][c] =
                                    in_m ? (uint32_t)__ldcg(p.ws + ((size_t)pl * p.N + n0 + c0 + (j0 + jj) * 16 + c) * p.M + m)
                                         : 0u;
                } else {
#pragma unroll
                    for (int jj = 0; jj < JB; jj++)
#pragma unroll
                        for (int pl = 0; pl < P; pl++)
                            tmem_ld16_nowait(tbase + (uint32_t)(pl * BN + c0 + (j0 + jj) * 16), r[jj][pl]);
                    tmem_wait_ld();
                }
#pragma unroll
                for (int jj = 0; jj < JB; jj++) {
                    const int j = j0 + jj;
                    float v[16];
#pragma unroll
                    for (int c = 0; c < 16; c++) {
                        int32_t a[P];
#pragma unroll
                        for (int pl = 0; pl < P; pl++) a[pl] = (int32_t)r[jj][pl][c] >> SHIFT;  // exact: a multiple of 2^SHIFT
                        v[c] = col_value<P, EPI>(a, a_s, s_wsc[c0 + j * 16 + c], s_all);
                    }
                    if constexpr (SWI) {
                        // (gate, up) column pairs -> 8 activations of this row
                        float o[8];
#pragma unroll
                        for (int q = 0; q < 8; q++)
                            o[q] = EPI == EPI_SWIGLU ? engine_swiglu(v[2 * q], v[2 * q + 1]) : mtp_swiglu(v[2 * q], v[2 * q + 1]);
                        float4* d = reinterpret_cast<float4*>(stg + lane * Ly::SROW + j * 8);
                        d[0] = make_float4(o[0], o[1], o[2], o[3]);
                        d[1] = make_float4(o[4], o[5], o[6], o[7]);
                    } else {
                        float4* d = reinterpret_cast<float4*>(stg + lane * Ly::SROW + j * 16);
#pragma unroll
                        for (int q = 0; q < 4; q++) d[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                    }
                }
            }
            __syncwarp();
            if (p.splits > 1 && p.slice_stride == 0 && in_m) {
                for (int pl = 0; pl < P; pl++)
                    for (int c = 0; c < HALF; c++) __stcg(p.ws + ((size_t)pl * p.N + n0 + c0 + c) * p.M + m, 0);
            }
            // Pass 2: whole rows, 4 adjacent columns per lane, coalesced.
            // Slices mode: split z writes its own int32 tile (reduced later).
            int32_t* oi = p.out_i32 ? p.out_i32 + (size_t)blockIdx.z * p.slice_stride : nullptr;
            if constexpr (SWI)
                store_rows<HALF / 2, Ly::SROW, EPI>(p, stg, m0t + sub * 32, (n0 + c0) >> 1, lane, oi);
            else
                store_rows<HALF, Ly::SROW, EPI>(p, stg, m0t + sub * 32, n0 + c0, lane, oi);
        }
        __syncwarp();  // this warp's staging rows are read before the next tile's pass 1 writes them
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Ly::TMEM_COLS));
    }
}

// ---------------------------------------------------------------------------
// Host side: tensor maps through the driver entry point (no libcuda link).
// ---------------------------------------------------------------------------
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

pf_status get_encode(EncodeTiled* fn) {
    static std::mutex mu;
    static EncodeTiled cached = nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!cached) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        PF_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q));
        PF_CHECK(f && q == cudaDriverEntryPointSuccess, "cuTensorMapEncodeTiled unavailable");
        cached = reinterpret_cast<EncodeTiled>(f);
    }
    *fn = cached;
    return PF_OK;
}

pf_status make_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t row_stride,
                   uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz) {
    EncodeTiled enc;
    PF_TRY(get_encode(&enc));
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {row_stride};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    PF_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return PF_OK;
}

template <int BN, int P, int WF, int EPI, int TM = 1>
pf_status launch_tc(const GemmParams& p, int plane_rows, cudaStream_t st) {
    using Ly = Layout<BN, P, WF, TM>;
    static_assert(Ly::STAGES >= 2, "shared memory budget too small");
    CUtensorMap ta, tb;
    const uint64_t a_rows = (P == 1) ? (uint64_t)p.M : (uint64_t)P * plane_rows;
    PF_TRY(make_map(&ta, p.A, (uint64_t)p.K, a_rows, (uint64_t)p.lda, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B));
    PF_TRY(make_map(&tb, p.W, (uint64_t)row_bytes<WF>(), (uint64_t)(p.K / BK) * p.N, (uint64_t)row_bytes<WF>(),
                    row_bytes<WF>(), BN, CU_TENSOR_MAP_SWIZZLE_NONE));
    static std::atomic<uint64_t> attr{0};
    PF_TRY(raise_smem_limit(gemm_tc_kernel<BN, P, WF, EPI, TM>, Ly::SMEM, attr));
    dim3 grid(p.N / BN, ceil_div(p.M, BM * TM), p.splits);
    uint32_t* err = device_error_flag();
    if (p.pdl) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = grid;
        cfg.blockDim = dim3(NUM_THREADS);
        cfg.dynamicSmemBytes = Ly::SMEM;
        cfg.stream = st;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        PF_CUDA(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, P, WF, EPI, TM>, ta, tb, p, plane_rows, err));
    } else {
        gemm_tc_kernel<BN, P, WF, EPI, TM><<<grid, NUM_THREADS, Ly::SMEM, st>>>(ta, tb, p, plane_rows, err);
    }
    return launch_check("gemm_tc");
}

template <int BN, int P, int EPI, int TM = 1>
pf_status launch_wf(const GemmParams& p, int plane_rows, cudaStream_t st) {
    switch (p.wf) {
        case WF_Q4: return launch_tc<BN, P, WF_Q4, EPI, TM>(p, plane_rows, st);
        case WF_Q2: return launch_tc<BN, P, WF_Q2, EPI, TM>(p, plane_rows, st);
        default: return launch_tc<BN, P, WF_I8, EPI, TM>(p, plane_rows, st);
    }
}

// Two 128-row M tiles per CTA (both accumulators in TMEM, each unpacked
// weight stage feeding both): ~30% fewer shared-memory bytes per MMA, for
// launches whose tile pairs still fill two waves (prefill-sized M).
bool use_two_m_tiles(const GemmParams& p, int planes, int bn) {
    return planes == 1 && bn == 256 && p.epi == EPI_SWIGLU && p.splits == 1 &&
           (size_t)ceil_div(p.M, 2 * BM) * (p.N / bn) >= 2 * 148;
}

template <int BN>
pf_status launch_bn(const GemmParams& p, int planes, int plane_rows, cudaStream_t st) {
    if (planes == 3) {
        if constexpr (BN <= 128) {  // three planes of 256 columns do not fit TMEM
            switch (p.epi) {
                case EPI_LOGITS3: return launch_wf<BN, 3, EPI_LOGITS3>(p, plane_rows, st);
                case EPI_MTP_SWIGLU3: return launch_wf<BN, 3, EPI_MTP_SWIGLU3>(p, plane_rows, st);
                default: return launch_wf<BN, 3, EPI_MTP_RESID3>(p, plane_rows, st);
            }
        } else {
            PF_CHECK(false, "gemm_tc: three planes need N tiles of at most 128");
        }
    }
    switch (p.epi) {
        case EPI_I32: return launch_wf<BN, 1, EPI_I32>(p, plane_rows, st);
        case EPI_F32: return launch_wf<BN, 1, EPI_F32>(p, plane_rows, st);
        case EPI_QKV: return launch_wf<BN, 1, EPI_QKV>(p, plane_rows, st);
        case EPI_RESID: return launch_wf<BN, 1, EPI_RESID>(p, plane_rows, st);
        default:
            if constexpr (BN == 256)
                if (use_two_m_tiles(p, planes, BN)) return launch_wf<BN, 1, EPI_SWIGLU, 2>(p, plane_rows, st);
            return launch_wf<BN, 1, EPI_SWIGLU>(p, plane_rows, st);
    }
}

// ---------------------------------------------------------------------------
// Packing to the tensor-core layout: [K/128][N][RB] with, per 128-wide block,
//   Q4: 4 chunks of 16 B; chunk c byte j = low nibble k 32c+j, high nibble k 32c+16+j;
//   Q2: 2 chunks of 16 B; chunk c byte j bits [2s, 2s+2) = k 64c+16s+j;
//   I8: the 128 bytes in order.  Fields are two's complement (v & 0xF, v & 0x3).
// ---------------------------------------------------------------------------
__global__ void pack_tc_kernel(const int8_t* __restrict__ w, int rows, int cols, int wf, uint8_t* __restrict__ out,
                               int nkb, uint32_t* err) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one 16-byte chunk
    const int rb = wf == WF_Q4 ? 64 : (wf == WF_Q2 ? 32 : 128);
    const int cpr = rb / 16;
    const int64_t total = (int64_t)nkb * rows * cpr;
    if (idx >= total) return;
    const int c = (int)(idx % cpr);
    const int64_t rem = idx / cpr;
    const int n = (int)(rem % rows);
    const int kb = (int)(rem / rows);
    auto val = [&](int k) -> int { return k < cols ? (int)w[(size_t)n * cols + k] : 0; };
    uint8_t bytes[16];
    bool bad = false;
    for (int j = 0; j < 16; j++) {
        const int k0 = kb * 128;
        if (wf == WF_Q4) {
            const int lo = val(k0 + 32 * c + j), hi = val(k0 + 32 * c + 16 + j);
            bad |= lo < -8 || lo > 7 || hi < -8 || hi > 7;
            bytes[j] = (uint8_t)((lo & 0xF) | ((hi & 0xF) << 4));
        } else if (wf == WF_Q2) {
            uint8_t b = 0;
            for (int s = 0; s < 4; s++) {
                const int v = val(k0 + 64 * c + 16 * s + j);
                bad |= v < -2 || v > 1;
                b |= (uint8_t)((v & 3) << (2 * s));
            }
            bytes[j] = b;
        } else {
            bytes[j] = (uint8_t)(val(k0 + 16 * c + j) & 0xFF);
        }
    }
    uint4 o;
    memcpy(&o, bytes, 16);
    reinterpret_cast<uint4*>(out)[idx] = o;
    if (bad) atomicOr(err, ERR_WEIGHT_RANGE);
}

}  // namespace

size_t packed_bytes_tc(int rows, int cols, int wf) {
    const int rb = wf == WF_Q4 ? 64 : (wf == WF_Q2 ? 32 : 128);
    return (size_t)ceil_div(cols, 128) * rows * rb;
}

pf_status pack_weights_tc(const int8_t* w, int rows, int cols, int wf, void* packed, cudaStream_t st) {
    PF_CHECK(rows > 0 && cols > 0 && w && packed, "pack_weights_tc: bad arguments");
    const int nkb = ceil_div(cols, 128);
    const int cpr = (wf == WF_Q4 ? 64 : (wf == WF_Q2 ? 32 : 128)) / 16;
    const int64_t total = (int64_t)nkb * rows * cpr;
    pack_tc_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(w, rows, cols, wf, (uint8_t*)packed, nkb,
                                                                     device_error_flag());
    return launch_check("pack_weights_tc");
}

int gemm_tc_pick_bn(int M, int N, int planes) {
    // Wider MMAs do more work per issued instruction and per stage barrier
    // (N = 64 runs below the tensor pipe's rate); narrow only where the wide
    // tile leaves too few CTAs.  Three accumulator planes of 256 columns do
    // not fit TMEM.
    const int mt = ceil_div(M, BM);
    if (planes == 1 && N % 256 == 0 && mt * (N / 256) >= 100) return 256;
    if (N % 128 == 0 && mt * (N / 128) >= 40) return 128;
    return 64;
}

int gemm_tc_slices(int M, int N, int K) {
    // Enough (tile, split) CTAs to cover the SMs once, at most 4 splits of at
    // least 4 K stages each.
    const int bn = gemm_tc_pick_bn(M, N, 1);
    const int tiles = ceil_div(M, BM) * (N / bn);
    const int s = std::min(148 / std::max(1, tiles), std::min(4, (K / BK) / 4));
    return std::max(1, s);
}

int gemm_tc_pick_splits(int M, int N, int K, int bn, bool have_ws) {
    if (!have_ws) return 1;
    const int tiles = ceil_div(M, BM) * (N / bn);
    const int nkt = K / BK;
    int s = (tiles >= 120) ? 1 : ceil_div(148, tiles);
    s = std::min(s, std::max(1, nkt / 2));
    return std::max(1, std::min(s, 8));
}

pf_status gemm_tc_launch(const GemmParams& p0, int planes, int plane_rows, cudaStream_t st) {
    GemmParams p = p0;
    PF_CHECK(p.M > 0 && p.N > 0 && p.K > 0, "gemm_tc: empty shape");
    PF_CHECK(p.N % 64 == 0, "gemm_tc: N=%d must be a multiple of 64", p.N);
    PF_CHECK(p.K % BK == 0, "gemm_tc: K=%d must be a multiple of %d", p.K, BK);
    PF_CHECK(p.lda % 16 == 0 && p.lda >= p.K, "gemm_tc: lda=%d must be >= K and a multiple of 16", p.lda);
    PF_CHECK((reinterpret_cast<uintptr_t>(p.A) & 15) == 0 && (reinterpret_cast<uintptr_t>(p.W) & 15) == 0,
             "gemm_tc: operands must be 16-byte aligned");
    PF_CHECK(planes == 1 || planes == 3, "gemm_tc: planes must be 1 or 3");
    // The epilogue writes 16-byte runs of rows (8-byte runs for the SwiGLU
    // forms) and reads RoPE angles in pairs.
    const void* dst = p.epi == EPI_I32 ? (const void*)p.out_i32
                      : (p.epi == EPI_RESID || p.epi == EPI_MTP_RESID3) ? (const void*)p.resid : (const void*)p.out;
    PF_CHECK(dst && (reinterpret_cast<uintptr_t>(dst) & 15) == 0 && p.ldo % 4 == 0,
             "gemm_tc: output must be 16-byte aligned with a row stride that is a multiple of 4");
    PF_CHECK(p.epi != EPI_QKV || p.rope_cols == 0 ||
                 (p.head_dim % 4 == 0 && p.rope_cols % 4 == 0 && ((reinterpret_cast<uintptr_t>(p.rope_cos) |
                                                                    reinterpret_cast<uintptr_t>(p.rope_sin)) & 7) == 0),
             "gemm_tc: RoPE tables must be 8-byte aligned and head_dim a multiple of 4");
    PF_CHECK(planes == 1 || (plane_rows >= p.M && p.plane_stride == (int64_t)plane_rows * p.lda),
             "gemm_tc: plane layout must be [planes][plane_rows][lda]");
    const bool three = p.epi == EPI_LOGITS3 || p.epi == EPI_MTP_SWIGLU3 || p.epi == EPI_MTP_RESID3;
    PF_CHECK(three == (planes == 3), "gemm_tc: epilogue %d does not take %d planes", p.epi, planes);
    if (gemv_applies(p, planes)) return gemv_launch(p, planes, st);  // a few rows: dp4a, weights streamed once
    const int bn = gemm_tc_pick_bn(p.M, p.N, planes);
    if (p.slice_stride > 0) {  // split K into separate int32 slices, reduced by the caller's next kernel
        PF_CHECK(p.epi == EPI_I32 && planes == 1 && p.splits >= 1 && p.splits <= p.K / BK,
                 "gemm_tc: slices need EPI_I32, one plane and 1..K/128 splits");
        PF_CHECK(p.slice_stride >= (int64_t)p.M * p.ldo, "gemm_tc: slice stride below M * ldo");
        if (bn == 256) return launch_bn<256>(p, planes, plane_rows, st);
        if (bn == 128) return launch_bn<128>(p, planes, plane_rows, st);
        return launch_bn<64>(p, planes, plane_rows, st);
    }
    if (p.splits <= 0) {  // automatic: split K only when the tiles do not fill the GPU and a workspace fits
        p.splits = gemm_tc_pick_splits(p.M, p.N, p.K, bn, p.ws != nullptr && p.counters != nullptr);
        const size_t tiles = (size_t)ceil_div(p.M, BM) * (p.N / bn);
        if (p.splits > 1 && ((size_t)planes * p.M * p.N > p.ws_elems || tiles > p.cnt_elems)) p.splits = 1;
    }
    PF_CHECK(p.splits == 1 || (p.ws && p.counters), "gemm_tc: split-K needs a workspace");
    PF_CHECK(p.splits <= p.K / BK, "gemm_tc: more splits than K blocks");
    if (bn == 256) return launch_bn<256>(p, planes, plane_rows, st);
    if (bn == 128) return launch_bn<128>(p, planes, plane_rows, st);
    return launch_bn<64>(p, planes, plane_rows, st);
}

}  // namespace pf

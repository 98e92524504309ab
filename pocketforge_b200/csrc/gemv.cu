// gemv.cu — the projection for a few activation rows (one or two sequences'
// verify rows, the MTP chain of one sequence): int8 activations x packed
// Q4 / Q2 / int8 weights on the dp4a path, every weight byte loaded once with
// coalesced 16-byte loads and unpacked in registers.
//
// Semantics are gemm_tc.cu's (matmul_int8 / matmul_quantized,
// src/matmul_neon.cpp:80-181): exact int32 sums, then the same epilogues.  At
// a few rows the tensor-core kernel's 128-row tiles are almost all padding and
// its per-launch costs dominate; this kernel streams the weights at the rate
// of the memory system instead.
//
// Weights are in gemm_tc.cu's packed layout [K/128][N][RB]: for one 128-wide
// K block the RB bytes of consecutive rows are contiguous, so a warp's 32
// 16-byte loads cover 32 * 16 / RB rows of one K block (Q4: 8 rows x 4
// chunks, Q2: 16 x 2, int8: 4 x 8).  Q4 chunk c byte j holds k = 32c + j in
// its low nibble and k = 32c + 16 + j in its high nibble; Q2 chunk c byte j
// holds k = 64c + 16s + j in bits 2s..2s+1; int8 chunk c holds k = 16c .. +15.
// Every field is moved to the top bits of its byte (v * 2^SHIFT, exact in
// int8) and the dp4a sums are shifted back (exact: multiples of 2^SHIFT).
//
// Grid (row tiles of 8 warps, K splits).  The activation rows of the CTA's K
// range are staged in shared memory; lane (row r, chunk c) accumulates one
// int32 sum per activation row, the CPR lanes of a row are added with
// shuffles, and the epilogue runs on the lanes of chunk 0.  Under
// programmatic dependent launch the first weight loads are issued before the
// previous kernel has finished; the activations are read after it.
#include <cuda_runtime.h>

#include <algorithm>

#include "gemm.cuh"
#include "numerics.cuh"
#include "gemm_tc.cuh"

namespace pf {

namespace {

constexpr int GV_WARPS = 8;
constexpr int GV_THREADS = 32 * GV_WARPS;
constexpr int GV_UNROLL = 4;  // K blocks whose weight loads are in flight per lane
constexpr size_t GV_SMEM_MAX = 160 * 1024;  // activation bytes a CTA stages (gemv_applies keeps launches below)

template <int WF>
struct Fmt {
    static constexpr int RB = WF == WF_Q4 ? 64 : (WF == WF_Q2 ? 32 : 128);  // bytes per row and K block
    static constexpr int CPR = RB / 16;                                       // 16-byte chunks per row
    static constexpr int RPW = 32 / CPR;                                      // rows per warp
    static constexpr int RPC = RPW * GV_WARPS;                                // rows per CTA
    static constexpr int KPC = 128 / CPR;                                     // K values per chunk
    static constexpr int SHIFT = WF == WF_Q4 ? 4 : (WF == WF_Q2 ? 6 : 0);
};

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

__device__ __forceinline__ float engine_swiglu(float g, float u) { return engine_swiglu_rn(g, u); }  // engine FFN form

// acc[r] += dot(activation row r over this chunk's K values, weights w)
template <int WF, int RT>
__device__ __forceinline__ void chunk_dot(const uint4 w, const uint8_t* __restrict__ a_chunk, int a_stride,
                                          int (&acc)[RT], int rows) {
    if constexpr (WF == WF_Q4) {
        constexpr uint32_t HI = 0xF0F0F0F0u;
        const uint32_t lo[4] = {(w.x << 4) & HI, (w.y << 4) & HI, (w.z << 4) & HI, (w.w << 4) & HI};
        const uint32_t hi[4] = {w.x & HI, w.y & HI, w.z & HI, w.w & HI};
#pragma unroll
        for (int r = 0; r < RT; r++) {
            if (r >= rows) break;
            const uint4 a0 = *reinterpret_cast<const uint4*>(a_chunk + (size_t)r * a_stride);       // k 32c .. +15
            const uint4 a1 = *reinterpret_cast<const uint4*>(a_chunk + (size_t)r * a_stride + 16);  // k 32c+16 .. +31
            int s = acc[r];
            s = dp4a((int)a0.x, (int)lo[0], s);
            s = dp4a((int)a0.y, (int)lo[1], s);
            s = dp4a((int)a0.z, (int)lo[2], s);
            s = dp4a((int)a0.w, (int)lo[3], s);
            s = dp4a((int)a1.x, (int)hi[0], s);
            s = dp4a((int)a1.y, (int)hi[1], s);
            s = dp4a((int)a1.z, (int)hi[2], s);
            s = dp4a((int)a1.w, (int)hi[3], s);
            acc[r] = s;
        }
    } else if constexpr (WF == WF_Q2) {
        constexpr uint32_t HI = 0xC0C0C0C0u;
        uint32_t q[4][4];
#pragma unroll
        for (int sft = 0; sft < 4; sft++) {  // k 64c + 16 sft + j: bits [2 sft, 2 sft + 2)
            const int sh = 6 - 2 * sft;
            q[sft][0] = (w.x << sh) & HI;
            q[sft][1] = (w.y << sh) & HI;
            q[sft][2] = (w.z << sh) & HI;
            q[sft][3] = (w.w << sh) & HI;
        }
#pragma unroll
        for (int r = 0; r < RT; r++) {
            if (r >= rows) break;
            int s = acc[r];
#pragma unroll
            for (int sft = 0; sft < 4; sft++) {
                const uint4 a = *reinterpret_cast<const uint4*>(a_chunk + (size_t)r * a_stride + 16 * sft);
                s = dp4a((int)a.x, (int)q[sft][0], s);
                s = dp4a((int)a.y, (int)q[sft][1], s);
                s = dp4a((int)a.z, (int)q[sft][2], s);
                s = dp4a((int)a.w, (int)q[sft][3], s);
            }
            acc[r] = s;
        }
    } else {
#pragma unroll
        for (int r = 0; r < RT; r++) {
            if (r >= rows) break;
            const uint4 a = *reinterpret_cast<const uint4*>(a_chunk + (size_t)r * a_stride);
            int s = acc[r];
            s = dp4a((int)a.x, (int)w.x, s);
            s = dp4a((int)a.y, (int)w.y, s);
            s = dp4a((int)a.z, (int)w.z, s);
            s = dp4a((int)a.w, (int)w.w, s);
            acc[r] = s;
        }
    }
}

// RT: activation rows (planes x M) the kernel is compiled for (>= the launch's).
template <int WF, int RT, int EPI, int P>
__global__ void __launch_bounds__(GV_THREADS) gemv_kernel(const GemmParams p) {
    using F = Fmt<WF>;
    extern __shared__ __align__(16) uint8_t gv_smem[];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = lane % F::CPR, rw = lane / F::CPR;
    const int n = blockIdx.x * F::RPC + warp * F::RPW + rw;  // this lane's output row (weight row)
    const bool n_ok = n < p.N;
    const int nkb = p.K / 128;
    const int splits = gridDim.y;
    const int per = (nkb + splits - 1) / splits;
    const int kb0 = blockIdx.y * per, kb1 = min(nkb, kb0 + per);
    const int nk = max(0, kb1 - kb0);
    const int M = p.M;
    const int rows = P * M;  // activation rows (plane-major)
    const uint8_t* Wb = reinterpret_cast<const uint8_t*>(p.W);
    auto wptr = [&](int kb) { return Wb + ((size_t)kb * p.N + n) * F::RB + c * 16; };

    // The weights do not depend on the previous kernel: the first loads go out now.
    uint4 wbuf[GV_UNROLL];
#pragma unroll
    for (int u = 0; u < GV_UNROLL; u++)
        wbuf[u] = (n_ok && u < nk) ? __ldg(reinterpret_cast<const uint4*>(wptr(kb0 + u))) : make_uint4(0, 0, 0, 0);

    asm volatile("griddepcontrol.wait;" ::: "memory");
    // ---- activations of [kb0, kb1) into shared memory: [rows][nk * 128] ----
    const int klen = nk * 128;
    for (int idx = threadIdx.x; idx < rows * (klen / 16); idx += GV_THREADS) {
        const int r = idx / (klen / 16), q = idx % (klen / 16);
        const int pl = r / M, m = r % M;
        const int8_t* src = p.A + pl * p.plane_stride + (size_t)m * p.lda + (size_t)kb0 * 128 + 16 * q;
        *reinterpret_cast<uint4*>(gv_smem + (size_t)r * klen + 16 * q) = *reinterpret_cast<const uint4*>(src);
    }
    __syncthreads();

    int acc[RT];
#pragma unroll
    for (int r = 0; r < RT; r++) acc[r] = 0;
    for (int i = 0; i < nk; i += GV_UNROLL) {
#pragma unroll
        for (int u = 0; u < GV_UNROLL; u++) {
            if (i + u >= nk) break;
            const uint4 w = wbuf[u];
            // the load of the K block GV_UNROLL ahead replaces this one
            if (n_ok && i + u + GV_UNROLL < nk) wbuf[u] = __ldg(reinterpret_cast<const uint4*>(wptr(kb0 + i + u + GV_UNROLL)));
            chunk_dot<WF, RT>(w, gv_smem + (size_t)(i + u) * 128 + c * F::KPC, klen, acc, rows);
        }
    }
    // ---- the CPR lanes of a row hold partial sums of its K range ----
#pragma unroll
    for (int r = 0; r < RT; r++)
#pragma unroll
        for (int o = 1; o < F::CPR; o <<= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
#pragma unroll
    for (int r = 0; r < RT; r++) acc[r] >>= F::SHIFT;  // exact: a multiple of 2^SHIFT
    const int m_act = p.m_dev ? min(M, *p.m_dev) : M;

    if constexpr (EPI == EPI_SWIGLU) {
        // interleaved (gate, up) rows: even rows n take the up sums of row n + 1
        int up[RT];
#pragma unroll
        for (int r = 0; r < RT; r++) up[r] = __shfl_down_sync(0xffffffffu, acc[r], F::CPR);
        if (c != 0 || !n_ok || (n & 1)) return;
        const float wg = p.w_scale ? p.w_scale[n] : 1.0f, wu = p.w_scale ? p.w_scale[n + 1] : 1.0f;
#pragma unroll
        for (int m = 0; m < RT; m++) {
            if (m >= m_act) break;
            const float as = p.a_scale[m];
            const float g = __fmul_rn(__fmul_rn(__int2float_rn(acc[m]), as), wg);
            const float uu = __fmul_rn(__fmul_rn(__int2float_rn(up[m]), as), wu);
            p.out[(size_t)m * p.ldo + (n >> 1)] = engine_swiglu(g, uu);
        }
    } else {
        if (c != 0 || !n_ok) return;
        if constexpr (EPI == EPI_I32) {
            int32_t* o = p.out_i32 + (size_t)blockIdx.y * p.slice_stride;
#pragma unroll
            for (int m = 0; m < RT; m++) {
                if (m >= m_act) break;
                o[(size_t)m * p.ldo + n] = acc[m];
            }
        } else if constexpr (EPI == EPI_F32) {
            const float ws = p.w_scale ? p.w_scale[n] : 1.0f;
#pragma unroll
            for (int m = 0; m < RT; m++) {
                if (m >= m_act) break;
                p.out[(size_t)m * p.ldo + n] = __fmul_rn(__fmul_rn(__int2float_rn(acc[m]), p.a_scale[m]), ws);
            }
        } else {  // EPI_LOGITS3: planes at rows m, M + m, 2M + m
            const float r254 = 1.0f / 254.0f;
#pragma unroll
            for (int m = 0; m < RT / 3; m++) {
                if (m >= m_act) break;
                int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
                for (int r = 0; r < RT; r++) {  // (register arrays need compile-time indices)
                    if (r == m) a0 = acc[r];
                    if (r == M + m) a1 = acc[r];
                    if (r == 2 * M + m) a2 = acc[r];
                }
                const float cmb = __fadd_rn(__int2float_rn(a0),
                                            __fmul_rn(__fadd_rn(__int2float_rn(a1), __fmul_rn(__int2float_rn(a2), r254)), r254));
                p.out[(size_t)m * p.ldo + n] = __fmul_rn(cmb, __fmul_rn(p.a_scale[m], p.w_scale_all));
            }
        }
    }
}

template <int WF, int RT, int EPI, int P>
pf_status launch_gv(const GemmParams& p, int splits, cudaStream_t st) {
    using F = Fmt<WF>;
    const int nkb = p.K / 128;
    const int per = (nkb + splits - 1) / splits;
    const size_t smem = (size_t)P * p.M * per * 128;
    // (the limit is raised once per device, to the largest size any launch uses)
    static std::atomic<uint64_t> attr{0};
    PF_TRY(raise_smem_limit(gemv_kernel<WF, RT, EPI, P>, GV_SMEM_MAX, attr));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ceil_div(p.N, F::RPC), splits);
    cfg.blockDim = dim3(GV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = p.pdl ? 1 : 0;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    PF_CUDA(cudaLaunchKernelEx(&cfg, gemv_kernel<WF, RT, EPI, P>, p));
    return launch_check("gemv");
}

template <int RT, int EPI, int P>
pf_status launch_gv_wf(const GemmParams& p, int splits, cudaStream_t st) {
    switch (p.wf) {
        case WF_Q4: return launch_gv<WF_Q4, RT, EPI, P>(p, splits, st);
        case WF_Q2: return launch_gv<WF_Q2, RT, EPI, P>(p, splits, st);
        default: return launch_gv<WF_I8, RT, EPI, P>(p, splits, st);
    }
}

template <int EPI, int P>
pf_status launch_gv_rt(const GemmParams& p, int splits, cudaStream_t st) {
    const int rows = P * p.M;
    if (rows <= 4) return launch_gv_wf<4, EPI, P>(p, splits, st);
    if (rows <= 8) return launch_gv_wf<8, EPI, P>(p, splits, st);
    if constexpr (P == 3) return launch_gv_wf<15, EPI, P>(p, splits, st);
    else return launch_gv_wf<16, EPI, P>(p, splits, st);
}

}  // namespace

bool gemv_applies(const GemmParams& p, int planes) {
    if (p.M < 1 || planes * p.M > kGemvMaxRows || (planes == 3 && p.M > kGemvMaxRows / 3)) return false;
    const bool slices = p.epi == EPI_I32 && p.slice_stride > 0;
    // the activation rows of a CTA's K range are staged in shared memory
    const int splits = slices ? std::max(1, p.splits) : 1;
    const int per = ceil_div(p.K / 128, splits);
    if ((size_t)planes * p.M * per * 128 > GV_SMEM_MAX) return false;
    if (planes == 1) {
        if (p.epi == EPI_I32) return slices || p.splits <= 1;
        return (p.epi == EPI_F32 || p.epi == EPI_SWIGLU) && p.splits <= 1;
    }
    return p.epi == EPI_LOGITS3 && p.splits <= 1;
}

pf_status gemv_launch(const GemmParams& p, int planes, cudaStream_t st) {
    PF_CHECK(gemv_applies(p, planes), "gemv: shape or epilogue not supported");
    PF_CHECK((reinterpret_cast<uintptr_t>(p.A) & 15) == 0 && p.lda % 16 == 0 && (p.plane_stride % 16) == 0,
             "gemv: activations must be 16-byte aligned");
    const bool slices = p.epi == EPI_I32 && p.slice_stride > 0;
    const int splits = slices ? p.splits : 1;
    PF_CHECK(splits >= 1 && splits <= p.K / 128, "gemv: bad split count");
    PF_CHECK(!slices || p.slice_stride >= (int64_t)p.M * p.ldo, "gemv: slice stride below M * ldo");
    // every split must own at least one K block, since the consumer sums all slices
    const int nkb = p.K / 128, per = (nkb + splits - 1) / splits;
    PF_CHECK((splits - 1) * per < nkb, "gemv: %d splits leave an empty slice of %d K blocks", splits, nkb);
    if (planes == 3) return launch_gv_rt<EPI_LOGITS3, 3>(p, splits, st);
    switch (p.epi) {
        case EPI_I32: return launch_gv_rt<EPI_I32, 1>(p, splits, st);
        case EPI_F32: return launch_gv_rt<EPI_F32, 1>(p, splits, st);
        default: return launch_gv_rt<EPI_SWIGLU, 1>(p, splits, st);
    }
}

}  // namespace pf

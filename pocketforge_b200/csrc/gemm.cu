// gemm.cu — int8 activations x packed int4/int2/int8 weights -> int32, with
// the projection epilogues of the decode step fused in.
//
// Tile 64 (activation rows) x 64 (weight rows) x 128 (k) per stage, 4 warps
// side by side along N (warp tile 64 x 16).  Activations stream through
// shared memory with cp.async (double buffered) and reach the tensor cores
// through ldmatrix; packed weights go straight from global memory into
// registers (one 128-bit load per lane per 8x128 weight group, prefetched a
// stage ahead) and are unpacked with a handful of integer ops.  The integer
// dot products are exact, so split-K partial sums are added with int32
// atomics in any order; the CTA that retires a tile last applies the
// epilogue and leaves the workspace zeroed for the next launch.
#include <cuda_runtime.h>

#include "gemm.cuh"

namespace pf {

namespace {

constexpr int BM = 64, BN = 64, BK = 128, NT = 128;
constexpr int A_STRIDE = BK + 16;  // bytes per smem row: conflict-free ldmatrix

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                            uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma_s8(int32_t (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Sign-extends four 4-bit (resp. 2-bit) fields held in the low bits of each byte.
__device__ __forceinline__ uint32_t sext4(uint32_t y) { return y | ((y & 0x08080808u) * 0x1Eu); }
__device__ __forceinline__ uint32_t sext2(uint32_t y) { return y | ((y & 0x02020202u) * 0x7Eu); }

template <int WF>
struct BChunk;
template <>
struct BChunk<WF_Q4> {
    uint4 v;
    __device__ __forceinline__ void load(const uint8_t* p) { v = __ldg(reinterpret_cast<const uint4*>(p)); }
    __device__ __forceinline__ void frag(int kk, uint32_t& b0, uint32_t& b1) const {
        const uint32_t w = kk == 0 ? v.x : kk == 1 ? v.y : kk == 2 ? v.z : v.w;
        b0 = sext4(w & 0x0F0F0F0Fu);
        b1 = sext4((w >> 4) & 0x0F0F0F0Fu);
    }
};
template <>
struct BChunk<WF_Q2> {
    uint2 v;
    __device__ __forceinline__ void load(const uint8_t* p) { v = __ldg(reinterpret_cast<const uint2*>(p)); }
    __device__ __forceinline__ void frag(int kk, uint32_t& b0, uint32_t& b1) const {
        const uint32_t w = (kk < 2) ? v.x : v.y;
        const int s = (kk & 1) * 4;
        b0 = sext2((w >> s) & 0x03030303u);
        b1 = sext2((w >> (s + 2)) & 0x03030303u);
    }
};
template <>
struct BChunk<WF_I8> {
    uint4 v0, v1;
    __device__ __forceinline__ void load(const uint8_t* p) {
        v0 = __ldg(reinterpret_cast<const uint4*>(p));
        v1 = __ldg(reinterpret_cast<const uint4*>(p) + 1);
    }
    __device__ __forceinline__ void frag(int kk, uint32_t& b0, uint32_t& b1) const {
        switch (kk) {
            case 0: b0 = v0.x; b1 = v0.y; break;
            case 1: b0 = v0.z; b1 = v0.w; break;
            case 2: b0 = v1.x; b1 = v1.y; break;
            default: b0 = v1.z; b1 = v1.w; break;
        }
    }
};

__device__ __forceinline__ float vscale(const GemmParams& p, int32_t acc, int m, int n) {
    const float ws = p.w_scale ? p.w_scale[n] : 1.0f;
    return __fmul_rn(__fmul_rn(__int2float_rn(acc), p.a_scale[m]), ws);
}

template <int NPL>
__device__ __forceinline__ float comb3(const int32_t (&a)[NPL]) {
    if constexpr (NPL == 3) {
        const float r = 1.0f / 254.0f;
        return (float)a[0] + ((float)a[1] + (float)a[2] * r) * r;
    } else {
        return (float)a[0];
    }
}

// Epilogue for the adjacent column pair (n, n+1) of row m.
template <int NPL, int EPI>
__device__ __forceinline__ void epilogue_pair(const GemmParams& p, int m, int n, const int32_t (&a)[NPL],
                                              const int32_t (&b)[NPL]) {
    if constexpr (EPI == EPI_I32) {
        *reinterpret_cast<int2*>(p.out_i32 + (size_t)m * p.ldo + n) = make_int2(a[0], b[0]);
    } else if constexpr (EPI == EPI_F32) {
        *reinterpret_cast<float2*>(p.out + (size_t)m * p.ldo + n) =
            make_float2(vscale(p, a[0], m, n), vscale(p, b[0], m, n + 1));
    } else if constexpr (EPI == EPI_QKV) {
        float x0 = vscale(p, a[0], m, n), x1 = vscale(p, b[0], m, n + 1);
        if (n < p.rope_cols) {  // adjacent-pair rotation (src/engine.cpp:737-748)
            const int i2 = (n % p.head_dim) >> 1;
            const size_t o = (size_t)p.row_pos[m] * (p.head_dim >> 1) + i2;
            const float c = p.rope_cos[o], s = p.rope_sin[o];
            const float r0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
            const float r1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
            x0 = r0;
            x1 = r1;
        }
        *reinterpret_cast<float2*>(p.out + (size_t)m * p.ldo + n) = make_float2(x0, x1);
    } else if constexpr (EPI == EPI_RESID) {
        if (p.row_skip && p.row_skip[m]) return;
        float2* r = reinterpret_cast<float2*>(p.resid + (size_t)m * p.ldo + n);
        float2 x = *r;
        x.x = __fadd_rn(x.x, vscale(p, a[0], m, n));
        x.y = __fadd_rn(x.y, vscale(p, b[0], m, n + 1));
        *r = x;
    } else if constexpr (EPI == EPI_SWIGLU) {
        const float g = vscale(p, a[0], m, n), u = vscale(p, b[0], m, n + 1);
        const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
        p.out[(size_t)m * p.ldo + (n >> 1)] = __fmul_rn(__fmul_rn(g, sig), u);
    } else if constexpr (EPI == EPI_LOGITS3) {
        const float s = p.a_scale[m] * p.w_scale_all;
        *reinterpret_cast<float2*>(p.out + (size_t)m * p.ldo + n) =
            make_float2(comb3<NPL>(a) * s, comb3<NPL>(b) * s);
    } else if constexpr (EPI == EPI_MTP_SWIGLU3) {
        const float g = comb3<NPL>(a) * p.a_scale[m] * p.w_scale[n];
        const float u = comb3<NPL>(b) * p.a_scale[m] * p.w_scale[n + 1];
        p.out[(size_t)m * p.ldo + (n >> 1)] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
    } else if constexpr (EPI == EPI_MTP_RESID3) {
        float2* r = reinterpret_cast<float2*>(p.resid + (size_t)m * p.ldo + n);
        float2 x = *r;
        x.x = __fadd_rn(x.x, comb3<NPL>(a) * p.a_scale[m] * p.w_scale[n]);
        x.y = __fadd_rn(x.y, comb3<NPL>(b) * p.a_scale[m] * p.w_scale[n + 1]);
        *r = x;
    }
}

template <int NPL, int WF, int EPI>
__global__ void __launch_bounds__(NT) gemm_kernel(const GemmParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int m_act = p.m_dev ? min(p.M, *p.m_dev) : p.M;
    if (m0 >= m_act) return;  // uniform over the split-K CTAs of this tile
    const int nkt = p.K / BK;
    const int per = (nkt + p.splits - 1) / p.splits;
    const int kt0 = blockIdx.z * per, kt1 = min(nkt, kt0 + per);

    int32_t acc[NPL][4][2][4];
#pragma unroll
    for (int pl = 0; pl < NPL; pl++)
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 2; j++)
#pragma unroll
                for (int c = 0; c < 4; c++) acc[pl][i][j][c] = 0;

    const uint32_t sbase = smem_u32(smem);
    constexpr int STAGE_BYTES = NPL * BM * A_STRIDE;
    auto load_a = [&](int stage, int kt) {
#pragma unroll
        for (int pl = 0; pl < NPL; pl++)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int chunk = tid + i * NT;
                const int row = chunk >> 3, c16 = chunk & 7;
                const bool ok = (m0 + row) < m_act;
                const int8_t* src = p.A + pl * p.plane_stride + (size_t)(ok ? m0 + row : 0) * p.lda +
                                    (size_t)kt * BK + c16 * 16;
                cp_async16(sbase + stage * STAGE_BYTES + (pl * BM + row) * A_STRIDE + c16 * 16, src, ok);
            }
    };
    const int cgroups = p.K / kPackCols;
    const uint8_t* wbase = reinterpret_cast<const uint8_t*>(p.W);
    const int nt8 = (n0 >> 3) + warp * 2;  // first 8-row weight group of this warp
    auto b_ptr = [&](int j, int kt) {
        return wbase + (((size_t)(nt8 + j) * cgroups + kt) * 32 + lane) * chunk_bytes(WF);
    };

    BChunk<WF> bcur[2], bnext[2];
    if (kt0 < kt1) {
        load_a(0, kt0);
        cp_async_commit();
        bnext[0].load(b_ptr(0, kt0));
        bnext[1].load(b_ptr(1, kt0));
    }
    for (int kt = kt0; kt < kt1; kt++) {
        const int cur = (kt - kt0) & 1;
        bcur[0] = bnext[0];
        bcur[1] = bnext[1];
        if (kt + 1 < kt1) {
            load_a(cur ^ 1, kt + 1);
            cp_async_commit();
            bnext[0].load(b_ptr(0, kt + 1));
            bnext[1].load(b_ptr(1, kt + 1));
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            uint32_t b0[2], b1[2];
            bcur[0].frag(kk, b0[0], b1[0]);
            bcur[1].frag(kk, b0[1], b1[1]);
#pragma unroll
            for (int pl = 0; pl < NPL; pl++)
#pragma unroll
                for (int mt = 0; mt < 4; mt++) {
                    const int row = mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                    const int col = kk * 32 + (lane >> 4) * 16;
                    uint32_t a[4];
                    ldmatrix_x4(sbase + cur * STAGE_BYTES + (pl * BM + row) * A_STRIDE + col, a[0], a[1],
                                a[2], a[3]);
                    mma_s8(acc[pl][mt][0], a, b0[0], b1[0]);
                    mma_s8(acc[pl][mt][1], a, b0[1], b1[1]);
                }
        }
        __syncthreads();
    }

    const int g = lane >> 2, t = lane & 3;
    if (p.splits > 1) {
        // Accumulate this split's partial sums; the last CTA of the tile finishes.
        for (int pl = 0; pl < NPL; pl++)
            for (int mt = 0; mt < 4; mt++)
                for (int j = 0; j < 2; j++)
                    for (int c = 0; c < 4; c++) {
                        const int m = m0 + mt * 16 + g + (c >> 1) * 8;
                        const int n = n0 + warp * 16 + j * 8 + t * 2 + (c & 1);
                        if (m < m_act && acc[pl][mt][j][c] != 0)
                            atomicAdd(p.ws + ((size_t)pl * p.M + m) * p.N + n, acc[pl][mt][j][c]);
                    }
        __threadfence();
        __syncthreads();
        __shared__ int s_last;
        const int tile = blockIdx.y * gridDim.x + blockIdx.x;
        if (tid == 0) s_last = (atomicAdd(p.counters + tile, 1) == p.splits - 1);
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        for (int pl = 0; pl < NPL; pl++)
            for (int mt = 0; mt < 4; mt++)
                for (int j = 0; j < 2; j++)
                    for (int c = 0; c < 4; c++) {
                        const int m = m0 + mt * 16 + g + (c >> 1) * 8;
                        const int n = n0 + warp * 16 + j * 8 + t * 2 + (c & 1);
                        acc[pl][mt][j][c] =
                            (m < m_act) ? atomicExch(p.ws + ((size_t)pl * p.M + m) * p.N + n, 0) : 0;
                    }
        if (tid == 0) p.counters[tile] = 0;
    }
#pragma unroll
    for (int mt = 0; mt < 4; mt++)
#pragma unroll
        for (int j = 0; j < 2; j++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int m = m0 + mt * 16 + g + h * 8;
                if (m >= m_act) continue;
                const int n = n0 + warp * 16 + j * 8 + t * 2;
                int32_t a[NPL], b[NPL];
#pragma unroll
                for (int pl = 0; pl < NPL; pl++) {
                    a[pl] = acc[pl][mt][j][2 * h];
                    b[pl] = acc[pl][mt][j][2 * h + 1];
                }
                epilogue_pair<NPL, EPI>(p, m, n, a, b);
            }
}

template <int NPL, int WF, int EPI>
pf_status launch_t(const GemmParams& p, cudaStream_t st) {
    const int smem = 2 * NPL * BM * A_STRIDE;
    static std::atomic<uint64_t> attr{0};
    PF_TRY(raise_smem_limit(gemm_kernel<NPL, WF, EPI>, smem, attr));
    dim3 grid(p.N / BN, ceil_div(p.M, BM), p.splits);
    gemm_kernel<NPL, WF, EPI><<<grid, NT, smem, st>>>(p);
    return launch_check("gemm");
}

template <int NPL, int EPI>
pf_status launch_wf(const GemmParams& p, cudaStream_t st) {
    switch (p.wf) {
        case WF_Q4: return launch_t<NPL, WF_Q4, EPI>(p, st);
        case WF_Q2: return launch_t<NPL, WF_Q2, EPI>(p, st);
        default: return launch_t<NPL, WF_I8, EPI>(p, st);
    }
}

}  // namespace

size_t gemm_workspace_bytes(int planes, int M, int N) { return (size_t)planes * M * N * sizeof(int32_t); }
size_t gemm_counter_count(int M, int N) { return (size_t)ceil_div(M, BM) * ceil_div(N, BN); }

int gemm_pick_splits(int M, int N, int K, bool have_ws) {
    if (!have_ws) return 1;
    const int tiles = ceil_div(M, BM) * ceil_div(N, BN);
    const int nkt = K / BK;
    int s = ceil_div(2 * 148, tiles);
    s = std::min(s, std::max(1, nkt / 2));
    return std::max(1, std::min(s, 16));
}

pf_status gemm_launch(const GemmParams& p, int planes, cudaStream_t st) {
    PF_CHECK(p.M > 0 && p.N > 0 && p.K > 0, "gemm: empty shape");
    PF_CHECK(p.N % BN == 0, "gemm: N=%d must be a multiple of %d", p.N, BN);
    PF_CHECK(p.K % BK == 0, "gemm: K=%d must be a multiple of %d", p.K, BK);
    PF_CHECK(p.lda % 16 == 0 && p.lda >= p.K, "gemm: lda=%d must be >= K and a multiple of 16", p.lda);
    PF_CHECK(p.splits == 1 || (p.ws && p.counters), "gemm: split-K needs a workspace");
    PF_CHECK(planes == 1 || planes == 3, "gemm: planes must be 1 or 3");
    const bool three = p.epi == EPI_LOGITS3 || p.epi == EPI_MTP_SWIGLU3 || p.epi == EPI_MTP_RESID3;
    PF_CHECK(three == (planes == 3), "gemm: epilogue %d does not take %d planes", p.epi, planes);
    if (planes == 3) {
        switch (p.epi) {
            case EPI_LOGITS3: return launch_wf<3, EPI_LOGITS3>(p, st);
            case EPI_MTP_SWIGLU3: return launch_wf<3, EPI_MTP_SWIGLU3>(p, st);
            default: return launch_wf<3, EPI_MTP_RESID3>(p, st);
        }
    }
    switch (p.epi) {
        case EPI_I32: return launch_wf<1, EPI_I32>(p, st);
        case EPI_F32: return launch_wf<1, EPI_F32>(p, st);
        case EPI_QKV: return launch_wf<1, EPI_QKV>(p, st);
        case EPI_RESID: return launch_wf<1, EPI_RESID>(p, st);
        default: return launch_wf<1, EPI_SWIGLU>(p, st);
    }
}

}  // namespace pf

// rows.cu — row-wise kernels of the decode step: RMSNorm + int8 quantization,
// activation quantization, the 3-digit split of fp32 rows for the exact-int
// tensor-core unembed, embedding gather, argmax, softmax.
//
// One CTA of 256 threads per row; thread t keeps elements t, t+256, ... in
// registers, so each row is read from memory once.  RMSNorm's sum of squares
// uses a fixed order ("device order"): every thread sums its elements in
// sequence, each warp combines its threads with an xor butterfly over offsets
// 16..1, and thread 0 adds the 8 warp totals in warp order.
// oracle/pf_oracle.cpp restates this order (order=1) so the GPU result is
// checked bit for bit, and the reference's sequential order (order=0) within
// tolerance.
#include "common.cuh"
#include "rows.cuh"

namespace pf {

namespace {
constexpr int RT = 256;      // threads per row
constexpr int EPT = 24;      // elements per thread held in registers (n <= 6144)

__device__ __forceinline__ float warp_sum_xor(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// Block sum in the device order; every thread gets the result.  Each warp
// publishes its xor-butterfly total, and after one barrier every thread adds
// the totals itself in warp order (the sequence thread 0 used to add them in,
// so the result is the same).  Sums use sh[0..7], maxima sh[16..23]: a kernel
// may take one of each without a barrier in between.
__device__ __forceinline__ float block_sum(float v, float* sh) {
    v = warp_sum_xor(v);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = sh[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); i++) t = __fadd_rn(t, sh[i]);
    return t;
}
__device__ __forceinline__ float block_max(float v, float* sh) {
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0) sh[16 + (threadIdx.x >> 5)] = v;
    __syncthreads();
    float t = sh[16];
    for (int i = 1; i < (int)(blockDim.x >> 5); i++) t = fmaxf(t, sh[16 + i]);
    return t;
}

// quantize_activation_row (src/matmul_neon.cpp:16-29): mul = 127/amax,
// q = round(x*mul) (half away from zero), scale = amax/127; 1 for zero rows.
__device__ __forceinline__ void row_quant_params(float amax, float& mul, float& scale) {
    mul = (amax == 0.0f) ? 1.0f : __fdiv_rn(127.0f, amax);
    scale = (amax == 0.0f) ? 1.0f : __fdiv_rn(amax, 127.0f);
}
__device__ __forceinline__ int8_t q8(float x, float mul) { return (int8_t)(int)roundf(__fmul_rn(x, mul)); }

__device__ __forceinline__ bool row_active(int row, int M, const int* m_dev) {
    return row < (m_dev ? min(M, *m_dev) : M);
}
}  // namespace

// ---------------------------------------------------------------------------
// RMSNorm (src/matmul_neon.cpp:231-239) fused with the activation quantizer,
// optionally preceded by the residual add of a K-split projection:
//   x += ((float)acc * a_scale[row]) * w_scale[col]   (acc = sum of the int32
//   slices; matmul_quantized's two roundings, src/matmul_neon.cpp:176-180;
//   rows with row_skip set keep x),
// then normed (optional) = RMSNorm(x) * w and q/qs its int8 row and scale.
// Template E = elements per thread (n <= 256 E).  Every load of the row is
// issued before the first use, without branches, so that a row costs one
// memory round trip.
// ---------------------------------------------------------------------------
constexpr int kMaxParts = 4;  // K-split slices summed per element

template <int E>
__global__ void __launch_bounds__(RT) norm_rows_kernel(
    float* __restrict__ x, const int32_t* __restrict__ parts, int n_parts, int64_t part_stride,
    const float* __restrict__ a_s, const float* __restrict__ w_s, const uint8_t* __restrict__ row_skip,
    const float* __restrict__ w, int n, float eps, int M, const int* m_dev, float* __restrict__ normed,
    int8_t* __restrict__ q, float* __restrict__ qs, int ldq) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // lets the next GEMM start its prologue
    __shared__ float sh[33];
    const int row = blockIdx.x, t = threadIdx.x;
    if (!row_active(row, M, m_dev)) return;
    float* xr = x + (size_t)row * n;
    const bool add = n_parts > 0 && !(row_skip && row_skip[row]);
    const int32_t* pr = parts ? parts + (size_t)row * n : nullptr;
    float v[E], wn[E], ws[E];
    int32_t acc[E];
#pragma unroll
    for (int i = 0; i < E; i++) {
        const int c = t + i * RT;
        const bool in = c < n;
        v[i] = in ? xr[c] : 0.0f;
        wn[i] = (in && w) ? w[c] : 0.0f;
        ws[i] = (in && add) ? w_s[c] : 0.0f;
        acc[i] = 0;
#pragma unroll
        for (int s2 = 0; s2 < kMaxParts; s2++) acc[i] += (in && add && s2 < n_parts) ? __ldcg(pr + s2 * part_stride + c) : 0;
    }
    float ss = 0.0f;
    if (add) {
        const float as = a_s[row];
#pragma unroll
        for (int i = 0; i < E; i++) {
            const int c = t + i * RT;
            if (c < n) {
                v[i] = __fadd_rn(v[i], __fmul_rn(__fmul_rn(__int2float_rn(acc[i]), as), ws[i]));
                xr[c] = v[i];
            }
        }
    }
#pragma unroll
    for (int i = 0; i < E; i++) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
    if (!w) return;
    ss = block_sum(ss, sh);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < E; i++) {
        const int c = t + i * RT;
        if (c < n) {
            v[i] = __fmul_rn(__fmul_rn(v[i], inv), wn[i]);
            if (normed) normed[(size_t)row * n + c] = v[i];
            amax = fmaxf(amax, fabsf(v[i]));
        }
    }
    if (!q) return;
    amax = block_max(amax, sh);
    float mul, scale;
    row_quant_params(amax, mul, scale);
#pragma unroll
    for (int i = 0; i < E; i++) {
        const int c = t + i * RT;
        if (c < n) q[(size_t)row * ldq + c] = q8(v[i], mul);
    }
    if (t == 0) qs[row] = scale;
}

static pf_status norm_rows(float* x, const int32_t* parts, int n_parts, int64_t part_stride, const float* a_s,
                           const float* w_s, const uint8_t* row_skip, const float* w, int n, float eps, int M,
                           const int* m_dev, float* normed, int8_t* q, float* qs, int ldq, cudaStream_t st) {
    PF_CHECK(n >= 1 && n <= RT * EPT, "rmsnorm: row length %d outside 1..%d", n, RT * EPT);
    PF_CHECK(!q || w, "rmsnorm: quantization needs the norm weights");
    if (n <= RT * 8)
        norm_rows_kernel<8><<<M, RT, 0, st>>>(x, parts, n_parts, part_stride, a_s, w_s, row_skip, w, n, eps, M, m_dev,
                                              normed, q, qs, ldq);
    else if (n <= RT * 16)
        norm_rows_kernel<16><<<M, RT, 0, st>>>(x, parts, n_parts, part_stride, a_s, w_s, row_skip, w, n, eps, M,
                                               m_dev, normed, q, qs, ldq);
    else
        norm_rows_kernel<EPT><<<M, RT, 0, st>>>(x, parts, n_parts, part_stride, a_s, w_s, row_skip, w, n, eps, M,
                                                m_dev, normed, q, qs, ldq);
    return launch_check("rmsnorm");
}

pf_status rmsnorm_quant(const float* x, const float* w, int n, float eps, int M, const int* m_dev, float* normed,
                        int8_t* q, float* qs, int ldq, cudaStream_t st) {
    PF_CHECK(w, "rmsnorm_quant: norm weights required");
    // x is only read when no slices are given.
    return norm_rows(const_cast<float*>(x), nullptr, 0, 0, nullptr, nullptr, nullptr, w, n, eps, M, m_dev, normed, q,
                     qs, ldq, st);
}

pf_status resid_rmsnorm_quant(float* x, const int32_t* parts, int n_parts, int64_t part_stride, const float* a_s,
                              const float* w_s, const uint8_t* row_skip, const float* w, int n, float eps, int M,
                              float* normed, int8_t* q, float* qs, int ldq, cudaStream_t st) {
    PF_CHECK(n_parts >= 1 && n_parts <= kMaxParts && part_stride >= (int64_t)M * n, "resid_rmsnorm_quant: bad slices");
    return norm_rows(x, parts, n_parts, part_stride, a_s, w_s, row_skip, w, n, eps, M, nullptr, normed, q, qs, ldq,
                     st);
}

// ---------------------------------------------------------------------------
// quantize_activation_row over M rows (any length: rows longer than the
// register cache take a second pass over memory).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(RT) quant_rows_kernel(const float* __restrict__ x, int n, int ldx, int M,
                                                        const int* m_dev, int8_t* __restrict__ q, float* __restrict__ qs,
                                                        int ldq) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // lets the next GEMM start its prologue
    __shared__ float sh[33];
    const int row = blockIdx.x, t = threadIdx.x;
    if (!row_active(row, M, m_dev)) return;
    const float* xr = x + (size_t)row * ldx;
    if ((n & 3) == 0 && (ldx & 3) == 0 && (ldq & 3) == 0 && n <= RT * EPT &&
        ((reinterpret_cast<uintptr_t>(x) & 15) | (reinterpret_cast<uintptr_t>(q) & 3)) == 0) {
        // 16-byte loads and 4-byte stores: thread t owns columns 4 (t + RT i) .. +3
        constexpr int E4 = EPT / 4;
        float4 v4[E4];
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < E4; i++) {
            const int c = 4 * (t + i * RT);
            v4[i] = c < n ? *reinterpret_cast<const float4*>(xr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v4[i].x), fabsf(v4[i].y)), fmaxf(fabsf(v4[i].z), fabsf(v4[i].w))));
        }
        amax = block_max(amax, sh);
        float mul, scale;
        row_quant_params(amax, mul, scale);
        int8_t* qr = q + (size_t)row * ldq;
#pragma unroll
        for (int i = 0; i < E4; i++) {
            const int c = 4 * (t + i * RT);
            if (c < n)
                *reinterpret_cast<char4*>(qr + c) =
                    make_char4(q8(v4[i].x, mul), q8(v4[i].y, mul), q8(v4[i].z, mul), q8(v4[i].w, mul));
        }
        if (t == 0) qs[row] = scale;
        return;
    }
    float v[EPT];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < EPT; i++) {
        const int c = t + i * RT;
        v[i] = c < n ? xr[c] : 0.0f;
        amax = fmaxf(amax, fabsf(v[i]));
    }
    for (int c = t + EPT * RT; c < n; c += RT) amax = fmaxf(amax, fabsf(xr[c]));
    amax = block_max(amax, sh);
    float mul, scale;
    row_quant_params(amax, mul, scale);
    int8_t* qr = q + (size_t)row * ldq;
#pragma unroll
    for (int i = 0; i < EPT; i++) {
        const int c = t + i * RT;
        if (c < n) qr[c] = q8(v[i], mul);
    }
    for (int c = t + EPT * RT; c < n; c += RT) qr[c] = q8(xr[c], mul);
    if (t == 0) qs[row] = scale;
}

pf_status quant_rows(const float* x, int n, int ldx, int M, const int* m_dev, int8_t* q, float* qs, int ldq,
                     cudaStream_t st) {
    quant_rows_kernel<<<M, RT, 0, st>>>(x, n, ldx, M, m_dev, q, qs, ldq);
    return launch_check("quant_rows");
}

// Rows quantized with caller-given scales: q = round(x / s) (the act_scales
// branch of matmul_quantized, src/matmul_neon.cpp:158-164).
__global__ void quant_rows_given_kernel(const float* __restrict__ x, int n, int M, const float* __restrict__ s,
                                        int8_t* __restrict__ q, float* __restrict__ qs, int ldq) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)M * n) return;
    const int row = (int)(i / n), col = (int)(i % n);
    q[(size_t)row * ldq + col] = (int8_t)(int)roundf(__fdiv_rn(x[i], s[row]));
    if (col == 0) qs[row] = s[row];
}

pf_status quant_rows_given(const float* x, int n, int M, const float* s, int8_t* q, float* qs, int ldq,
                           cudaStream_t st) {
    const int64_t tot = (int64_t)M * n;
    quant_rows_given_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, st>>>(x, n, M, s, q, qs, ldq);
    return launch_check("quant_rows_given");
}

// ---------------------------------------------------------------------------
// Three int8 digit planes of an fp32 row: with s = amax/127 and r0 = x*127/amax,
// q1 = rint(r0), q2 = rint((r0-q1)*254), q3 = rint(((r0-q1)*254-q2)*254), so
// x ~= s*(q1 + q2/254 + q3/254^2) to ~2^-23 of amax.  Integer MMAs over the
// planes then reproduce an fp32 dot product to ~1e-7 relative.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(RT) split_digits_kernel(const float* __restrict__ x, int n, int ldx, int M,
                                                          const int* m_dev, int8_t* __restrict__ q, int64_t plane,
                                                          int ldq, float* __restrict__ qs) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // lets the next GEMM start its prologue
    __shared__ float sh[33];
    const int row = blockIdx.x, t = threadIdx.x;
    if (!row_active(row, M, m_dev)) return;
    const float* xr = x + (size_t)row * ldx;
    float v[EPT];
    float amax = 0.0f;
    int bad = 0;  // a NaN or inf in this thread's part of the row (fmaxf drops NaN)
#pragma unroll
    for (int i = 0; i < EPT; i++) {
        const int c = t + i * RT;
        v[i] = c < n ? xr[c] : 0.0f;
        amax = fmaxf(amax, fabsf(v[i]));
        bad |= !isfinite(v[i]);
    }
    amax = block_max(amax, sh);
    if (__syncthreads_or(bad)) amax = __int_as_float(0x7fc00000);
    const float mul = (amax == 0.0f || !isfinite(amax)) ? 0.0f : __fdiv_rn(127.0f, amax);
#pragma unroll
    for (int i = 0; i < EPT; i++) {
        const int c = t + i * RT;
        if (c >= n) continue;
        const float r0 = __fmul_rn(v[i], mul);
        const float d1 = rintf(r0);
        const float r1 = __fmul_rn(__fsub_rn(r0, d1), 254.0f);
        const float d2 = rintf(r1);
        const float r2 = __fmul_rn(__fsub_rn(r1, d2), 254.0f);
        const float d3 = fminf(127.0f, fmaxf(-127.0f, rintf(r2)));
        const size_t o = (size_t)row * ldq + c;
        q[o] = (int8_t)(int)d1;
        q[o + plane] = (int8_t)(int)d2;
        q[o + 2 * plane] = (int8_t)(int)d3;
    }
    // A row that overflowed float range gives NaN products, as the reference's
    // fp32 dot products over it do (inf * 0 and inf - inf terms).
    if (t == 0) qs[row] = !isfinite(amax) ? __int_as_float(0x7fc00000) : (amax == 0.0f) ? 1.0f : __fdiv_rn(amax, 127.0f);
}

pf_status split_digits(const float* x, int n, int ldx, int M, const int* m_dev, int8_t* q, int64_t plane,
                       int ldq, float* qs, cudaStream_t st) {
    PF_CHECK(n <= RT * EPT, "split_digits: row length %d above %d", n, RT * EPT);
    split_digits_kernel<<<M, RT, 0, st>>>(x, n, ldx, M, m_dev, q, plane, ldq, qs);
    return launch_check("split_digits");
}

// ---------------------------------------------------------------------------
// An MTP head's projection from K-split int32 slices of the digit-plane rows
// stacked along M ([parts][3 M][N]: rows m, M + m, 2 M + m are the planes of
// row m), with the GEMM epilogue's arithmetic (comb3 of the exact plane sums,
// * a_scale[m] * w_scale[col]), then the three digit planes of the result row
// (as split_digits) for the next projection:
//   SWIGLU: N = 2 d interleaved (gate, up) columns -> act = mtp_swiglu(g, u)
//   RESID : N = d, x[m] += value (the residual of the head, updated in place)
// a_s and qs may be the same array (each row reads its scale first).
// ---------------------------------------------------------------------------
constexpr int kMtpMaxParts = 4;

template <bool SWIGLU>
__global__ void __launch_bounds__(RT) mtp_finish_kernel(const int32_t* __restrict__ parts, int n_parts,
                                                        int64_t part_stride, const float* a_s,
                                                        const float* __restrict__ w_s, int d, int M,
                                                        float* __restrict__ x, int8_t* __restrict__ q, float* qs,
                                                        int8_t* __restrict__ q2, int64_t plane2, float* qs2) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // lets the next GEMM start its prologue
    __shared__ float sh[33];
    const int row = blockIdx.x, t = threadIdx.x;
    if (row >= M) return;
    constexpr int E = 8;  // d <= 2048
    const int N = SWIGLU ? 2 * d : d;
    const float as = a_s[row];
    // every load first: the three planes' slices of this thread's columns
    int32_t acc[E][3][SWIGLU ? 2 : 1];
    float ws[E][SWIGLU ? 2 : 1], xr[E];
#pragma unroll
    for (int i = 0; i < E; i++) {
        const int c = t + i * RT;
        const bool in = c < d;
        xr[i] = (!SWIGLU && in) ? x[(size_t)row * d + c] : 0.0f;
#pragma unroll
        for (int p = 0; p < 3; p++) {
            const size_t base = ((size_t)p * M + row) * N;
            if constexpr (SWIGLU) {
                acc[i][p][0] = acc[i][p][1] = 0;
#pragma unroll
                for (int s2 = 0; s2 < kMtpMaxParts; s2++) {
                    const int2 v = (in && s2 < n_parts)
                                       ? __ldcg(reinterpret_cast<const int2*>(parts + s2 * part_stride + base + 2 * c))
                                       : make_int2(0, 0);
                    acc[i][p][0] += v.x;
                    acc[i][p][1] += v.y;
                }
            } else {
                acc[i][p][0] = 0;
#pragma unroll
                for (int s2 = 0; s2 < kMtpMaxParts; s2++)
                    acc[i][p][0] += (in && s2 < n_parts) ? __ldcg(parts + s2 * part_stride + base + c) : 0;
            }
        }
        if constexpr (SWIGLU) {
            const float2 w2 = in ? *reinterpret_cast<const float2*>(w_s + 2 * c) : make_float2(0.f, 0.f);
            ws[i][0] = w2.x;
            ws[i][1] = w2.y;
        } else {
            ws[i][0] = in ? w_s[c] : 0.0f;
        }
    }
    const float r = 1.0f / 254.0f;
    auto comb3 = [&](int32_t a0, int32_t a1, int32_t a2) {
        return __fadd_rn(__int2float_rn(a0), __fmul_rn(__fadd_rn(__int2float_rn(a1), __fmul_rn(__int2float_rn(a2), r)), r));
    };
    float v[E];
    float amax = 0.0f;
    int bad = 0;  // a NaN or inf in this thread's columns (fmaxf drops NaN)
#pragma unroll
    for (int i = 0; i < E; i++) {
        const int c = t + i * RT;
        v[i] = 0.0f;
        if (c >= d) continue;
        // The two scales are multiplied first: the chained heads can grow the
        // hidden state to ~1e35, where sum * a_scale alone would overflow
        // although the product with the (small) weight scale is finite, as
        // the reference's float dot product of h with the dequantized row is.
        if constexpr (SWIGLU) {
            const float g = __fmul_rn(comb3(acc[i][0][0], acc[i][1][0], acc[i][2][0]), __fmul_rn(as, ws[i][0]));
            const float u = __fmul_rn(comb3(acc[i][0][1], acc[i][1][1], acc[i][2][1]), __fmul_rn(as, ws[i][1]));
            v[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);  // the GEMM epilogue's mtp_swiglu
        } else {
            v[i] = __fadd_rn(xr[i], __fmul_rn(comb3(acc[i][0][0], acc[i][1][0], acc[i][2][0]), __fmul_rn(as, ws[i][0])));
            x[(size_t)row * d + c] = v[i];
        }
        amax = fmaxf(amax, fabsf(v[i]));
        bad |= !isfinite(v[i]);
    }
    // digit planes of the row, as split_digits_kernel; a row holding NaN or
    // inf gets a NaN scale, so every product over it is NaN, as the
    // reference's float dot products over such a row are
    amax = block_max(amax, sh);
    if (__syncthreads_or(bad)) amax = __int_as_float(0x7fc00000);
    const float mul = (amax == 0.0f || !isfinite(amax)) ? 0.0f : __fdiv_rn(127.0f, amax);
    const size_t plane = (size_t)M * d;
#pragma unroll
    for (int i = 0; i < E; i++) {
        const int c = t + i * RT;
        if (c >= d) continue;
        const float r0 = __fmul_rn(v[i], mul);
        const float d1 = rintf(r0);
        const float r1 = __fmul_rn(__fsub_rn(r0, d1), 254.0f);
        const float d2 = rintf(r1);
        const float r2 = __fmul_rn(__fsub_rn(r1, d2), 254.0f);
        const float d3 = fminf(127.0f, fmaxf(-127.0f, rintf(r2)));
        const size_t o = (size_t)row * d + c;
        q[o] = (int8_t)(int)d1;
        q[o + plane] = (int8_t)(int)d2;
        q[o + 2 * plane] = (int8_t)(int)d3;
        if (q2) {
            q2[o] = (int8_t)(int)d1;
            q2[o + plane2] = (int8_t)(int)d2;
            q2[o + 2 * plane2] = (int8_t)(int)d3;
        }
    }
    if (t == 0) {
        const float sc = !isfinite(amax) ? __int_as_float(0x7fc00000) : (amax == 0.0f) ? 1.0f : __fdiv_rn(amax, 127.0f);
        qs[row] = sc;
        if (qs2) qs2[row] = sc;
    }
}

pf_status mtp_finish(bool swiglu, const int32_t* parts, int n_parts, int64_t part_stride, const float* a_s,
                     const float* w_s, int d, int M, float* x, int8_t* q, float* qs, cudaStream_t st, int8_t* q2,
                     int64_t plane2, float* qs2) {
    PF_CHECK(!q2 || (qs2 && plane2 >= (int64_t)M * d), "mtp_finish: bad second copy");
    PF_CHECK(d <= RT * 8, "mtp_finish: row length %d above %d", d, RT * 8);
    PF_CHECK(n_parts >= 1 && n_parts <= kMtpMaxParts &&
                 part_stride >= (int64_t)3 * M * (swiglu ? 2 * d : d),
             "mtp_finish: bad slices");
    PF_CHECK(swiglu || x, "mtp_finish: the residual form needs x");
    if (swiglu)
        mtp_finish_kernel<true><<<M, RT, 0, st>>>(parts, n_parts, part_stride, a_s, w_s, d, M, x, q, qs, q2, plane2,
                                                  qs2);
    else
        mtp_finish_kernel<false><<<M, RT, 0, st>>>(parts, n_parts, part_stride, a_s, w_s, d, M, x, q, qs, q2, plane2,
                                                   qs2);
    return launch_check("mtp_finish");
}

// ---------------------------------------------------------------------------
// Tied embedding gather (src/engine.cpp:476-484): x = E[token] * global_scale,
// zeros for ids outside [0, n_vocab).
// ---------------------------------------------------------------------------
__global__ void embed_kernel(const int8_t* __restrict__ emb, float gscale, int d, int V, const int* __restrict__ tok,
                             int M, const int* m_dev, float* __restrict__ x) {
    const int row = blockIdx.x;
    const int m_act = m_dev ? min(M, *m_dev) : M;
    if (row >= m_act) return;
    const int t = tok[row];
    const bool ok = t >= 0 && t < V;
    for (int i = threadIdx.x; i < d; i += blockDim.x)
        x[(size_t)row * d + i] = ok ? __fmul_rn((float)emb[(size_t)t * d + i], gscale) : 0.0f;
}

pf_status embed(const int8_t* emb, float gscale, int d, int V, const int* tok, int M, const int* m_dev, float* x,
                cudaStream_t st) {
    embed_kernel<<<M, 256, 0, st>>>(emb, gscale, d, V, tok, M, m_dev, x);
    return launch_check("embed");
}

// ---------------------------------------------------------------------------
// argmax with the first-maximum rule (strict >, src/engine.cpp:918-928).
// ---------------------------------------------------------------------------
__global__ void argmax_kernel(const float* __restrict__ v, int n, int ld, int M, const int* m_dev,
                              int* __restrict__ out) {
    const int row = blockIdx.x;
    const int m_act = m_dev ? min(M, *m_dev) : M;
    if (row >= m_act) return;
    const float* r = v + (size_t)row * ld;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    auto take = [&](float x, int i) {
        if (x > best) {  // ascending scan: earlier index wins ties within a thread
            best = x;
            bi = i;
        }
    };
    int done = 0;
    if (((ld | n) & 3) == 0 && (reinterpret_cast<uintptr_t>(v) & 15) == 0) {
        // 16-byte loads, four in flight per thread before any comparison.
        const float4* r4 = reinterpret_cast<const float4*>(r);
        const int n4 = n >> 2;
        constexpr int U = 4;
        for (int b = threadIdx.x; b < n4; b += U * blockDim.x) {
            float4 x[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int j = b + u * blockDim.x;
                x[u] = j < n4 ? r4[j] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int i = 4 * (b + u * blockDim.x);
                take(x[u].x, i);
                take(x[u].y, i + 1);
                take(x[u].z, i + 2);
                take(x[u].w, i + 3);
            }
        }
        done = n;
    }
    for (int i = done + threadIdx.x; i < n; i += blockDim.x) take(r[i], i);
    for (int o = 16; o >= 1; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) {
            best = ob;
            bi = oi;
        }
    }
    __shared__ float sb[32];
    __shared__ int si[32];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sb[w] = best;
        si[w] = bi;
    }
    __syncthreads();
    if (w == 0) {
        const int nw = blockDim.x >> 5;
        best = lane < nw ? sb[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : 0x7fffffff;
        for (int o = 16; o >= 1; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ob > best || (ob == best && oi < bi)) {
                best = ob;
                bi = oi;
            }
        }
        // All -inf / NaN rows: the reference returns index 0.
        if (lane == 0) out[row] = (bi == 0x7fffffff) ? 0 : bi;
    }
}

pf_status argmax_rows(const float* v, int n, int ld, int M, const int* m_dev, int* out, cudaStream_t st) {
    argmax_kernel<<<M, 256, 0, st>>>(v, n, ld, M, m_dev, out);
    return launch_check("argmax");
}

// ---------------------------------------------------------------------------
// Reference-interface helpers (kernel-level C ABI only).
// ---------------------------------------------------------------------------
// forge::rmsnorm over rows of any length, in the device order of rmsnorm_quant.
__global__ void __launch_bounds__(RT) rmsnorm_rows_kernel(float* __restrict__ out, const float* __restrict__ x,
                                                          const float* __restrict__ w, int M, int n) {
    __shared__ float sh[33];
    const int row = blockIdx.x, t = threadIdx.x;
    if (row >= M) return;
    const float* xr = x + (size_t)row * n;
    float ss = 0.0f;
    for (int c = t; c < n; c += RT) ss = __fadd_rn(ss, __fmul_rn(xr[c], xr[c]));
    ss = block_sum(ss, sh);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), 1e-6f)));
    for (int c = t; c < n; c += RT) out[(size_t)row * n + c] = __fmul_rn(__fmul_rn(xr[c], inv), w[c]);
}

pf_status rmsnorm_rows(float* out, const float* x, const float* w, int M, int n, cudaStream_t st) {
    rmsnorm_rows_kernel<<<M, RT, 0, st>>>(out, x, w, M, n);
    return launch_check("rmsnorm_rows");
}

__global__ void softmax_rows_kernel(float* __restrict__ v, int M, int n) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= M) return;
    float* r = v + (size_t)row * n;
    float mx = -INFINITY;
    for (int i = lane; i < n; i += 32) mx = fmaxf(mx, r[i]);
    mx = warp_max(mx);
    float s = 0.0f;
    for (int i = lane; i < n; i += 32) {
        const float e = expf(__fsub_rn(r[i], mx));
        r[i] = e;
        s = __fadd_rn(s, e);
    }
    s = warp_sum_xor(s);
    const float inv = __fdiv_rn(1.0f, __fadd_rn(s, 1e-10f));
    for (int i = lane; i < n; i += 32) r[i] = __fmul_rn(r[i], inv);
}

pf_status softmax_rows(float* v, int M, int n, cudaStream_t st) {
    softmax_rows_kernel<<<ceil_div(M, 4), 128, 0, st>>>(v, M, n);
    return launch_check("softmax_rows");
}

}  // namespace pf

// gemm.cuh — int8 x packed-weight GEMM with fused epilogues.
#pragma once
#include "common.cuh"

namespace pf {

// Epilogues.  `v(n)` below is ((float)acc * a_scale[m]) * w_scale[n], the two
// roundings of matmul_quantized (src/matmul_neon.cpp:176-180).  The 3-plane
// forms combine an fp32 activation split into three int8 digit planes
// (see split_digits in rows.cu): acc = c1 + (c2 + c3/254)/254.
enum Epi : int {
    EPI_I32 = 0,        // out_i32[m][n] = acc                                (matmul_int8)
    EPI_F32 = 1,        // out[m][n] = v(n)                                   (matmul_quantized)
    EPI_QKV = 2,        // out[m][n] = v(n), RoPE on column pairs n < rope_cols
    EPI_RESID = 3,      // resid[m][n] += v(n) unless row_skip[m]
    EPI_SWIGLU = 4,     // out[m][n/2] = g*(1/(1+exp(-g)))*u, g=v(n), u=v(n+1) (engine FFN)
    EPI_LOGITS3 = 5,    // out[m][n] = comb * a_scale[m] * w_scale_all       (tied unembed)
    EPI_MTP_SWIGLU3 = 6,// out[m][n/2] = (g/(1+exp(-g)))*u over comb forms      (MTP head FFN)
    EPI_MTP_RESID3 = 7  // resid[m][n] += comb * a_scale[m] * w_scale[n]      (MTP down + residual)
};

struct GemmParams {
    const int8_t* A = nullptr;  // planes of [M][lda] int8
    int64_t plane_stride = 0;   // elements between digit planes
    int lda = 0;
    const float* a_scale = nullptr;  // [M]
    const int* m_dev = nullptr;      // optional: rows >= *m_dev are inactive
    int M = 0, N = 0, K = 0;
    const void* W = nullptr;  // packed weights (pack.cu layout), N x K
    int wf = WF_Q4;
    const float* w_scale = nullptr;  // [N]; nullptr = 1
    float w_scale_all = 1.0f;
    int epi = EPI_F32;
    float* out = nullptr;
    int ldo = 0;
    int32_t* out_i32 = nullptr;
    float* resid = nullptr;
    const uint8_t* row_skip = nullptr;
    const float* rope_cos = nullptr;  // [pos][head_dim/2]
    const float* rope_sin = nullptr;
    const int* row_pos = nullptr;     // [M]
    int rope_cols = 0, head_dim = 64;
    int splits = 1;          // gemm_tc_launch: 0 = choose automatically
    int32_t* ws = nullptr;  // split-K workspace, zero on entry, left zero on exit
    int* counters = nullptr;
    size_t ws_elems = 0, cnt_elems = 0;  // capacities of ws / counters
    bool pdl = false;        // gemm_tc_launch: programmatic dependent launch
    // gemm_tc_launch with EPI_I32: > 0 splits K over `splits` CTAs per tile,
    // each writing its int32 partial tile to out_i32 + split * slice_stride
    // (no reduction; the consumer sums the slices).
    int64_t slice_stride = 0;
};

// Scratch needed by a split-K launch (bytes of int32 workspace, counters).
size_t gemm_workspace_bytes(int planes, int M, int N);
size_t gemm_counter_count(int M, int N);
// Chooses the split count for a shape (1 when no workspace is given).
int gemm_pick_splits(int M, int N, int K, bool have_ws);
// Launches the GEMM; planes = 1 or 3 (EPI_*3 use 3).
pf_status gemm_launch(const GemmParams& p, int planes, cudaStream_t st);

}  // namespace pf

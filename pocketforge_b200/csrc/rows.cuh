// rows.cuh — row-wise kernels (rows.cu) and the step kernels (attention.cu,
// accept.cu) used by the engine and the kernel-level C ABI.
#pragma once
#include "common.cuh"

namespace pf {

pf_status pack_weights(const int8_t* w, int rows, int cols, int wf, void* packed, cudaStream_t st);
pf_status dequant_ref(const uint8_t* src, int8_t* dst, int64_t n, int kind, cudaStream_t st);

pf_status rmsnorm_quant(const float* x, const float* w, int n, float eps, int M, const int* m_dev, float* normed,
                        int8_t* q, float* qs, int ldq, cudaStream_t st);
// x[M][n] += sum of n_parts int32 slices (part_stride apart) * a_s[row] * w_s[col]
// (rows with row_skip set unchanged), then, if w, RMSNorm + quantization.
pf_status resid_rmsnorm_quant(float* x, const int32_t* parts, int n_parts, int64_t part_stride, const float* a_s,
                              const float* w_s, const uint8_t* row_skip, const float* w, int n, float eps, int M,
                              float* normed, int8_t* q, float* qs, int ldq, cudaStream_t st);
pf_status quant_rows(const float* x, int n, int ldx, int M, const int* m_dev, int8_t* q, float* qs, int ldq,
                     cudaStream_t st);
pf_status quant_rows_given(const float* x, int n, int M, const float* s, int8_t* q, float* qs, int ldq,
                           cudaStream_t st);
// An MTP head projection's finish from K-split slices of its stacked digit-plane
// rows ([parts][3 M][N]): the GEMM epilogue's arithmetic (SwiGLU over (gate, up)
// column pairs, N = 2 d; or the residual x += value, N = d), then the three
// digit planes of the resulting rows into q ([3][M][d]) and qs, and, if q2 is
// given, a second copy into q2 (planes plane2 apart) and qs2.
pf_status mtp_finish(bool swiglu, const int32_t* parts, int n_parts, int64_t part_stride, const float* a_s,
                     const float* w_s, int d, int M, float* x, int8_t* q, float* qs, cudaStream_t st,
                     int8_t* q2 = nullptr, int64_t plane2 = 0, float* qs2 = nullptr);
pf_status split_digits(const float* x, int n, int ldx, int M, const int* m_dev, int8_t* q, int64_t plane,
                       int ldq, float* qs, cudaStream_t st);
pf_status embed(const int8_t* emb, float gscale, int d, int V, const int* tok, int M, const int* m_dev, float* x,
                cudaStream_t st);
pf_status argmax_rows(const float* v, int n, int ld, int M, const int* m_dev, int* out, cudaStream_t st);
pf_status rmsnorm_rows(float* out, const float* x, const float* w, int M, int n, cudaStream_t st);
pf_status softmax_rows(float* v, int M, int n, cudaStream_t st);

}  // namespace pf

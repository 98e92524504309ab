// forge/matmul_neon.hpp — the reference's matrix free functions
// (include/forge/matmul_neon.hpp:20-92 there), executed on the GPU.
//
// Same signatures and meaning: caller-owned HOST buffers in and out.  Each
// call copies its inputs to the device, runs the sm_100a kernel of
// libpf_b200 (include/pf_b200.h) and copies the result back, synchronously.
// Integer results are the reference's bit for bit; float results follow the
// reference's formulas.  There is no CPU path: without an sm_100 device the
// calls print the library error and leave the outputs untouched.
#ifndef FORGE_B200_MATMUL_NEON_HPP
#define FORGE_B200_MATMUL_NEON_HPP

#include <cstdint>
#include <vector>

#include "types.hpp"

namespace forge {

FORGE_API void quantize_activation_row(const float* src, int8_t* dst, float* scale_out, uint32_t n);
FORGE_API void dequant_q4_to_int8(const uint8_t* q4_data, int8_t* i8_data, float scale, uint32_t n);
FORGE_API void dequant_q2_to_int8(const uint8_t* q2_data, int8_t* i8_data, float scale, uint32_t n);
FORGE_API void dequant_ternary_to_int8(const uint8_t* t_data, int8_t* i8_data, uint32_t n);
// C[M][N] = A[M][K] . B[N][K]^T, int8 in, int32 out.
FORGE_API void matmul_int8(const int8_t* A, const int8_t* B, int32_t* C, uint32_t M, uint32_t N, uint32_t K);
// Quantize A per row, int8 GEMM, C = ((float)acc * a_scale) * w_scale.
FORGE_API void matmul_quantized(const float* A, const int8_t* B, float* C, uint32_t M, uint32_t N, uint32_t K,
                                const float* weight_scales, const float* act_scales);
FORGE_API float dot_product(const float* a, const float* b, uint32_t n);
FORGE_API void softmax(float* vals, uint32_t n);
FORGE_API void rmsnorm(float* out, const float* x, const float* weight, uint32_t n);

}  // namespace forge

#endif  // FORGE_B200_MATMUL_NEON_HPP

// numerics.cuh — branch-free device arithmetic with exactly specified results.
#pragma once
#include <cuda_runtime.h>

namespace pf {

// Correctly rounded 1 / x (round to nearest even) for float x >= 1 (finite or
// +inf; NaN propagates), without a data-dependent branch, so that many of
// them can be interleaved by the compiler (the IEEE division and reciprocal
// routines take a per-element branch to a slow path).
//
// Method: Newton-Raphson iteration for the reciprocal in double precision,
// y <- y + y (1 - x y) with fused multiply-adds, twice from the hardware's
// double reciprocal approximation (relative error below 2^-20, so the
// result's error is below 2^-52), then one rounding to float.  That rounding
// is the correct one: 1/x is never within 2^-49 (relative) of a midpoint of
// two floats — x * m = 1 for a float x and a midpoint m would need an odd
// 25-bit integer times a 24-bit integer to be a power of two — so an
// approximation that close rounds to the same float as 1/x itself.
// Verified against __frcp_rn for every float in [1, inf] by a GPU test.
__device__ __forceinline__ float recip_rn_ge1(float x) {
    const double xd = (double)x;
    double y;
    asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(y) : "d"(xd));
    double e = __fma_rn(-xd, y, 1.0);
    y = __fma_rn(y, e, y);
    e = __fma_rn(-xd, y, 1.0);
    y = __fma_rn(y, e, y);
    const float r = __double2float_rn(y);
    return x == __int_as_float(0x7f800000) ? 0.0f : r;  // 1 / inf (the iteration gives NaN there)
}

// The engine's FFN activation g * (1 / (1 + exp(-g))) * u with the float
// roundings of src/engine.cpp:834-838.
__device__ __forceinline__ float engine_swiglu_rn(float g, float u) {
    const float sig = recip_rn_ge1(__fadd_rn(1.0f, expf(-g)));
    return __fmul_rn(__fmul_rn(g, sig), u);
}

}  // namespace pf

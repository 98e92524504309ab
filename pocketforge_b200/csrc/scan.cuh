// scan.cuh — the reference's sequential float sums, reproduced exactly by one
// warp (the sampler's normalising sum and cumulative scan, src/engine.cpp:
// 895-1003).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace pf {

// The reference's cumulative float sum of a[0, n) in index order (terms
// >= 0), continuing from cum, computed exactly by one warp.  Returns the first
// i whose partial sum c satisfies stop(c) (cum is then that sum), else n (cum
// is the full sum); stop must be monotone in c.
//
// While the running sum c lies in one binade [2^E, 2^(E+1)), every addition
// lands on the grid g = 2^(E-23): with c = R g (R an integer in [2^23, 2^24))
// and t / g = a + f (a an integer, 0 <= f < 1), the rounded sum is (R + a) g
// for f < 1/2, (R + a + 1) g for f > 1/2, and the even one of the two for
// f = 1/2.  As a map of R: R -> R + alpha + beta (R mod 2), with alpha = a or
// a + 1 and beta = 0 off ties; a tie gives (a, 1) for even a and (a + 1, -1)
// for odd a.  The maps compose: (alpha1, beta1) followed by (alpha2, beta2) is
//   (alpha1 + alpha2 + beta2 (alpha1 mod 2),
//    beta1 != 0 ? beta1 : beta2 (1 - 2 (alpha1 mod 2)))
// (after a map with beta != 0 the parity of R is that of alpha, whatever R
// was).  A window of 512 terms is 16 consecutive terms per lane: each lane
// composes its own, a warp scan composes the lanes, and every partial sum of
// the window follows exactly; the lane whose run holds the first event walks
// it term by term.  The first addition whose sum would leave the
// binade (or whose term is not finite) is done as a float addition, and the
// next window starts after it.  While the sum is zero, below 2^-100 or not
// finite, lane 0 adds the terms one at a time (as the reference does), and a
// NaN sum ends the scan.
//
// DESC: the terms never increase (sorted rows).  Then once a term is below a
// quarter of the spacing of floats above the sum, every later term rounds
// away (RN(c + q) = c for 0 <= q < ulp(c)/2; the factor 2 of margin covers a
// term one float step above its predecessor, the double exp being within an
// ulp but not guaranteed monotone): the sum is final and a stop that has not
// held cannot start to, so the scan ends with the result of the full walk.
__device__ __forceinline__ float quarter_ulp(float c) {  // c >= 0; 0 when too small to matter
    const uint32_t e = __float_as_uint(c) >> 23;
    return e >= 26 ? __uint_as_float((e - 25) << 23) : 0.0f;
}
constexpr int kWinPer = 16;         // terms per lane and window
constexpr int kMapCap = 1 << 26;    // alpha saturates here (only past the end of a binade)
struct GridMap {
    int a, b;
};
__device__ __forceinline__ GridMap map_then(GridMap p, GridMap q) {
    const int par = p.a & 1;
    return GridMap{min(p.a + q.a + (par ? q.b : 0), kMapCap), p.b != 0 ? p.b : (par ? -q.b : q.b)};
}
__device__ __forceinline__ int map_apply(GridMap p, int R) { return R + p.a + ((R & 1) ? p.b : 0); }
// Adding t >= 0 on the grid 2^-k, mult = 2^k: t * mult is exact (a
// power-of-two scaling) unless it underflows, and then it is far below 1/2.
__device__ __forceinline__ GridMap map_of(float t, float mult) {
    const float x = __fmul_rn(t, mult);
    if (!(x < 33554432.0f)) return GridMap{kMapCap, 0};  // 2^25: past the binade; inf, NaN
    const int a = (int)x;
    const float f = __fsub_rn(x, (float)a);  // exact
    if (f < 0.5f) return GridMap{a, 0};
    if (f > 0.5f) return GridMap{a + 1, 0};
    return (a & 1) ? GridMap{a + 1, -1} : GridMap{a, 1};
}
// Every lane of one warp calls this; a is 16-byte aligned shared memory.  The
// result and cum are the same in every lane.
template <bool DESC, typename Stop>
__device__ __forceinline__ int ordered_scan_warp(const float* a, int n, float& cum, Stop stop) {
    constexpr unsigned FULL = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const float kMin = __uint_as_float(27u << 23);  // 2^-100
    float c = cum;
    int pos = 0;
    while (pos < n) {
        if (!(c >= kMin && c < INFINITY)) {
            // A sum that is zero, tiny, inf or NaN: lane 0 adds term by term
            // until the sum is in range again.  A NaN sum stays NaN, so a
            // stop that did not hold for it never will.
            int k = n, stopped = 0;
            float cc = c;
            if (lane == 0) {
                for (k = pos; k < n; k++) {
                    cc = __fadd_rn(cc, a[k]);
                    if (stop(cc)) {
                        stopped = 1;
                        break;
                    }
                    if (cc >= kMin && cc < INFINITY) break;
                    if (cc != cc) {
                        k = n;
                        break;
                    }
                }
            }
            k = __shfl_sync(FULL, k, 0);
            c = __shfl_sync(FULL, cc, 0);
            if (__shfl_sync(FULL, stopped, 0) || k >= n) {
                cum = c;
                return k;
            }
            pos = k + 1;
            continue;
        }
        if (DESC && a[pos] < quarter_ulp(c)) {
            cum = c;
            return n;
        }
        const int E = (int)((__float_as_uint(c) >> 23) & 0xFF) - 127;  // -100 <= E <= 127
        const float g = __uint_as_float((uint32_t)(E + 104) << 23);      // 2^(E-23)
        const float mult = __uint_as_float((uint32_t)(150 - E) << 23);   // 2^(23-E)
        const int R = (int)__fmul_rn(c, mult);
        const int ws = pos & ~3;  // 16-byte aligned window start; terms before pos add nothing
        const int base = ws + kWinPer * lane;
        float t[kWinPer];
#pragma unroll
        for (int q = 0; q < kWinPer / 4; q++) {
            const int i = base + 4 * q;
            float4 v;
            if (i + 3 < n) {
                v = *reinterpret_cast<const float4*>(a + i);
            } else {
                v.x = i < n ? a[i] : 0.0f;
                v.y = i + 1 < n ? a[i + 1] : 0.0f;
                v.z = i + 2 < n ? a[i + 2] : 0.0f;
                v.w = i + 3 < n ? a[i + 3] : 0.0f;
            }
            t[4 * q] = v.x;
            t[4 * q + 1] = v.y;
            t[4 * q + 2] = v.z;
            t[4 * q + 3] = v.w;
        }
#pragma unroll
        for (int j = 0; j < kWinPer; j++)
            if (base + j < pos) t[j] = 0.0f;
        // this lane's 16 maps composed as a tree (depth 4, not a chain of 16)
        GridMap m[kWinPer];
#pragma unroll
        for (int j = 0; j < kWinPer; j++) m[j] = map_of(t[j], mult);
#pragma unroll
        for (int s = 1; s < kWinPer; s <<= 1)
#pragma unroll
            for (int j = 0; j + s < kWinPer; j += 2 * s) m[j] = map_then(m[j], m[j + s]);
        GridMap inc = m[0];  // lanes 0 .. lane
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const GridMap y{__shfl_up_sync(FULL, inc.a, o), __shfl_up_sync(FULL, inc.b, o)};
            if (lane >= o) inc = map_then(y, inc);
        }
        // R and stop are monotone along the window: a lane's run holds the
        // first event (an addition leaving the binade, or the stop) if its
        // last partial sum has one and no earlier lane's does.
        const int r_end = map_apply(inc, R);
        const unsigned hit =
            __ballot_sync(FULL, r_end >= (1 << 24) || stop(__fmul_rn(__int2float_rn(r_end), g)));
        if (hit == 0) {
            c = __fmul_rn(__int2float_rn(__shfl_sync(FULL, r_end, 31)), g);
            pos = ws + 32 * kWinPer;
            continue;
        }
        const int src = __ffs(hit) - 1;
        GridMap exc{__shfl_up_sync(FULL, inc.a, 1), __shfl_up_sync(FULL, inc.b, 1)};
        if (lane == 0) exc = GridMap{0, 0};
        // lane src walks its run to the event
        int ev = kWinPer, rev = 0, evstop = 0;
        if (lane == src) {
            int r = map_apply(exc, R);
#pragma unroll
            for (int j = 0; j < kWinPer; j++) {
                if (ev == kWinPer) {
                    const int rn = map_apply(map_of(t[j], mult), r);
                    if (rn >= (1 << 24)) {
                        ev = j;
                        rev = r;
                    } else if (stop(__fmul_rn(__int2float_rn(rn), g))) {
                        ev = j;
                        rev = rn;
                        evstop = 1;
                    }
                    r = rn;
                }
            }
        }
        const int i = ws + kWinPer * src + __shfl_sync(FULL, ev, src);
        const float cb = __fmul_rn(__int2float_rn(__shfl_sync(FULL, rev, src)), g);
        if (__shfl_sync(FULL, evstop, src)) {
            cum = cb;
            return i;
        }
        c = __fadd_rn(cb, a[i]);  // the addition that leaves the binade
        if (stop(c)) {
            cum = c;
            return i;
        }
        pos = i + 1;
    }
    cum = c;
    return n;
}

// The same sum as a plain one-thread loop (the reference's own form), for the
// self-check of ordered_scan_warp.
template <typename Stop>
__device__ __forceinline__ int ordered_scan_serial(const float* a, int n, float& cum, Stop stop) {
    float c = cum;
    for (int i = 0; i < n; i++) {
        c = __fadd_rn(c, a[i]);
        if (stop(c)) {
            cum = c;
            return i;
        }
    }
    cum = c;
    return n;
}

}  // namespace pf

// selftest.cu — device checks of this library's own arithmetic helpers that
// tests run on the GPU (every input of a range, not samples).
#include "common.cuh"
#include "numerics.cuh"
#include "scan.cuh"

namespace pf {
namespace {

// Every float bit pattern in [lo, hi]: recip_rn_ge1 against the library's
// correctly rounded reciprocal.
__global__ void check_recip_kernel(uint32_t lo, uint32_t hi, unsigned long long* mismatches, uint32_t* first) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    unsigned long long bad = 0;
    for (uint64_t b = lo + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; b <= hi; b += stride) {
        const float x = __uint_as_float((uint32_t)b);
        const uint32_t want = __float_as_uint(__frcp_rn(x)), got = __float_as_uint(recip_rn_ge1(x));
        if (want != got) {
            bad++;
            atomicMin(first, (uint32_t)b);
        }
    }
    if (bad) atomicAdd(mismatches, bad);
}

// One row per CTA of one warp: the warp scan against the one-thread loop,
// for the full sum and for the stop at u <= c || c >= p.  Bit-identical sums
// (both NaN counts as identical) and the same index, or the row counts.
template <bool DESC>
__global__ void check_scan_kernel(const float* __restrict__ terms, int n, const float* __restrict__ u,
                                  const float* __restrict__ p, uint32_t* mismatches) {
    extern __shared__ __align__(16) float row[];
    const int r = blockIdx.x, lane = threadIdx.x;
    for (int i = lane; i < n; i += 32) row[i] = terms[(size_t)r * n + i];
    __syncwarp();
    const float ur = u[r], pr = p[r];
    auto never = [](float) { return false; };
    auto stop = [ur, pr](float c) { return ur <= c || c >= pr; };
    auto same = [](float a, float b) { return __float_as_uint(a) == __float_as_uint(b) || (isnan(a) && isnan(b)); };
    float s_w = 0.0f, s_s = 0.0f, c_w = 0.0f, c_s = 0.0f;
    const int j_w = ordered_scan_warp<DESC>(row, n, s_w, never);
    const int i_w = ordered_scan_warp<DESC>(row, n, c_w, stop);
    if (lane == 0) {
        const int j_s = ordered_scan_serial(row, n, s_s, never);
        const int i_s = ordered_scan_serial(row, n, c_s, stop);
        if (j_w != j_s || !same(s_w, s_s) || i_w != i_s || !same(c_w, c_s)) atomicAdd(mismatches, 1u);
    }
}

}  // namespace
}  // namespace pf

using namespace pf;

extern "C" pf_status pf_check_reciprocal(uint64_t* mismatches, uint32_t* first_bad) {
    PF_TRY(require_device());
    PF_CHECK(mismatches && first_bad, "pf_check_reciprocal: null argument");
    unsigned long long* d_bad = nullptr;
    uint32_t* d_first = nullptr;
    PF_CUDA(cudaMalloc(&d_bad, sizeof(unsigned long long) + sizeof(uint32_t)));
    d_first = reinterpret_cast<uint32_t*>(d_bad + 1);
    const uint32_t init_first = 0xFFFFFFFFu;
    pf_status st = PF_OK;
    if (cudaMemset(d_bad, 0, sizeof(unsigned long long)) != cudaSuccess ||
        cudaMemcpy(d_first, &init_first, sizeof(uint32_t), cudaMemcpyHostToDevice) != cudaSuccess) {
        st = PF_ERR_CUDA;
    } else {
        // [1.0, +inf]: 0x3f800000 .. 0x7f800000
        check_recip_kernel<<<148 * 8, 256>>>(0x3f800000u, 0x7f800000u, d_bad, d_first);
        unsigned long long h_bad = 0;
        if (cudaGetLastError() != cudaSuccess || cudaMemcpy(&h_bad, d_bad, sizeof(h_bad), cudaMemcpyDeviceToHost) != cudaSuccess ||
            cudaMemcpy(first_bad, d_first, sizeof(uint32_t), cudaMemcpyDeviceToHost) != cudaSuccess)
            st = PF_ERR_CUDA;
        *mismatches = h_bad;
    }
    cudaFree(d_bad);
    if (st != PF_OK) set_error("pf_check_reciprocal: CUDA error");
    return st;
}

extern "C" pf_status pf_check_ordered_scan(const float* terms, int32_t rows, int32_t n, int32_t sorted, const float* u,
                                           const float* p, uint32_t* mismatches) {
    PF_TRY(require_device());
    PF_CHECK(terms && u && p && mismatches && rows > 0 && n > 0 && n <= 16384, "pf_check_ordered_scan: bad arguments");
    uint32_t* d_bad = nullptr;
    PF_CUDA(cudaMalloc(&d_bad, sizeof(uint32_t)));
    const size_t smem = (size_t)n * sizeof(float);
    static std::atomic<uint64_t> attr_asc{0}, attr_desc{0};
    pf_status st = sorted ? raise_smem_limit(check_scan_kernel<true>, 16384 * sizeof(float), attr_desc)
                          : raise_smem_limit(check_scan_kernel<false>, 16384 * sizeof(float), attr_asc);
    if (st == PF_OK) {
        if (cudaMemset(d_bad, 0, sizeof(uint32_t)) != cudaSuccess) {
            st = PF_ERR_CUDA;
        } else {
            if (sorted)
                check_scan_kernel<true><<<rows, 32, smem>>>(terms, n, u, p, d_bad);
            else
                check_scan_kernel<false><<<rows, 32, smem>>>(terms, n, u, p, d_bad);
            if (cudaGetLastError() != cudaSuccess ||
                cudaMemcpy(mismatches, d_bad, sizeof(uint32_t), cudaMemcpyDeviceToHost) != cudaSuccess)
                st = PF_ERR_CUDA;
        }
        if (st != PF_OK) set_error("pf_check_ordered_scan: CUDA error");
    }
    cudaFree(d_bad);
    return st;
}

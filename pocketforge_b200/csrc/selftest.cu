// selftest.cu — device checks of this library's own arithmetic helpers that
// tests run on the GPU (every input of a range, not samples).
#include "common.cuh"
#include "numerics.cuh"

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

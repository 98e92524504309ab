// common.cu — error text, device checks and the device error latch.
#include <cstdarg>
#include <mutex>

#include "common.cuh"
#include "gemm_tc.cuh"

namespace pf {

static thread_local char g_err[1024] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

const char* last_error() { return g_err; }

pf_status require_device() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        set_error("no CUDA device visible");
        return PF_ERR_NO_DEVICE;
    }
    int dev = 0, major = 0;
    PF_CUDA(cudaGetDevice(&dev));
    PF_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    if (major != 10) {
        set_error("device %d has compute capability %d.x; this library is built for sm_100a only", dev, major);
        return PF_ERR_NO_DEVICE;
    }
    return PF_OK;
}

pf_status launch_check(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("launch of %s failed: %s", what, cudaGetErrorString(e));
        return PF_ERR_CUDA;
    }
    return PF_OK;
}

// One latch word per device, allocated on first use.
uint32_t* device_error_flag() {
    static std::mutex mu;
    static uint32_t* flags[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!flags[dev]) {
        if (cudaMalloc(&flags[dev], sizeof(uint32_t)) != cudaSuccess) return nullptr;
        cudaMemset(flags[dev], 0, sizeof(uint32_t));
    }
    return flags[dev];
}

}  // namespace pf

extern "C" const char* pf_last_error(void) { return pf::last_error(); }

extern "C" pf_status pf_read_device_error(uint32_t* flags, int32_t clear) {
    PF_TRY(pf::require_device());
    PF_CHECK(flags, "pf_read_device_error: null argument");
    uint32_t* f = pf::device_error_flag();
    PF_CHECK(f, "pf_read_device_error: no error flag on this device");
    PF_CUDA(cudaDeviceSynchronize());
    PF_CUDA(cudaMemcpy(flags, f, 4, cudaMemcpyDeviceToHost));
    if (clear) PF_CUDA(cudaMemset(f, 0, 4));
    return PF_OK;
}

extern "C" int32_t pf_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int c = 0;
    for (int i = 0; i < n; i++) {
        int major = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, i) == cudaSuccess && major == 10) c++;
    }
    return c;
}

extern "C" size_t pf_packed_weight_bytes(int32_t rows, int32_t cols, int32_t qtype) {
    if (rows <= 0 || cols <= 0) return 0;
    return pf::packed_bytes_tc(rows, cols, pf::wfmt_of_qtype(qtype));
}

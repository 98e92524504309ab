// common.cuh — shared helpers for the sm_100a kernels of pocketforge_b200.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdio>
#include <string>

#include "../../include/pf_b200.h"

namespace pf {

// Thread-local last error text (pf_last_error).
void set_error(const char* fmt, ...);
const char* last_error();

#define PF_CUDA(call)                                                                   \
    do {                                                                                \
        cudaError_t _e = (call);                                                        \
        if (_e != cudaSuccess) {                                                        \
            ::pf::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call,                  \
                            cudaGetErrorString(_e));                                    \
            cudaGetLastError(); /* not reported again by the next launch check */       \
            return PF_ERR_CUDA;                                                         \
        }                                                                               \
    } while (0)

#define PF_CHECK(cond, ...)                     \
    do {                                        \
        if (!(cond)) {                          \
            ::pf::set_error(__VA_ARGS__);       \
            return PF_ERR_INVALID;              \
        }                                       \
    } while (0)

#define PF_TRY(expr)                 \
    do {                             \
        pf_status _s = (expr);       \
        if (_s != PF_OK) return _s;  \
    } while (0)

// Fails with PF_ERR_NO_DEVICE unless an sm_100 device is current.
pf_status require_device();
// Returns the launch error of the last kernel, if any.
pf_status launch_check(const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Device-side error latch: kernels set bits here instead of trapping.
enum : uint32_t {
    ERR_BOUNDS = 1u,      // an index was out of the buffer it addresses
    ERR_WEIGHT_RANGE = 2u,// a weight value does not fit its packed format
    ERR_TOKEN = 4u,       // a token id outside [0, n_vocab)
    ERR_CONTEXT = 8u      // a position beyond the cache capacity
};
uint32_t* device_error_flag();  // per-device global (allocated on first use)

// cudaFuncSetAttribute acts on the current device's instance of a kernel, so the
// raised dynamic shared-memory limit (and the shared-memory carveout) is recorded per device: `done` holds one bit
// per device id (< 64; above that the attribute is set on every call).
template <typename Kernel>
inline pf_status raise_smem_limit(Kernel kernel, size_t bytes, std::atomic<uint64_t>& done) {
    int dev = 0;
    PF_CUDA(cudaGetDevice(&dev));
    const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return PF_OK;
    PF_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    // all of the unified L1 / shared array as shared memory, so that as many
    // CTAs as the registers allow fit on an SM
    PF_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared));
    done.fetch_or(bit, std::memory_order_acq_rel);
    return PF_OK;
}

__host__ __device__ inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Packed weight layout (see pack.cu): groups of 8 rows x 128 columns; within a
// group every lane of a warp owns a fixed chunk (Q4 16 B, Q2 8 B, I8 32 B).
enum WFmt : int { WF_I8 = 0, WF_Q4 = 1, WF_Q2 = 2 };
constexpr int kPackRows = 8;
constexpr int kPackCols = 128;
__host__ __device__ inline int chunk_bytes(int wf) { return wf == WF_Q4 ? 16 : (wf == WF_Q2 ? 8 : 32); }
inline size_t packed_bytes(int rows, int cols, int wf) {
    const size_t groups = (size_t)ceil_div(rows, kPackRows) * (size_t)ceil_div(cols, kPackCols);
    return groups * 32u * (size_t)chunk_bytes(wf);
}
// Device format of a reference quantization type.
inline int wfmt_of_qtype(int qt) {
    return qt == PF_QT_Q4 ? WF_Q4 : ((qt == PF_QT_Q2 || qt == PF_QT_Q15) ? WF_Q2 : WF_I8);
}

}  // namespace pf

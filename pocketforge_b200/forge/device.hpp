// device.hpp — helpers of the forge:: compatibility layer: device buffers and
// the error convention of the reference (print to stderr, no exceptions).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <cstdio>

#include "pf_b200.h"

namespace forge {
namespace dev {

// A device allocation that grows on demand and is freed with its owner.
class Buffer {
public:
    Buffer() = default;
    explicit Buffer(size_t bytes) { reserve(bytes); }
    ~Buffer() {
        if (p_) cudaFree(p_);
    }
    Buffer(const Buffer&) = delete;
    Buffer& operator=(const Buffer&) = delete;
    Buffer(Buffer&& o) noexcept : p_(o.p_), cap_(o.cap_) {
        o.p_ = nullptr;
        o.cap_ = 0;
    }
    Buffer& operator=(Buffer&& o) noexcept {
        if (this != &o) {
            if (p_) cudaFree(p_);
            p_ = o.p_;
            cap_ = o.cap_;
            o.p_ = nullptr;
            o.cap_ = 0;
        }
        return *this;
    }
    // Device memory of at least `bytes`; previous contents are not kept.
    void* reserve(size_t bytes) {
        if (bytes > cap_) {
            if (p_) cudaFree(p_);
            p_ = nullptr;
            cap_ = 0;
            if (cudaMalloc(&p_, bytes) != cudaSuccess) {
                cudaGetLastError();
                std::fprintf(stderr, "forge: cudaMalloc of %zu bytes failed\n", bytes);
                p_ = nullptr;
                return nullptr;
            }
            cap_ = bytes;
        }
        return p_;
    }
    template <class T>
    T* as() const { return static_cast<T*>(p_); }
    size_t capacity() const { return cap_; }

private:
    void* p_ = nullptr;
    size_t cap_ = 0;
};

inline bool ok(pf_status s, const char* what) {
    if (s == PF_OK) return true;
    std::fprintf(stderr, "forge::%s: %s\n", what, pf_last_error());
    return false;
}
inline bool cuda_ok(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return true;
    std::fprintf(stderr, "forge::%s: %s\n", what, cudaGetErrorString(e));
    return false;
}
inline bool to_dev(void* d, const void* h, size_t n, const char* what) {
    return n == 0 || cuda_ok(cudaMemcpy(d, h, n, cudaMemcpyHostToDevice), what);
}
inline bool to_host(void* h, const void* d, size_t n, const char* what) {
    return n == 0 || cuda_ok(cudaMemcpy(h, d, n, cudaMemcpyDeviceToHost), what);
}

}  // namespace dev

namespace detail {
// MTPHeads::quantize_q4 of a rows x cols float matrix (src/mtp.cpp:174-197):
// per-row scales amax / 127, two values per byte, low nibble first.
void quantize_q4_rows(const float* src, uint8_t* dst, float* scales, uint32_t rows, uint32_t cols);
}  // namespace detail

}  // namespace forge

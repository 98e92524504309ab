// matmul.cpp — forge:: matrix free functions on the GPU
// (the reference's src/matmul_neon.cpp:16-239 as host-buffer calls).
#include "forge/matmul_neon.hpp"

#include "device.hpp"

namespace forge {
namespace {

// Per-thread staging buffers: inputs a, b, c, output o.
struct Stage {
    dev::Buffer a, b, c, o;
};
Stage& stage() {
    static thread_local Stage s;
    return s;
}

}  // namespace

void quantize_activation_row(const float* src, int8_t* dst, float* scale_out, uint32_t n) {
    Stage& s = stage();
    float* x = static_cast<float*>(s.a.reserve((size_t)n * 4 + 16));
    int8_t* q = static_cast<int8_t*>(s.o.reserve((size_t)n + 16));
    float* sc = static_cast<float*>(s.b.reserve(16));
    if (!x || !q || !sc || !dev::to_dev(x, src, (size_t)n * 4, "quantize_activation_row")) return;
    if (!dev::ok(pf_quantize_activation_rows(x, q, sc, 1, (int32_t)n, nullptr), "quantize_activation_row")) return;
    dev::to_host(dst, q, n, "quantize_activation_row");
    dev::to_host(scale_out, sc, 4, "quantize_activation_row");
}

template <class F>
static void dequant(const uint8_t* src, size_t src_bytes, int8_t* dst, uint32_t n, F run, const char* what) {
    Stage& s = stage();
    uint8_t* d_src = static_cast<uint8_t*>(s.a.reserve(src_bytes + 16));
    int8_t* d_dst = static_cast<int8_t*>(s.o.reserve((size_t)n + 16));
    if (!d_src || !d_dst || !dev::to_dev(d_src, src, src_bytes, what)) return;
    if (!dev::ok(run(d_src, d_dst), what)) return;
    dev::to_host(dst, d_dst, n, what);
}

void dequant_q4_to_int8(const uint8_t* q4_data, int8_t* i8_data, float scale, uint32_t n) {
    dequant(q4_data, (n + 1) / 2, i8_data, n,
            [&](const uint8_t* a, int8_t* b) { return pf_dequant_q4_to_int8(a, b, scale, n, nullptr); },
            "dequant_q4_to_int8");
}
void dequant_q2_to_int8(const uint8_t* q2_data, int8_t* i8_data, float scale, uint32_t n) {
    dequant(q2_data, (n + 3) / 4, i8_data, n,
            [&](const uint8_t* a, int8_t* b) { return pf_dequant_q2_to_int8(a, b, scale, n, nullptr); },
            "dequant_q2_to_int8");
}
void dequant_ternary_to_int8(const uint8_t* t_data, int8_t* i8_data, uint32_t n) {
    dequant(t_data, (n + 1) / 2, i8_data, n,
            [&](const uint8_t* a, int8_t* b) { return pf_dequant_ternary_to_int8(a, b, n, nullptr); },
            "dequant_ternary_to_int8");
}

void matmul_int8(const int8_t* A, const int8_t* B, int32_t* C, uint32_t M, uint32_t N, uint32_t K) {
    Stage& s = stage();
    int8_t* a = static_cast<int8_t*>(s.a.reserve((size_t)M * K + 16));
    int8_t* b = static_cast<int8_t*>(s.b.reserve((size_t)N * K + 16));
    int32_t* c = static_cast<int32_t*>(s.o.reserve((size_t)M * N * 4 + 16));
    if (!a || !b || !c || !dev::to_dev(a, A, (size_t)M * K, "matmul_int8") ||
        !dev::to_dev(b, B, (size_t)N * K, "matmul_int8"))
        return;
    if (!dev::ok(pf_matmul_int8(a, b, c, (int32_t)M, (int32_t)N, (int32_t)K, nullptr), "matmul_int8")) return;
    dev::to_host(C, c, (size_t)M * N * 4, "matmul_int8");
}

void matmul_quantized(const float* A, const int8_t* B, float* C, uint32_t M, uint32_t N, uint32_t K,
                      const float* weight_scales, const float* act_scales) {
    Stage& s = stage();
    // a: A then the act scales; b: B; c: weight scales; o: C
    const size_t a_bytes = (size_t)M * K * 4;
    float* a = static_cast<float*>(s.a.reserve(a_bytes + (size_t)M * 4 + 16));
    int8_t* b = static_cast<int8_t*>(s.b.reserve((size_t)N * K + 16));
    float* ws = static_cast<float*>(s.c.reserve((size_t)N * 4 + 16));
    float* c = static_cast<float*>(s.o.reserve((size_t)M * N * 4 + 16));
    if (!a || !b || !ws || !c) return;
    float* as = a + (size_t)M * K;
    if (!dev::to_dev(a, A, a_bytes, "matmul_quantized") || !dev::to_dev(b, B, (size_t)N * K, "matmul_quantized") ||
        !dev::to_dev(ws, weight_scales, (size_t)N * 4, "matmul_quantized") ||
        (act_scales && !dev::to_dev(as, act_scales, (size_t)M * 4, "matmul_quantized")))
        return;
    if (!dev::ok(pf_matmul_quantized(a, b, c, (int32_t)M, (int32_t)N, (int32_t)K, ws, act_scales ? as : nullptr,
                                     nullptr),
                 "matmul_quantized"))
        return;
    dev::to_host(C, c, (size_t)M * N * 4, "matmul_quantized");
}

float dot_product(const float* a, const float* b, uint32_t n) {
    Stage& s = stage();
    float* da = static_cast<float*>(s.a.reserve((size_t)n * 4 + 16));
    float* db = static_cast<float*>(s.b.reserve((size_t)n * 4 + 16));
    float* out = static_cast<float*>(s.o.reserve(16));
    float r = 0.0f;
    if (!da || !db || !out || !dev::to_dev(da, a, (size_t)n * 4, "dot_product") ||
        !dev::to_dev(db, b, (size_t)n * 4, "dot_product"))
        return r;
    if (dev::ok(pf_dot_f32(da, db, n, out, nullptr), "dot_product")) dev::to_host(&r, out, 4, "dot_product");
    return r;
}

void softmax(float* vals, uint32_t n) {
    if (n == 0) return;
    Stage& s = stage();
    float* v = static_cast<float*>(s.a.reserve((size_t)n * 4 + 16));
    if (!v || !dev::to_dev(v, vals, (size_t)n * 4, "softmax")) return;
    if (dev::ok(pf_softmax_rows(v, 1, (int32_t)n, nullptr), "softmax")) dev::to_host(vals, v, (size_t)n * 4, "softmax");
}

void rmsnorm(float* out, const float* x, const float* weight, uint32_t n) {
    Stage& s = stage();
    float* dx = static_cast<float*>(s.a.reserve((size_t)n * 4 + 16));
    float* dw = static_cast<float*>(s.b.reserve((size_t)n * 4 + 16));
    float* dout = static_cast<float*>(s.o.reserve((size_t)n * 4 + 16));
    if (!dx || !dw || !dout || !dev::to_dev(dx, x, (size_t)n * 4, "rmsnorm") ||
        !dev::to_dev(dw, weight, (size_t)n * 4, "rmsnorm"))
        return;
    if (dev::ok(pf_rmsnorm_rows(dout, dx, dw, 1, (int32_t)n, nullptr), "rmsnorm"))
        dev::to_host(out, dout, (size_t)n * 4, "rmsnorm");
}

}  // namespace forge

// capi.cu — kernel-level C ABI: the reference's free functions
// (include/forge/matmul_neon.hpp, Engine::sample*) on caller-owned device
// buffers.  Shapes the projection kernel cannot take directly (K not a
// multiple of 128, N not a multiple of 64) go through zero-padded copies in
// stream-ordered scratch memory (cudaMallocAsync on the caller's stream).
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"
#include "gemm_tc.cuh"
#include "rows.cuh"
#include "step.cuh"

using namespace pf;

namespace {

struct Scratch {
    cudaStream_t st;
    std::vector<void*> bufs;
    explicit Scratch(cudaStream_t s) : st(s) {}
    template <typename T>
    pf_status get(T** p, size_t n) {
        void* q = nullptr;
        if (cudaMallocAsync(&q, std::max<size_t>(n * sizeof(T), 16), st) != cudaSuccess) {
            cudaGetLastError();
            set_error("scratch allocation of %zu bytes failed", n * sizeof(T));
            return PF_ERR_OOM;
        }
        bufs.push_back(q);
        *p = reinterpret_cast<T*>(q);
        return PF_OK;
    }
    ~Scratch() {
        for (void* p : bufs) cudaFreeAsync(p, st);
    }
};

int round_up(int a, int b) { return ceil_div(a, b) * b; }

__global__ void iota_kernel(int* out, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = i;
}

}  // namespace

extern "C" {

pf_status pf_quantize_activation_rows(const float* x, int8_t* q, float* scales, int32_t M, int32_t K, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(x && q && scales && M >= 0 && K > 0, "pf_quantize_activation_rows: bad arguments");
    if (M == 0) return PF_OK;
    return quant_rows(x, K, K, M, nullptr, q, scales, K, as_stream(stream));
}

pf_status pf_dequant_q4_to_int8(const uint8_t* src, int8_t* dst, float, int64_t n, void* stream) {
    PF_TRY(require_device());
    return dequant_ref(src, dst, n, 0, as_stream(stream));
}
pf_status pf_dequant_q2_to_int8(const uint8_t* src, int8_t* dst, float, int64_t n, void* stream) {
    PF_TRY(require_device());
    return dequant_ref(src, dst, n, 1, as_stream(stream));
}
pf_status pf_dequant_ternary_to_int8(const uint8_t* src, int8_t* dst, int64_t n, void* stream) {
    PF_TRY(require_device());
    return dequant_ref(src, dst, n, 2, as_stream(stream));
}

pf_status pf_pack_weights(const int8_t* w, int32_t rows, int32_t cols, int32_t qtype, void* packed, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(qtype >= 0 && qtype <= 3, "pf_pack_weights: bad qtype %d", qtype);
    PF_CHECK(rows >= 0 && cols > 0, "pf_pack_weights: bad shape %d x %d", rows, cols);
    if (rows == 0) return PF_OK;  // no rows: nothing to pack
    return pack_weights_tc(w, rows, cols, wfmt_of_qtype(qtype), packed, as_stream(stream));
}

pf_status pf_gemm_packed(const int8_t* Aq, const float* a_scale, const void* packed_w, const float* w_scale,
                         int32_t qtype, float* C, int32_t M, int32_t N, int32_t K, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(M >= 0, "pf_gemm_packed: M=%d", M);
    if (M == 0) return PF_OK;  // no rows: nothing to compute (as the reference's row loop)
    PF_CHECK(Aq && a_scale && packed_w && C, "pf_gemm_packed: null argument");
    GemmParams p;
    p.A = Aq; p.lda = K; p.a_scale = a_scale; p.M = M; p.N = N; p.K = K;
    p.W = packed_w; p.wf = wfmt_of_qtype(qtype); p.w_scale = w_scale;
    p.epi = EPI_F32; p.out = C; p.ldo = N;
    return gemm_tc_launch(p, 1, M, as_stream(stream));
}

pf_status pf_matmul_int8(const int8_t* A, const int8_t* B, int32_t* C, int32_t M, int32_t N, int32_t K,
                         void* stream) {
    PF_TRY(require_device());
    PF_CHECK(M >= 0 && N > 0 && K > 0, "pf_matmul_int8: bad shape");
    if (M == 0) return PF_OK;  // no rows: nothing to compute (as the reference's row loop)
    PF_CHECK(A && B && C, "pf_matmul_int8: null argument");
    cudaStream_t st = as_stream(stream);
    const int Kp = round_up(K, 128), Np = round_up(N, 64);
    Scratch s(st);
    int8_t* ap;
    uint8_t* wp;
    float* ones;
    PF_TRY(s.get(&ap, (size_t)M * Kp));
    PF_TRY(s.get(&wp, packed_bytes(N, K, WF_I8)));
    PF_TRY(s.get(&ones, (size_t)M));
    PF_CUDA(cudaMemsetAsync(ap, 0, (size_t)M * Kp, st));
    PF_CUDA(cudaMemcpy2DAsync(ap, Kp, A, K, K, M, cudaMemcpyDeviceToDevice, st));
    PF_TRY(pack_weights(B, N, K, WF_I8, wp, st));
    int32_t* cp = C;
    if (Np != N) PF_TRY(s.get(&cp, (size_t)M * Np));
    GemmParams p;
    p.A = ap; p.lda = Kp; p.a_scale = ones; p.M = M; p.N = Np; p.K = Kp;
    p.W = wp; p.wf = WF_I8; p.epi = EPI_I32; p.out_i32 = cp; p.ldo = Np;
    PF_TRY(gemm_launch(p, 1, st));
    if (cp != C) PF_CUDA(cudaMemcpy2DAsync(C, (size_t)N * 4, cp, (size_t)Np * 4, (size_t)N * 4, M, cudaMemcpyDeviceToDevice, st));
    return PF_OK;
}

pf_status pf_matmul_quantized(const float* A, const int8_t* B, float* C, int32_t M, int32_t N, int32_t K,
                              const float* weight_scales, const float* act_scales, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(M >= 0 && N > 0 && K > 0, "pf_matmul_quantized: bad shape");
    if (M == 0) return PF_OK;  // no rows: nothing to compute (as the reference's row loop)
    PF_CHECK(A && B && C && weight_scales, "pf_matmul_quantized: null argument");
    cudaStream_t st = as_stream(stream);
    const int Kp = round_up(K, 128), Np = round_up(N, 64);
    Scratch s(st);
    int8_t* aq;
    float* as;
    uint8_t* wp;
    float* ws = const_cast<float*>(weight_scales);
    PF_TRY(s.get(&aq, (size_t)M * Kp));
    PF_TRY(s.get(&as, (size_t)M));
    PF_TRY(s.get(&wp, packed_bytes(N, K, WF_I8)));
    PF_CUDA(cudaMemsetAsync(aq, 0, (size_t)M * Kp, st));
    if (act_scales) PF_TRY(quant_rows_given(A, K, M, act_scales, aq, as, Kp, st));
    else PF_TRY(quant_rows(A, K, K, M, nullptr, aq, as, Kp, st));
    PF_TRY(pack_weights(B, N, K, WF_I8, wp, st));
    float* cp = C;
    if (Np != N) {
        PF_TRY(s.get(&cp, (size_t)M * Np));
        PF_TRY(s.get(&ws, (size_t)Np));
        PF_CUDA(cudaMemsetAsync(ws, 0, (size_t)Np * 4, st));
        PF_CUDA(cudaMemcpyAsync(ws, weight_scales, (size_t)N * 4, cudaMemcpyDeviceToDevice, st));
    }
    GemmParams p;
    p.A = aq; p.lda = Kp; p.a_scale = as; p.M = M; p.N = Np; p.K = Kp;
    p.W = wp; p.wf = WF_I8; p.w_scale = ws; p.epi = EPI_F32; p.out = cp; p.ldo = Np;
    PF_TRY(gemm_launch(p, 1, st));
    if (cp != C) PF_CUDA(cudaMemcpy2DAsync(C, (size_t)N * 4, cp, (size_t)Np * 4, (size_t)N * 4, M, cudaMemcpyDeviceToDevice, st));
    return PF_OK;
}

pf_status pf_rmsnorm_rows(float* out, const float* x, const float* w, int32_t M, int32_t n, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(out && x && w && M >= 0 && n > 0, "pf_rmsnorm_rows: bad arguments");
    if (M == 0) return PF_OK;
    return rmsnorm_rows(out, x, w, M, n, as_stream(stream));
}

pf_status pf_softmax_rows(float* v, int32_t M, int32_t n, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(v && M >= 0 && n > 0, "pf_softmax_rows: bad arguments");
    if (M == 0) return PF_OK;
    return softmax_rows(v, M, n, as_stream(stream));
}

pf_status pf_argmax_rows(const float* logits, int32_t M, int32_t n, int32_t* out, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(logits && out && M >= 0 && n > 0, "pf_argmax_rows: bad arguments");
    if (M == 0) return PF_OK;
    return argmax_rows(logits, n, n, M, nullptr, out, as_stream(stream));
}

pf_status pf_sample_rows(const float* logits, int32_t M, int32_t n, const pf_sampling_config* cfg,
                         const float* uniforms, int32_t* out, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(logits && cfg && out && M >= 0 && n > 0, "pf_sample_rows: bad arguments");
    if (M == 0) return PF_OK;
    cudaStream_t st = as_stream(stream);
    if (cfg->greedy || cfg->temperature <= 0.0f) return argmax_rows(logits, n, n, M, nullptr, out, st);
    PF_CHECK(uniforms, "pf_sample_rows: uniforms required for stochastic sampling");
    Scratch s(st);
    int* rows;
    PF_TRY(s.get(&rows, (size_t)M));
    iota_kernel<<<ceil_div(M, 128), 128, 0, st>>>(rows, M);
    PF_TRY(launch_check("iota"));
    return sample_rows(logits, n, n, rows, M, *cfg, uniforms, 1, out, st);
}

}  // extern "C"

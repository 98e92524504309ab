// static_ws.cu — pf_gemm_packed_static: the packed-weight projection kernel
// with its split-K scratch inside the library image instead of in memory the
// library or the caller allocates.
//
// Who needs it: a host runtime that owns every byte of device memory through
// its own pool (and forbids other allocators), or a latency-critical path
// that must not allocate because cudaMalloc can synchronise the device.  Such
// callers still pass their own input and output buffers; the only extra
// memory the kernel needs — int32 partial sums and per-tile counters of the
// split-K reduction — is the file-scope array below.
//
// The array is a fixed part of the module: every GPU that loads the library
// holds it (kStaticWsElems * 4 + kStaticCounters * 4 bytes) until the process
// exits.  All calls on a device share it and it keeps the last call's
// contents, so each call clears the part it uses on the caller's stream
// before launching; two calls whose work overlaps on the GPU (different
// streams, no ordering between them) race on it and must not be issued.
// Every call looks up the array's device address (cudaGetSymbolAddress) with
// the caller's device current.  The first lookup on a device loads the
// module there, so make the first call before any stream capture.  Later
// lookups are cheap, and looking up every time keeps a call after
// cudaDeviceReset (which unloads the module; the array may come back at
// another address) from writing through a stale pointer.
#include "gemm.cuh"
#include "gemm_tc.cuh"

namespace pf {
namespace {

constexpr size_t kStaticWsElems = (size_t)1 << 20;  // int32 partial sums: M*N <= 1,048,576
constexpr int kStaticCounters = 4096;                // split-K tiles: ceil(M/128)*ceil(N/64) <= 4096

static __device__ __align__(256) int32_t g_split_ws[kStaticWsElems];
static __device__ __align__(256) int g_split_cnt[kStaticCounters];

struct StaticAddr {
    int32_t* ws = nullptr;
    int* cnt = nullptr;
};

pf_status static_addr(StaticAddr* out) {
    // In host code g_split_ws names a host-side shadow, not device memory:
    // the kernel gets the address the device sees.
    void* ws = nullptr;
    void* cnt = nullptr;
    PF_CUDA(cudaGetSymbolAddress(&ws, g_split_ws));
    PF_CUDA(cudaGetSymbolAddress(&cnt, g_split_cnt));
    out->ws = static_cast<int32_t*>(ws);
    out->cnt = static_cast<int*>(cnt);
    return PF_OK;
}

}  // namespace
}  // namespace pf

using namespace pf;

extern "C" pf_status pf_gemm_packed_static(const int8_t* Aq, const float* a_scale, const void* packed_w,
                                           const float* w_scale, int32_t qtype, float* C, int32_t M, int32_t N,
                                           int32_t K, void* stream) {
    PF_TRY(require_device());
    PF_CHECK(M >= 0, "pf_gemm_packed_static: M=%d", M);
    if (M == 0) return PF_OK;  // no rows: nothing to compute (as pf_gemm_packed)
    PF_CHECK(Aq && a_scale && packed_w && C, "pf_gemm_packed_static: null argument");
    PF_CHECK(N > 0 && K > 0, "pf_gemm_packed_static: empty shape");
    PF_CHECK((size_t)M * (size_t)N <= kStaticWsElems,
             "pf_gemm_packed_static: M*N = %lld exceeds the static workspace of %zu partial sums",
             (long long)M * N, kStaticWsElems);
    const size_t tiles = (size_t)ceil_div(M, 128) * (size_t)ceil_div(N, 64);
    PF_CHECK(tiles <= (size_t)kStaticCounters, "pf_gemm_packed_static: %zu output tiles exceed the %d static tile counters",
             tiles, kStaticCounters);
    StaticAddr a;
    PF_TRY(static_addr(&a));
    cudaStream_t st = as_stream(stream);
    GemmParams p;
    p.A = Aq; p.lda = K; p.a_scale = a_scale; p.M = M; p.N = N; p.K = K;
    p.W = packed_w; p.wf = wfmt_of_qtype(qtype); p.w_scale = w_scale;
    p.epi = EPI_F32; p.out = C; p.ldo = N;
    const int bn = gemm_tc_pick_bn(M, N, 1);
    p.splits = std::min(K / 128, std::max(2, gemm_tc_pick_splits(M, N, K, bn, true)));
    p.ws = a.ws;
    p.counters = a.cnt;
    p.ws_elems = kStaticWsElems;
    p.cnt_elems = kStaticCounters;
    // The kernel leaves the workspace zeroed, but an earlier call that did not
    // complete may not have: clear what this call reads before its first use
    // (the partial sums [n][m] and the counters of every tile index the launch
    // can form, ceil(M/128) * N/BN <= tiles).
    PF_CUDA(cudaMemsetAsync(a.ws, 0, (size_t)M * N * sizeof(int32_t), st));
    PF_CUDA(cudaMemsetAsync(a.cnt, 0, tiles * sizeof(int), st));
    return gemm_tc_launch(p, 1, M, st);
}

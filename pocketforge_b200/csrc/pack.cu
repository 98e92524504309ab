// pack.cu — device weight formats.
//
// The reference keeps every projection as int8 values in [-8,7] (Q4), [-2,1]
// (Q2) or {-1,0,1} (Q1.5) after WeightLoader::load_block_with_scales
// (src/quant_format.cpp:399-419).  On the device they stay packed at 4 or 2
// bits and are unpacked in registers right before the tensor-core MMA, so a
// projection reads 0.5 B (Q4) or 0.25 B (Q2, Q1.5) per weight from HBM.
//
// Layout: groups of 8 rows x 128 columns, row-group major.  Inside a group,
// lane l = 4*g + t of a warp owns row g and, for every 32-column block kb,
// the 4 columns kb*32 + 4t + {0..3} (low half) and kb*32 + 16 + 4t + {0..3}
// (high half) — exactly the B fragment of mma.m16n8k32 — so one 128-bit load
// per lane fetches a full fragment set with no shuffles.
//   Q4 (16 B/lane): word kb, byte j: low nibble = low half j, high nibble = high half j.
//   Q2 ( 8 B/lane): word w covers kb = 2w, 2w+1; byte j bits [2s,2s+2) hold
//                   s=0: kb 2w low, s=1: kb 2w high, s=2: kb 2w+1 low, s=3: kb 2w+1 high.
//   I8 (32 B/lane): word 2kb = low half, word 2kb+1 = high half.
// Values are stored as two's complement fields (v & 0xF, v & 0x3).
#include "common.cuh"

namespace pf {

__global__ void pack_weights_kernel(const int8_t* __restrict__ w, int rows, int cols, int wf,
                                    uint32_t* __restrict__ out, int col_groups, int n_groups,
                                    uint32_t* err) {
    const int gid = blockIdx.x * blockDim.x + threadIdx.x;  // (group, lane)
    if (gid >= n_groups * 32) return;
    const int group = gid >> 5, lane = gid & 31;
    const int gr = group / col_groups, gc = group % col_groups;
    const int row = gr * kPackRows + (lane >> 2), t = lane & 3;
    const int c0 = gc * kPackCols;
    auto val = [&](int c) -> int {
        if (row >= rows || c >= cols) return 0;
        return (int)w[(size_t)row * cols + c];
    };
    bool bad = false;
    if (wf == WF_Q4) {
        uint32_t words[4];
        for (int kb = 0; kb < 4; kb++) {
            uint32_t word = 0;
            for (int j = 0; j < 4; j++) {
                const int lo = val(c0 + kb * 32 + 4 * t + j), hi = val(c0 + kb * 32 + 16 + 4 * t + j);
                bad |= lo < -8 || lo > 7 || hi < -8 || hi > 7;
                word |= (uint32_t)((lo & 0xF) | ((hi & 0xF) << 4)) << (8 * j);
            }
            words[kb] = word;
        }
        uint4* dst = reinterpret_cast<uint4*>(out) + (size_t)group * 32 + lane;
        *dst = make_uint4(words[0], words[1], words[2], words[3]);
    } else if (wf == WF_Q2) {
        uint32_t words[2];
        for (int ww = 0; ww < 2; ww++) {
            uint32_t word = 0;
            for (int j = 0; j < 4; j++) {
                uint32_t byte = 0;
                for (int s = 0; s < 4; s++) {
                    const int kb = 2 * ww + (s >> 1);
                    const int c = c0 + kb * 32 + (s & 1) * 16 + 4 * t + j;
                    const int v = val(c);
                    bad |= v < -2 || v > 1;
                    byte |= (uint32_t)(v & 3) << (2 * s);
                }
                word |= byte << (8 * j);
            }
            words[ww] = word;
        }
        uint2* dst = reinterpret_cast<uint2*>(out) + (size_t)group * 32 + lane;
        *dst = make_uint2(words[0], words[1]);
    } else {
        uint32_t words[8];
        for (int kb = 0; kb < 4; kb++)
            for (int h = 0; h < 2; h++) {
                uint32_t word = 0;
                for (int j = 0; j < 4; j++)
                    word |= (uint32_t)(val(c0 + kb * 32 + h * 16 + 4 * t + j) & 0xFF) << (8 * j);
                words[2 * kb + h] = word;
            }
        uint4* dst = reinterpret_cast<uint4*>(out) + ((size_t)group * 32 + lane) * 2;
        dst[0] = make_uint4(words[0], words[1], words[2], words[3]);
        dst[1] = make_uint4(words[4], words[5], words[6], words[7]);
    }
    if (bad) atomicOr(err, ERR_WEIGHT_RANGE);
}

pf_status pack_weights(const int8_t* w, int rows, int cols, int wf, void* packed, cudaStream_t st) {
    PF_CHECK(rows > 0 && cols > 0 && w && packed, "pack_weights: bad arguments");
    const int cg = ceil_div(cols, kPackCols);
    const int ng = ceil_div(rows, kPackRows) * cg;
    const int threads = 256;
    const int blocks = ceil_div(ng * 32, threads);
    pack_weights_kernel<<<blocks, threads, 0, st>>>(w, rows, cols, wf, (uint32_t*)packed, cg, ng,
                                                    device_error_flag());
    return launch_check("pack_weights");
}

// ---------------------------------------------------------------------------
// The reference's decoders (src/matmul_neon.cpp:34-75), elementwise.
// ---------------------------------------------------------------------------
__global__ void dequant_ref_kernel(const uint8_t* __restrict__ src, int8_t* __restrict__ dst,
                                   int64_t n, int kind) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    int v;
    if (kind == 0) {  // Q4: element 2k low nibble, 2k+1 high nibble, minus 8
        const uint8_t b = src[i >> 1];
        v = (int)((i & 1) ? (b >> 4) : (b & 0xF)) - 8;
    } else if (kind == 1) {  // Q2: 4 codes per byte, LSB first, minus 2
        const uint8_t b = src[i >> 2];
        v = (int)((b >> (2 * (i & 3))) & 3) - 2;
    } else {  // ternary: 2 codes per byte in bits 0-1, 2-3; LUT {-1,0,1,0}
        const uint8_t b = src[i >> 1];
        const int code = (b >> (2 * (i & 1))) & 3;
        v = (code == 0) ? -1 : (code == 2 ? 1 : 0);
    }
    dst[i] = (int8_t)v;
}

pf_status dequant_ref(const uint8_t* src, int8_t* dst, int64_t n, int kind, cudaStream_t st) {
    PF_CHECK(n >= 0 && (n == 0 || (src && dst)), "dequant: bad arguments");
    if (n == 0) return PF_OK;
    const int threads = 256;
    dequant_ref_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, st>>>(src, dst, n, kind);
    return launch_check("dequant");
}

}  // namespace pf

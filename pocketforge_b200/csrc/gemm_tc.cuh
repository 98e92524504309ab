// gemm_tc.cuh — tcgen05 (5th-generation tensor core) projection GEMM.
#pragma once
#include "gemm.cuh"

namespace pf {

// Bytes of a weight matrix in the tensor-core packed layout (gemm_tc.cu).
size_t packed_bytes_tc(int rows, int cols, int wf);
pf_status pack_weights_tc(const int8_t* w, int rows, int cols, int wf, void* packed, cudaStream_t st);
int gemm_tc_pick_bn(int M, int N, int planes);
int gemm_tc_pick_splits(int M, int N, int K, int bn, bool have_ws);
// K splits for a slices-mode launch (GemmParams::slice_stride) of an M x N x K product.
int gemm_tc_slices(int M, int N, int K);
// planes == 3: A holds three digit planes of plane_rows rows each
// (plane_stride == plane_rows * lda).  p.splits == 0 picks the split count.
// Launches of at most kGemvMaxRows activation rows (planes x M) with the
// I32 (slices or whole K), F32, SWIGLU or LOGITS3 epilogue run on the dp4a
// kernel of gemv.cu instead of the tensor-core tiles.
pf_status gemm_tc_launch(const GemmParams& p, int planes, int plane_rows, cudaStream_t st);

// The few-row projection (gemv.cu).
constexpr int kGemvMaxRows = 16;
bool gemv_applies(const GemmParams& p, int planes);
pf_status gemv_launch(const GemmParams& p, int planes, cudaStream_t st);

}  // namespace pf

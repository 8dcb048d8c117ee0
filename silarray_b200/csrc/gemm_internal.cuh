// Internal interface between the GEMM dispatcher (gemm.cu) and the tcgen05
// tensor-core path (tc_gemm.cu).
#pragma once

#include "common.cuh"

namespace silcu {

enum GemmPath { kPathFfma = 0, kPathSkinny = 1, kPathTc = 2 };

// Which kernel family silcu_sgemm_ex uses for these arguments.
int gemm_path(const silcu_gemm_args &a);

// Epilogue of the CUDA-core GEMMs: alpha, bias[col % bias_len], activation,
// residual, in the reference's order.
struct SkinnyEpi {
  float alpha;
  const float *bias;
  int64_t bias_len;
  int act;
  const float *residual;
  int64_t ldr;
};

// Skinny GEMM (2 <= M <= 32, plain row-major operands whose rows are
// 16-byte aligned): one wave of clusters streaming W by TMA tile loads
// (skinny.cu).  No workspace.
bool skinny_tma_eligible(const silcu_gemm_args &a);
silcu_status skinny_tma_run(const silcu_gemm_args &a, const SkinnyEpi &epi, cudaStream_t s);

// Workspace of the 3xTF32 path: the hi/lo split operands, K-major.
size_t tc_workspace_bytes(const silcu_gemm_args &a);
// Implicit-GEMM convolution operand: the exact tf32 split of an NHWC input
// [N, H, W, C] (C % 16 == 0, 16-byte aligned), read by im2col TMA boxes as
// the A operand of a GEMM with M = N*H*W rows and K = Kf*Kf*C in (kh, kw, c)
// order (stride 1, zero padding pad).
struct TcConv {
  const float *in_hi, *in_lo;
  int64_t N, H, W, C, Kf, pad;
};
// Exact tf32 split of n contiguous floats (n % 4 == 0, 16-byte aligned).
silcu_status split_contiguous(const float *src, uint64_t n, float *hi, float *lo, cudaStream_t s);
silcu_status tc_run(const silcu_gemm_args &a, void *ws, size_t ws_bytes, cudaStream_t s,
                    const TcConv *conv = nullptr);
// The 3xTF32 path's tiling and split-K choice for these arguments.
void tc_describe(const silcu_gemm_args &a, silcu_gemm_plan *out);

}  // namespace silcu

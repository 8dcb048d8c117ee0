// Internal interface between the GEMM dispatcher (gemm.cu) and the tcgen05
// tensor-core path (tc_gemm.cu).
#pragma once

#include "common.cuh"

namespace silcu {

enum GemmPath { kPathFfma = 0, kPathSkinny = 1, kPathTc = 2 };

// Which kernel family silcu_sgemm_ex uses for these arguments.
int gemm_path(const silcu_gemm_args &a);

// Workspace of the 3xTF32 path: the hi/lo split operands, K-major.
size_t tc_workspace_bytes(const silcu_gemm_args &a);
silcu_status tc_run(const silcu_gemm_args &a, void *ws, size_t ws_bytes, cudaStream_t s);
// The 3xTF32 path's tiling and split-K choice for these arguments.
void tc_describe(const silcu_gemm_args &a, silcu_gemm_plan *out);

}  // namespace silcu

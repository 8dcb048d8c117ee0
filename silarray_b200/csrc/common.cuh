// Shared helpers for the sm_100a kernels behind include/silcu.h.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/silcu.h"

namespace silcu {

// 148 SMs on B200; the grid helpers query the real count once per device.
int sm_count();

// Records a message for silcu_last_error() and returns the status.
silcu_status fail(silcu_status st, const char *fmt, ...);

// Device address of the error word that bounded waits set (per device).
int *device_error_ptr();

// Counts `launches` kernel launches and maps cudaGetLastError() into a status.
silcu_status check_launch(const char *what, int launches = 1);

inline cudaStream_t as_stream(silcu_stream s) {
  return reinterpret_cast<cudaStream_t>(s);
}

inline bool aligned16(const void *p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// ---------------------------------------------------------------- device side
// IEEE round-to-nearest arithmetic without contraction: the reference CPU
// path rounds after every operation, so fused kernels use these to keep the
// same rounding sequence (nvcc would otherwise fuse a*b+c into one FMA).
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float div_rn(float a, float b) { return __fdiv_rn(a, b); }

// sigmoid in the reference's order (include/cpu.h:290-297): negate, exp,
// add one, reciprocal.  expf is CUDA's accurate single-precision exp.
__device__ __forceinline__ float sigmoid_ref(float x) {
  float t = expf(-x);
  t = __fadd_rn(t, 1.0f);
  return __frcp_rn(t);
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace silcu

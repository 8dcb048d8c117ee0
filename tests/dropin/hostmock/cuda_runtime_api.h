// Test double of the CUDA runtime for the CPU tests of the drop-in host layer
// (include/sil_b200): just the calls its headers make, on host memory.  Used
// only by tests/test_dropin_host.py; the product links the real runtime.
#pragma once
#include <cstddef>
#include <cstdlib>

typedef int cudaError_t;
typedef struct CUstream_st *cudaStream_t;
enum { cudaSuccess = 0, cudaErrorMemoryAllocation = 2 };
enum { cudaMemAttachGlobal = 1, cudaStreamNonBlocking = 1 };

inline const char *cudaGetErrorString(cudaError_t e) { return e ? "mock error" : "no error"; }
inline cudaError_t cudaMallocManaged(void **p, size_t bytes, unsigned = cudaMemAttachGlobal) {
  *p = std::aligned_alloc(256, (bytes + 255) / 256 * 256);
  return *p ? cudaSuccess : cudaErrorMemoryAllocation;
}
inline cudaError_t cudaMalloc(void **p, size_t bytes) { return cudaMallocManaged(p, bytes); }
inline cudaError_t cudaFree(void *p) {
  std::free(p);
  return cudaSuccess;
}
inline cudaError_t cudaStreamCreateWithFlags(cudaStream_t *s, unsigned) {
  *s = reinterpret_cast<cudaStream_t>(0x5);
  return cudaSuccess;
}
inline cudaError_t cudaStreamSynchronize(cudaStream_t) { return cudaSuccess; }

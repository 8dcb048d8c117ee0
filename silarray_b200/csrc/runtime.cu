// Host-side plumbing shared by every entry point of include/silcu.h:
// error reporting, SM count, stream sync and the device error word.
#include <stdarg.h>
#include <string.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace silcu {

static thread_local char g_last_error[512] = "";

// Set by bounded device-side waits when they give up (see tc_gemm.cu).
__device__ int g_device_error = 0;

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

silcu_status fail(silcu_status st, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return st;
}

int *device_error_ptr() {
  static int *cached[64] = {nullptr};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cached[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) == cudaSuccess) cached[dev] = static_cast<int *>(p);
  }
  return cached[dev];
}

static unsigned long long g_launches = 0;

silcu_status check_launch(const char *what, int launches) {
  __atomic_fetch_add(&g_launches, (unsigned long long)launches, __ATOMIC_RELAXED);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SILCU_CUDA_ERROR, "%s: %s", what, cudaGetErrorString(e));
  return SILCU_OK;
}

// One CTA waits on an mbarrier that nothing arrives at, through the same
// bounded wait as the tensor-core kernels but with the caller's limit.
__global__ void bounded_wait_probe(int *err, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(tc::smem_u32(&bar), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  tc::mbar_wait_limit(tc::smem_u32(&bar), 0, err, 77, limit_ns);
  __syncthreads();
}

}  // namespace silcu

extern "C" {

silcu_status silcu_check_bounded_wait(uint32_t limit_us, silcu_stream stream) {
  if (limit_us == 0 || limit_us > 1000000u)
    return silcu::fail(SILCU_INVALID_ARGUMENT, "check_bounded_wait: limit %u us outside 1..1000000", limit_us);
  int *err = silcu::device_error_ptr();
  if (!err) return silcu::fail(SILCU_CUDA_ERROR, "check_bounded_wait: no device error word");
  silcu::bounded_wait_probe<<<1, 64, 0, silcu::as_stream(stream)>>>(err, 1000ull * limit_us);
  return silcu::check_launch("check_bounded_wait");
}

const char *silcu_last_error(void) { return silcu::g_last_error; }

int silcu_abi_version(void) { return 2; }

unsigned long long silcu_kernel_launches(void) {
  return __atomic_load_n(&silcu::g_launches, __ATOMIC_RELAXED);
}

silcu_status silcu_synchronize(silcu_stream stream) {
  cudaError_t e = cudaStreamSynchronize(silcu::as_stream(stream));
  if (e != cudaSuccess)
    return silcu::fail(SILCU_CUDA_ERROR, "synchronize: %s", cudaGetErrorString(e));
  return SILCU_OK;
}

silcu_status silcu_device_status(silcu_stream stream) {
  int host = 0, zero = 0;
  cudaStream_t s = silcu::as_stream(stream);
  cudaError_t e = cudaMemcpyFromSymbolAsync(&host, silcu::g_device_error, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess)
    e = cudaMemcpyToSymbolAsync(silcu::g_device_error, &zero, sizeof(int), 0,
                                cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess)
    return silcu::fail(SILCU_CUDA_ERROR, "device_status: %s", cudaGetErrorString(e));
  if (host) return silcu::fail(SILCU_TIMEOUT, "a bounded device wait gave up (code %d)", host);
  return SILCU_OK;
}

}  // extern "C"

// silarray's GPU backend on the B200 (replaces the reference's include/gpu.h).
//
// `class gpu` keeps every static function array.h calls, with the same
// names, arguments and meaning (reference include/gpu.h:266-1036), and runs
// each through the C ABI of include/silcu.h (libsilcu.so, sm_100a kernels):
// a storage handle becomes `(float *)data + off` and its `len`.  Work is
// queued on CUDA's legacy default stream; gpu_context::flush() waits for it,
// as the reference's command-buffer commit/wait does (gpu.h:107-123).  Errors
// surface as std::runtime_error with the library's message.
//
// The host layer owns the only allocations: managed storage (unified_memory.h)
// and one growing device workspace for the multi-pass kernels.
#pragma once

#include <types.h>
#include <device.h>

#include <cuda_runtime_api.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <type_traits>

#include "silcu.h"

namespace sil {

namespace b200 {

inline void check(silcu_status st) {
  if (st != SILCU_OK) throw std::runtime_error(std::string("silarray b200: ") + silcu_last_error());
}

inline silcu_stream stream() { return nullptr; }  // legacy default stream

// Device workspace for multi-pass kernels, grown on demand.  Growth waits for
// queued work first, since kernels in flight may still use the old buffer.
inline void *workspace(size_t bytes) {
  static void *ptr = nullptr;
  static size_t cap = 0;
  if (bytes == 0) return ptr;
  if (bytes > cap) {
    if (ptr) {
      cudaStreamSynchronize(nullptr);
      cudaFree(ptr);
    }
    size_t want = bytes + bytes / 4 + (1u << 20);
    if (cudaMalloc(&ptr, want) != cudaSuccess) {
      ptr = nullptr;
      cap = 0;
      throw std::runtime_error("silarray b200: workspace allocation failed");
    }
    cap = want;
  }
  return ptr;
}

inline size_t workspace_cap(size_t bytes) { return bytes ? bytes + bytes / 4 + (1u << 20) : 0; }

template <class T>
inline T *ptr(const storage &s) {
  return static_cast<T *>(s.data) + s.off;
}

inline void queued() { gpu_pending_ = true; }

inline silcu_gemm_args gemm_args(const storage &A, const storage &B, storage &C, uint32_t M, uint32_t N,
                                 uint32_t K, uint32_t lda, uint32_t ldb, bool tA, bool tB) {
  silcu_gemm_args a{};
  a.A = ptr<const float>(A);
  a.B = ptr<const float>(B);
  a.C = ptr<float>(C);
  a.M = M;
  a.N = N;
  a.K = K;
  a.lda = lda;
  a.ldb = ldb;
  a.ldc = N;
  a.trans_a = tA;
  a.trans_b = tB;
  a.batch = 1;
  a.alpha = 1.0f;
  a.algo = SILCU_GEMM_AUTO;
  return a;
}

inline void run_gemm(const silcu_gemm_args &a) {
  size_t need = silcu_sgemm_workspace_bytes(&a);
  void *ws = workspace(need);
  check(silcu_sgemm_ex(&a, ws, need ? workspace_cap(need) : 0, stream()));
  queued();
}

}  // namespace b200

class gpu_context {
 public:
  static gpu_context &instance() {
    static gpu_context ctx;
    return ctx;
  }
  // Waits for every queued kernel (the reference's commit + waitUntilCompleted).
  void flush() {
    b200::check(silcu_synchronize(b200::stream()));
    b200::check(silcu_device_status(b200::stream()));
    gpu_pending_ = false;
  }
};

class gpu {
  template <value_type T>
  static void arith_(int op, const storage &A, const storage &B, storage &OUT) {
    using b200::ptr;
    silcu_status st;
    if constexpr (std::is_same_v<T, float>) {
      auto a = ptr<const float>(A), b = ptr<const float>(B);
      auto o = ptr<float>(OUT);
      switch (op) {
        case 0: st = silcu_add_f32(a, A.len, b, B.len, o, OUT.len, b200::stream()); break;
        case 1: st = silcu_sub_f32(a, A.len, b, B.len, o, OUT.len, b200::stream()); break;
        case 2: st = silcu_mul_f32(a, A.len, b, B.len, o, OUT.len, b200::stream()); break;
        case 3: st = silcu_div_f32(a, A.len, b, B.len, o, OUT.len, b200::stream()); break;
        default: st = silcu_pow_f32(a, A.len, b, B.len, o, OUT.len, b200::stream()); break;
      }
    } else if constexpr (std::is_same_v<T, int>) {
      auto a = ptr<const int32_t>(A), b = ptr<const int32_t>(B);
      auto o = ptr<int32_t>(OUT);
      switch (op) {
        case 0: st = silcu_add_i32(a, A.len, b, B.len, o, OUT.len, b200::stream()); break;
        case 1: st = silcu_sub_i32(a, A.len, b, B.len, o, OUT.len, b200::stream()); break;
        case 2: st = silcu_mul_i32(a, A.len, b, B.len, o, OUT.len, b200::stream()); break;
        case 3: st = silcu_div_i32(a, A.len, b, B.len, o, OUT.len, b200::stream()); break;
        default: st = silcu_pow_i32(a, A.len, b, B.len, o, OUT.len, b200::stream()); break;
      }
    } else {
      throw std::runtime_error("silarray b200: arithmetic on bool arrays runs on the CPU");
    }
    b200::check(st);
    b200::queued();
  }

  static size_t reduce_(silcu_status (*fn)(const float *, size_t, float *, void *, size_t, silcu_stream),
                        const storage &IN, storage &OUT, size_t length) {
    size_t need = silcu_reduce_workspace_bytes(length);
    void *ws = b200::workspace(need);
    b200::check(fn(b200::ptr<const float>(IN), length, b200::ptr<float>(OUT), ws, b200::workspace_cap(need),
                   b200::stream()));
    b200::queued();
    return 1;  // the result is finished on the device: one "partial"
  }

 public:
  // include/gpu.h:289-312
  template <value_type T> static void add(const storage &A, const storage &B, storage &OUT) { arith_<T>(0, A, B, OUT); }
  template <value_type T> static void sub(const storage &A, const storage &B, storage &OUT) { arith_<T>(1, A, B, OUT); }
  template <value_type T> static void mul(const storage &A, const storage &B, storage &OUT) { arith_<T>(2, A, B, OUT); }
  template <value_type T> static void div(const storage &A, const storage &B, storage &OUT) { arith_<T>(3, A, B, OUT); }
  template <value_type T> static void pow(const storage &A, const storage &B, storage &OUT) { arith_<T>(4, A, B, OUT); }

  // include/gpu.h:314-320
  static void sigmoid(const storage &IN, storage &OUT) {
    b200::check(silcu_sigmoid_f32(b200::ptr<const float>(IN), b200::ptr<float>(OUT), OUT.len, b200::stream()));
    b200::queued();
  }
  static void relu(const storage &IN, storage &OUT) {
    b200::check(silcu_relu_f32(b200::ptr<const float>(IN), b200::ptr<float>(OUT), OUT.len, b200::stream()));
    b200::queued();
  }

  // include/gpu.h:323-354, 409-470: the number of partials the caller must
  // finish on the host; here the device finishes, so it is always one.
  static size_t sum_f32_num_tg(size_t) { return 1; }
  static size_t min_f32_num_tg(size_t) { return 1; }
  static size_t max_f32_num_tg(size_t) { return 1; }
  static size_t sum_f32(const storage &IN, storage &OUT, size_t length) { return reduce_(silcu_sum_f32, IN, OUT, length); }
  static size_t min_f32(const storage &IN, storage &OUT, size_t length) { return reduce_(silcu_min_f32, IN, OUT, length); }
  static size_t max_f32(const storage &IN, storage &OUT, size_t length) { return reduce_(silcu_max_f32, IN, OUT, length); }

  // include/gpu.h:385-406 (the partial buffer of the two-pass Metal kernel is not needed)
  static void sum_axis0_f32(const storage &IN, storage &OUT, size_t rows, size_t cols, const storage &,
                            size_t, size_t) {
    size_t need = silcu_sum_axis_workspace_bytes(1, rows, cols);
    void *ws = b200::workspace(need);
    b200::check(silcu_sum_axis_f32(b200::ptr<const float>(IN), b200::ptr<float>(OUT), 1, rows, cols, ws,
                                   b200::workspace_cap(need), b200::stream()));
    b200::queued();
  }

  // include/gpu.h:473-501
  static void layer_norm(const storage &IN, storage &OUT, const storage &gamma, const storage &beta, uint32_t rows,
                         uint32_t cols, float eps) {
    b200::check(silcu_layer_norm_f32(b200::ptr<const float>(IN), b200::ptr<float>(OUT),
                                     b200::ptr<const float>(gamma), b200::ptr<const float>(beta), rows, cols, eps,
                                     b200::stream()));
    b200::queued();
  }

  // include/gpu.h:509-535, 577-581 (the STEEL / non-STEEL split is the backend's choice here)
  static void sgemm(const storage &A, const storage &B, storage &C, uint32_t M, uint32_t N, uint32_t K,
                    uint32_t lda, uint32_t ldb, bool transA, bool transB) {
    b200::run_gemm(b200::gemm_args(A, B, C, M, N, K, lda, ldb, transA, transB));
  }
  static void sgemm_steel(const storage &A, const storage &B, storage &C, uint32_t M, uint32_t N, uint32_t K,
                          uint32_t lda, uint32_t ldb) {
    b200::run_gemm(b200::gemm_args(A, B, C, M, N, K, lda, ldb, false, false));
  }
  static void sgemm_batched(const storage &A, const storage &B, storage &C, uint32_t M, uint32_t N, uint32_t K,
                            uint32_t lda, uint32_t ldb, uint32_t batch, uint32_t stride_a, uint32_t stride_b,
                            uint32_t stride_c) {
    auto a = b200::gemm_args(A, B, C, M, N, K, lda, ldb, false, false);
    a.batch = batch;
    a.stride_a = stride_a;
    a.stride_b = stride_b;
    a.stride_c = stride_c;
    b200::run_gemm(a);
  }
  static void sgemm_steel_batched(const storage &A, const storage &B, storage &C, uint32_t M, uint32_t N,
                                  uint32_t K, uint32_t lda, uint32_t ldb, uint32_t batch, uint32_t stride_a,
                                  uint32_t stride_b, uint32_t stride_c) {
    sgemm_batched(A, B, C, M, N, K, lda, ldb, batch, stride_a, stride_b, stride_c);
  }
  // include/gpu.h:549-574
  static void sgemv(const storage &x, const storage &B, storage &y, uint32_t N, uint32_t K) {
    b200::run_gemm(b200::gemm_args(x, B, y, 1, N, K, K, N, false, false));
  }
  // include/gpu.h:584-590, 609-615: bias[col % bias_len] (+ sigmoid) fused in the epilogue
  static void sgemm_bias_steel(const storage &A, const storage &B, storage &C, const storage &bias,
                               uint32_t bias_len, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb) {
    auto a = b200::gemm_args(A, B, C, M, N, K, lda, ldb, false, false);
    a.bias = b200::ptr<const float>(bias);
    a.bias_len = bias_len;
    b200::run_gemm(a);
  }
  static void sgemm_bias_sigmoid_steel(const storage &A, const storage &B, storage &C, const storage &bias,
                                       uint32_t bias_len, uint32_t M, uint32_t N, uint32_t K, uint32_t lda,
                                       uint32_t ldb) {
    auto a = b200::gemm_args(A, B, C, M, N, K, lda, ldb, false, false);
    a.bias = b200::ptr<const float>(bias);
    a.bias_len = bias_len;
    a.act = SILCU_ACT_SIGMOID;
    b200::run_gemm(a);
  }
  // include/gpu.h:1296-1328: transposed operands, physical row-major layouts
  static void dot_f32_ex(const storage &A, const storage &B, storage &OUT, size_t, size_t phys_A_cols, size_t,
                         size_t phys_B_cols, size_t M, size_t N, size_t K, bool transA, bool transB) {
    b200::run_gemm(b200::gemm_args(A, B, OUT, uint32_t(M), uint32_t(N), uint32_t(K), uint32_t(phys_A_cols),
                                   uint32_t(phys_B_cols), transA, transB));
  }

  // include/gpu.h:890-942
  static void argmax_f32(const storage &IN, storage &OUT, uint32_t rows, uint32_t cols) {
    size_t need = silcu_argmax_workspace_bytes(rows, cols);
    void *ws = b200::workspace(need);
    b200::check(silcu_argmax_f32(b200::ptr<const float>(IN), b200::ptr<int32_t>(OUT), rows, cols, ws,
                                 b200::workspace_cap(need), b200::stream()));
    b200::queued();
  }
  static void softmax(const storage &IN, storage &OUT, uint32_t rows, uint32_t cols) {
    b200::check(silcu_softmax_f32(b200::ptr<const float>(IN), b200::ptr<float>(OUT), rows, cols, b200::stream()));
    b200::queued();
  }

  // include/gpu.h:945-1004
  static void sigmoid_backward(const storage &dout, const storage &x, storage &OUT, size_t n) {
    b200::check(silcu_sigmoid_backward_f32(b200::ptr<const float>(dout), b200::ptr<const float>(x),
                                           b200::ptr<float>(OUT), n, b200::stream()));
    b200::queued();
  }
  static void bias_sigmoid(storage &data, const storage &bias, size_t n, size_t cols) {
    b200::check(silcu_bias_sigmoid_f32(b200::ptr<float>(data), b200::ptr<const float>(bias), n, cols,
                                       b200::stream()));
    b200::queued();
  }
  // The reference's CPU branch applies a folded affine with two roundings
  // below 5,000,000 elements and with fmaf above (include/array.h:2003-2015);
  // the same rule keeps GPU and CPU results equal.
  static void affine(const storage &IN, storage &OUT, size_t n, float scale, float offset) {
    b200::check(silcu_affine_f32(b200::ptr<const float>(IN), b200::ptr<float>(OUT), n, scale, offset,
                                 n >= 5000000 ? 1 : 0, b200::stream()));
    b200::queued();
  }

  // conv2d and its transpose helper are not part of this backend.
  template <class... A>
  static void conv2d(A &&...) {
    throw std::runtime_error("silarray b200: conv2d is not provided by this backend");
  }
  template <class... A>
  static void transpose(A &&...) {
    throw std::runtime_error("silarray b200: transpose kernel is not provided by this backend");
  }
};

using msl = gpu;
using mps = gpu;

inline void synchronize() { gpu_context::instance().flush(); }

};  // namespace sil

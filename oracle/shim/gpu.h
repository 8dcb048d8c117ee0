// Test infrastructure only: stand-in for silarray's Metal backend
// (include/gpu.h) in the CPU-only oracle build.  The oracle always runs with
// sil::use_cpu(); every gpu:: entry throws so that an accidental GPU dispatch
// is loud instead of silently computing something else.
#pragma once

#include <types.h>
#include <device.h>

#include <cstddef>
#include <stdexcept>

namespace sil {

[[noreturn]] inline void oracle_no_gpu_() {
  throw std::runtime_error("oracle build: the Metal backend is not available");
}

class gpu_context {
 public:
  static gpu_context &instance() {
    static gpu_context ctx;
    return ctx;
  }
  void flush() {}
};

class gpu {
 public:
  template <class T, class... A> static void add(A &&...) { oracle_no_gpu_(); }
  template <class T, class... A> static void sub(A &&...) { oracle_no_gpu_(); }
  template <class T, class... A> static void mul(A &&...) { oracle_no_gpu_(); }
  template <class T, class... A> static void div(A &&...) { oracle_no_gpu_(); }
  template <class T, class... A> static void pow(A &&...) { oracle_no_gpu_(); }
#define SIL_ORACLE_STUB(name) \
  template <class... A> static size_t name(A &&...) { oracle_no_gpu_(); }
  SIL_ORACLE_STUB(sigmoid)
  SIL_ORACLE_STUB(relu)
  SIL_ORACLE_STUB(sum_f32_num_tg)
  SIL_ORACLE_STUB(sum_f32)
  SIL_ORACLE_STUB(sum_axis0_f32)
  SIL_ORACLE_STUB(min_f32_num_tg)
  SIL_ORACLE_STUB(min_f32)
  SIL_ORACLE_STUB(max_f32_num_tg)
  SIL_ORACLE_STUB(max_f32)
  SIL_ORACLE_STUB(layer_norm)
  SIL_ORACLE_STUB(sgemm)
  SIL_ORACLE_STUB(sgemm_batched)
  SIL_ORACLE_STUB(sgemm_steel_batched)
  SIL_ORACLE_STUB(sgemv)
  SIL_ORACLE_STUB(sgemm_steel)
  SIL_ORACLE_STUB(sgemm_bias_steel)
  SIL_ORACLE_STUB(sgemm_bias_sigmoid_steel)
  SIL_ORACLE_STUB(conv2d)
  SIL_ORACLE_STUB(dot_f32_ex)
  SIL_ORACLE_STUB(argmax_f32)
  SIL_ORACLE_STUB(softmax)
  SIL_ORACLE_STUB(sigmoid_backward)
  SIL_ORACLE_STUB(bias_sigmoid)
  SIL_ORACLE_STUB(affine)
#undef SIL_ORACLE_STUB
};

using msl = gpu;
using mps = gpu;

inline void synchronize() {}

};  // namespace sil

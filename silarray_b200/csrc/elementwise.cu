// Elementwise kernels: binary ops with storage-length broadcasting, unary
// activations, the affine pass and the fused-chain interpreter.
//
// All of them are HBM-bound streams: 4 consecutive elements per thread with
// 128-bit loads/stores where the operand is contiguous and 16-byte aligned,
// grid sized to a multiple of the SM count (grid-stride loop).  Broadcast
// operands are indexed i % len as the reference's CPU loops do
// (include/cpu.h:76-237); one modulo per 4 elements, then wrap-increments.
#include "common.cuh"

namespace silcu {
namespace {

constexpr int kThreads = 256;

enum BinOp { kAdd = 0, kSub = 1, kMul = 2, kDiv = 3, kPow = 4 };

template <int OP>
__device__ __forceinline__ float bin(float x, float y) {
  if (OP == kAdd) return __fadd_rn(x, y);
  if (OP == kSub) return __fsub_rn(x, y);
  if (OP == kMul) return __fmul_rn(x, y);
  if (OP == kDiv) return __fdiv_rn(x, y);
  return powf(x, y);
}

// (int)std::pow(double(x), double(y)) as the reference's int path computes it
// (include/cpu.h:215-237), evaluated exactly: the power is an integer, so
// repeated multiplication in double is exact while it stays below 2^53, and
// any result outside int32 converts like x86-64's cvttsd2si (INT32_MIN).
__device__ __forceinline__ int32_t ipow_ref(int32_t x, int32_t y) {
  if (y < 0) {
    if (x == 1) return 1;
    if (x == -1) return (y & 1) ? -1 : 1;
    if (x == 0) return INT32_MIN;  // 1/0 = inf
    return 0;                      // |1/x^k| < 1 truncates to 0
  }
  double r = 1.0, b = double(x);
  uint32_t e = uint32_t(y);
  while (e) {
    if (e & 1u) r *= b;
    e >>= 1;
    if (e) b *= b;
    if (fabs(r) > 2147483648.0 || fabs(b) > 9.0e15) {
      // the exact result leaves int32 unless the remaining factors are +-1/0
      if (fabs(double(x)) > 1.0) return INT32_MIN;
    }
  }
  if (r >= 2147483648.0 || r < -2147483648.0) return INT32_MIN;
  return int32_t(r);
}

template <int OP>
__device__ __forceinline__ int32_t bin(int32_t x, int32_t y) {
  uint32_t ux = static_cast<uint32_t>(x), uy = static_cast<uint32_t>(y);
  if (OP == kAdd) return static_cast<int32_t>(ux + uy);
  if (OP == kSub) return static_cast<int32_t>(ux - uy);
  if (OP == kMul) return static_cast<int32_t>(ux * uy);
  if (OP == kDiv) return y == 0 ? 0 : (y == -1 ? static_cast<int32_t>(0u - ux) : x / y);
  return ipow_ref(x, y);
}

// Loads 4 values of a broadcast operand starting at logical index i.
template <typename T>
__device__ __forceinline__ void load4(const T *p, uint64_t len, uint64_t i, bool vec, T (&v)[4]) {
  if (len == 1) {
    T s = p[0];
    v[0] = v[1] = v[2] = v[3] = s;
    return;
  }
  uint64_t j = (len == 0xFFFFFFFFFFFFFFFFull) ? i : i % len;
  if (vec) {  // len % 4 == 0, pointer 16B aligned, i % 4 == 0 => j % 4 == 0
    static_assert(sizeof(T) == 4, "4-byte element types only");
    float4 f = *reinterpret_cast<const float4 *>(p + j);
    memcpy(v, &f, sizeof(f));
    return;
  }
#pragma unroll
  for (int k = 0; k < 4; k++) {
    v[k] = p[j];
    if (++j == len) j = 0;
  }
}

template <int OP, typename T>
__global__ void __launch_bounds__(kThreads) binary_kernel(const T *__restrict__ a, uint64_t la,
                                                          const T *__restrict__ b, uint64_t lb,
                                                          T *__restrict__ out, uint64_t n,
                                                          bool va, bool vb, bool vo) {
  const uint64_t stride = uint64_t(gridDim.x) * kThreads * 4;
  for (uint64_t i = (uint64_t(blockIdx.x) * kThreads + threadIdx.x) * 4; i < n; i += stride) {
    if (i + 4 <= n) {
      T x[4], y[4], r[4];
      load4(a, la == n ? 0xFFFFFFFFFFFFFFFFull : la, i, va, x);
      load4(b, lb == n ? 0xFFFFFFFFFFFFFFFFull : lb, i, vb, y);
#pragma unroll
      for (int k = 0; k < 4; k++) r[k] = bin<OP>(x[k], y[k]);
      if (vo) {
        float4 f;
        f.x = *reinterpret_cast<float *>(&r[0]);
        f.y = *reinterpret_cast<float *>(&r[1]);
        f.z = *reinterpret_cast<float *>(&r[2]);
        f.w = *reinterpret_cast<float *>(&r[3]);
        *reinterpret_cast<float4 *>(out + i) = f;
      } else {
#pragma unroll
        for (int k = 0; k < 4; k++) out[i + k] = r[k];
      }
    } else {
      for (uint64_t k = i; k < n; k++) out[k] = bin<OP>(a[k % la], b[k % lb]);
    }
  }
}

int grid_for(uint64_t n) {
  uint64_t want = (n + kThreads * 4 - 1) / (kThreads * 4);
  uint64_t cap = uint64_t(sm_count()) * 8;  // 8 resident CTAs of 256 threads per SM
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  return static_cast<int>(want);
}

template <int OP, typename T>
silcu_status launch_binary(const char *name, const T *a, size_t la, const T *b, size_t lb, T *out,
                           size_t n, silcu_stream stream) {
  if (n == 0) return SILCU_OK;
  if (!a || !b || !out || la == 0 || lb == 0)
    return fail(SILCU_INVALID_ARGUMENT, "%s: null pointer or empty operand", name);
  bool va = (la % 4 == 0) && aligned16(a);
  bool vb = (lb % 4 == 0) && aligned16(b);
  bool vo = aligned16(out);
  binary_kernel<OP, T><<<grid_for(n), kThreads, 0, as_stream(stream)>>>(a, la, b, lb, out, n, va, vb, vo);
  return check_launch(name);
}

// ------------------------------------------------------------------ unary
enum UnOp { kSigmoid = 0, kRelu = 1 };

template <int OP>
__global__ void __launch_bounds__(kThreads) unary_kernel(const float *__restrict__ in,
                                                         float *__restrict__ out, uint64_t n, bool vec) {
  const uint64_t stride = uint64_t(gridDim.x) * kThreads * 4;
  for (uint64_t i = (uint64_t(blockIdx.x) * kThreads + threadIdx.x) * 4; i < n; i += stride) {
    if (vec && i + 4 <= n) {
      float4 v = *reinterpret_cast<const float4 *>(in + i);
      float *e = &v.x;
#pragma unroll
      for (int k = 0; k < 4; k++) e[k] = OP == kSigmoid ? sigmoid_ref(e[k]) : (e[k] >= 0.0f ? e[k] : 0.0f);
      *reinterpret_cast<float4 *>(out + i) = v;
    } else {
      for (uint64_t k = i; k < n && k < i + 4; k++) {
        float x = in[k];
        out[k] = OP == kSigmoid ? sigmoid_ref(x) : (x >= 0.0f ? x : 0.0f);
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads) sigmoid_bwd_kernel(const float *__restrict__ dout,
                                                               const float *__restrict__ x,
                                                               float *__restrict__ out, uint64_t n) {
  const uint64_t stride = uint64_t(gridDim.x) * kThreads;
  for (uint64_t i = uint64_t(blockIdx.x) * kThreads + threadIdx.x; i < n; i += stride) {
    float s = sigmoid_ref(x[i]);
    out[i] = __fmul_rn(__fmul_rn(dout[i], s), __fsub_rn(1.0f, s));
  }
}

__global__ void __launch_bounds__(kThreads) bias_sigmoid_kernel(float *__restrict__ data,
                                                                const float *__restrict__ bias,
                                                                uint64_t n, uint64_t cols) {
  const uint64_t stride = uint64_t(gridDim.x) * kThreads;
  for (uint64_t i = uint64_t(blockIdx.x) * kThreads + threadIdx.x; i < n; i += stride)
    data[i] = sigmoid_ref(__fadd_rn(data[i], bias[i % cols]));
}

__global__ void __launch_bounds__(kThreads) affine_kernel(const float *__restrict__ in,
                                                          float *__restrict__ out, uint64_t n,
                                                          float scale, float offset, bool fused,
                                                          bool vec) {
  const uint64_t stride = uint64_t(gridDim.x) * kThreads * 4;
  for (uint64_t i = (uint64_t(blockIdx.x) * kThreads + threadIdx.x) * 4; i < n; i += stride) {
    if (vec && i + 4 <= n) {
      float4 v = *reinterpret_cast<const float4 *>(in + i);
      float *e = &v.x;
#pragma unroll
      for (int k = 0; k < 4; k++)
        e[k] = fused ? __fmaf_rn(e[k], scale, offset) : __fadd_rn(__fmul_rn(e[k], scale), offset);
      *reinterpret_cast<float4 *>(out + i) = v;
    } else {
      for (uint64_t k = i; k < n && k < i + 4; k++)
        out[k] = fused ? __fmaf_rn(in[k], scale, offset) : __fadd_rn(__fmul_rn(in[k], scale), offset);
    }
  }
}

// ------------------------------------------------------ fused interpreter
struct FusedParams {
  silcu_program prog;
  const float *in[SILCU_MAX_INPUTS];
  uint64_t len[SILCU_MAX_INPUTS];
  float *outs[SILCU_MAX_OUTPUTS];  // STORE targets
  int implicit_store;              // 1: the last instruction's dst goes to `out`
};

constexpr int kRegs = 8;

// The program is uniform across the grid, so every branch below is
// warp-uniform.  Registers live in shared memory (one float4 per thread per
// register) so that operand selection is an indexed 128-bit load instead of
// a chain of selects.
__global__ void __launch_bounds__(kThreads) fused_kernel(const __grid_constant__ FusedParams p,
                                                         float *__restrict__ out, uint64_t n) {
  __shared__ float4 regs[kRegs][kThreads];
  const uint64_t stride = uint64_t(gridDim.x) * kThreads * 4;
  const int last = p.prog.n_instr - 1;
  const int t = threadIdx.x;
  for (uint64_t i = (uint64_t(blockIdx.x) * kThreads + t) * 4; i < n; i += stride) {
    const int cnt = (i + 4 <= n) ? 4 : int(n - i);
    for (int pc = 0; pc < p.prog.n_instr; pc++) {
      const silcu_instr ins = p.prog.code[pc];
      float4 v;
      float *e = &v.x;
      if (ins.op == SILCU_OP_STORE) {
        const float4 r = regs[ins.a & (kRegs - 1)][t];
        float *dst = p.outs[ins.b & (SILCU_MAX_OUTPUTS - 1)];
        if (cnt == 4 && ((reinterpret_cast<uintptr_t>(dst + i) & 15) == 0)) {
          *reinterpret_cast<float4 *>(dst + i) = r;
        } else {
          const float *rr = &r.x;
          for (int k = 0; k < cnt; k++) dst[i + k] = rr[k];
        }
        continue;
      }
      if (ins.op == SILCU_OP_LOAD) {
        const float *src = p.in[ins.a];
        const uint64_t L = p.len[ins.a];
        if (L == n && cnt == 4 && ((reinterpret_cast<uintptr_t>(src + i) & 15) == 0)) {
          v = *reinterpret_cast<const float4 *>(src + i);
        } else if (L == 1) {
          e[0] = e[1] = e[2] = e[3] = src[0];
        } else {
          uint64_t j = (L == n) ? i : i % L;
#pragma unroll
          for (int k = 0; k < 4; k++) {
            e[k] = k < cnt ? src[j] : 0.0f;
            if (++j == L) j = 0;
          }
        }
      } else {
        const float4 xa = regs[ins.a & (kRegs - 1)][t];
        const float4 xb = regs[ins.b & (kRegs - 1)][t];
        const float *x = &xa.x, *y = &xb.x;
#pragma unroll
        for (int k = 0; k < 4; k++) {
          switch (ins.op) {
            case SILCU_OP_ADD: e[k] = __fadd_rn(x[k], y[k]); break;
            case SILCU_OP_SUB: e[k] = __fsub_rn(x[k], y[k]); break;
            case SILCU_OP_MUL: e[k] = __fmul_rn(x[k], y[k]); break;
            case SILCU_OP_DIV: e[k] = __fdiv_rn(x[k], y[k]); break;
            case SILCU_OP_POW: e[k] = powf(x[k], y[k]); break;
            case SILCU_OP_AFFINE: e[k] = __fadd_rn(__fmul_rn(x[k], ins.imm0), ins.imm1); break;
            case SILCU_OP_AFFINE_FMA: e[k] = __fmaf_rn(x[k], ins.imm0, ins.imm1); break;
            case SILCU_OP_SIGMOID: e[k] = sigmoid_ref(x[k]); break;
            case SILCU_OP_RELU: e[k] = x[k] >= 0.0f ? x[k] : 0.0f; break;
            case SILCU_OP_SIGMOID_BWD: {
              float sg = sigmoid_ref(y[k]);
              e[k] = __fmul_rn(__fmul_rn(x[k], sg), __fsub_rn(1.0f, sg));
              break;
            }
            case SILCU_OP_RDIV_IMM: e[k] = __fdiv_rn(ins.imm0, x[k]); break;
            default: e[k] = 0.0f; break;
          }
        }
      }
      regs[ins.dst & (kRegs - 1)][t] = v;
    }
    if (!p.implicit_store) continue;
    const float4 res = regs[p.prog.code[last].dst & (kRegs - 1)][t];
    if (cnt == 4 && ((reinterpret_cast<uintptr_t>(out + i) & 15) == 0)) {
      *reinterpret_cast<float4 *>(out + i) = res;
    } else {
      const float *r = &res.x;
      for (int k = 0; k < cnt; k++) out[i + k] = r[k];
    }
  }
}

}  // namespace
}  // namespace silcu

using namespace silcu;

extern "C" {

#define SILCU_BIN(NAME, OP, T)                                                                    \
  silcu_status silcu_##NAME(const T *a, size_t la, const T *b, size_t lb, T *out, size_t n,      \
                            silcu_stream s) {                                                     \
    return launch_binary<OP, T>(#NAME, a, la, b, lb, out, n, s);                                  \
  }
SILCU_BIN(add_f32, kAdd, float)
SILCU_BIN(sub_f32, kSub, float)
SILCU_BIN(mul_f32, kMul, float)
SILCU_BIN(div_f32, kDiv, float)
SILCU_BIN(pow_f32, kPow, float)
SILCU_BIN(add_i32, kAdd, int32_t)
SILCU_BIN(sub_i32, kSub, int32_t)
SILCU_BIN(mul_i32, kMul, int32_t)
SILCU_BIN(div_i32, kDiv, int32_t)
SILCU_BIN(pow_i32, kPow, int32_t)
#undef SILCU_BIN

silcu_status silcu_sigmoid_f32(const float *in, float *out, size_t n, silcu_stream s) {
  if (n == 0) return SILCU_OK;
  if (!in || !out) return fail(SILCU_INVALID_ARGUMENT, "sigmoid: null pointer");
  unary_kernel<kSigmoid><<<grid_for(n), kThreads, 0, as_stream(s)>>>(in, out, n, aligned16(in) && aligned16(out));
  return check_launch("sigmoid");
}

silcu_status silcu_relu_f32(const float *in, float *out, size_t n, silcu_stream s) {
  if (n == 0) return SILCU_OK;
  if (!in || !out) return fail(SILCU_INVALID_ARGUMENT, "relu: null pointer");
  unary_kernel<kRelu><<<grid_for(n), kThreads, 0, as_stream(s)>>>(in, out, n, aligned16(in) && aligned16(out));
  return check_launch("relu");
}

silcu_status silcu_sigmoid_backward_f32(const float *dout, const float *x, float *out, size_t n,
                                        silcu_stream s) {
  if (n == 0) return SILCU_OK;
  if (!dout || !x || !out) return fail(SILCU_INVALID_ARGUMENT, "sigmoid_backward: null pointer");
  sigmoid_bwd_kernel<<<grid_for(n * 4), kThreads, 0, as_stream(s)>>>(dout, x, out, n);
  return check_launch("sigmoid_backward");
}

silcu_status silcu_bias_sigmoid_f32(float *data, const float *bias, size_t n, size_t cols,
                                    silcu_stream s) {
  if (n == 0) return SILCU_OK;
  if (!data || !bias || cols == 0) return fail(SILCU_INVALID_ARGUMENT, "bias_sigmoid: bad argument");
  bias_sigmoid_kernel<<<grid_for(n * 4), kThreads, 0, as_stream(s)>>>(data, bias, n, cols);
  return check_launch("bias_sigmoid");
}

silcu_status silcu_affine_f32(const float *in, float *out, size_t n, float scale, float offset,
                              int fused, silcu_stream s) {
  if (n == 0) return SILCU_OK;
  if (!in || !out) return fail(SILCU_INVALID_ARGUMENT, "affine: null pointer");
  affine_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(in, out, n, scale, offset, fused != 0,
                                                            aligned16(in) && aligned16(out));
  return check_launch("affine");
}

static silcu_status fused_launch(const char *what, const silcu_program *prog, const float *const *inputs,
                                 const size_t *lens, float *const *outs, int n_outs, float *out, size_t n,
                                 silcu_stream s) {
  if (n == 0) return SILCU_OK;
  if (!prog || prog->n_instr <= 0 || prog->n_instr > SILCU_MAX_PROGRAM || prog->n_inputs < 0 ||
      prog->n_inputs > SILCU_MAX_INPUTS)
    return fail(SILCU_INVALID_ARGUMENT, "%s: bad program", what);
  FusedParams p;
  memset(&p, 0, sizeof(p));
  p.prog = *prog;
  for (int j = 0; j < prog->n_inputs; j++) {
    if (!inputs[j] || lens[j] == 0) return fail(SILCU_INVALID_ARGUMENT, "%s: input %d empty", what, j);
    p.in[j] = inputs[j];
    p.len[j] = lens[j];
  }
  for (int j = 0; j < n_outs; j++) {
    if (!outs[j]) return fail(SILCU_INVALID_ARGUMENT, "%s: output %d is null", what, j);
    p.outs[j] = outs[j];
  }
  p.implicit_store = out != nullptr;
  for (int pc = 0; pc < prog->n_instr; pc++) {
    const silcu_instr &ins = prog->code[pc];
    if (ins.op == SILCU_OP_STORE) {
      if (out || ins.a < 0 || ins.a >= kRegs || ins.b < 0 || ins.b >= n_outs)
        return fail(SILCU_INVALID_ARGUMENT, "%s: bad store %d", what, pc);
      continue;
    }
    if (ins.dst < 0 || ins.dst >= kRegs || ins.op < 0 || ins.op > SILCU_OP_RDIV_IMM ||
        (ins.op != SILCU_OP_LOAD && (ins.a < 0 || ins.a >= kRegs || ins.b < 0 || ins.b >= kRegs)))
      return fail(SILCU_INVALID_ARGUMENT, "%s: bad instruction %d", what, pc);
    if (ins.op == SILCU_OP_LOAD && (ins.a < 0 || ins.a >= prog->n_inputs))
      return fail(SILCU_INVALID_ARGUMENT, "%s: instruction %d loads a missing input", what, pc);
  }
  fused_kernel<<<grid_for(n), kThreads, 0, as_stream(s)>>>(p, out, n);
  return check_launch(what);
}

silcu_status silcu_fused_f32(const silcu_program *prog, const float *const *inputs,
                             const size_t *lens, float *out, size_t n, silcu_stream s) {
  if (!out) return fail(SILCU_INVALID_ARGUMENT, "fused: null output");
  return fused_launch("fused", prog, inputs, lens, nullptr, 0, out, n, s);
}

silcu_status silcu_fused_multi_f32(const silcu_program *prog, const float *const *inputs, const size_t *lens,
                                   float *const *outputs, int n_outputs, size_t n, silcu_stream s) {
  if (n_outputs < 1 || n_outputs > SILCU_MAX_OUTPUTS || !outputs)
    return fail(SILCU_INVALID_ARGUMENT, "fused_multi: 1..%d outputs", SILCU_MAX_OUTPUTS);
  return fused_launch("fused_multi", prog, inputs, lens, outputs, n_outputs, nullptr, n, s);
}

}  // extern "C"

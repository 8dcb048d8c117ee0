// Test double of libsilcu for the CPU tests of the drop-in host layer: the
// elementwise entry points, the fused interpreter (silcu_fused_multi_f32 with
// the STORE instruction), the reductions, the row ops, a plain-loop GEMM and
// the bookkeeping calls, as host loops with the same launch counting as the
// library (values agree with it to rounding, not bit for bit).  Used only by
// tests/test_dropin_host.py.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "silcu.h"

static unsigned long long g_launches = 0;
static char g_msg[256] = "";

static silcu_status fail(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return SILCU_INVALID_ARGUMENT;
}

static float sigm(float x) { return 1.0f / (std::exp(-x) + 1.0f); }

template <class T, class F>
static silcu_status binary(const T *a, size_t la, const T *b, size_t lb, T *o, size_t n, F f) {
  if (!a || !b || !o || !la || !lb) return fail("binary: null or empty operand");
  for (size_t i = 0; i < n; i++) o[i] = f(a[i % la], b[i % lb]);
  g_launches++;
  return SILCU_OK;
}

extern "C" {
const char *silcu_last_error(void) { return g_msg; }
int silcu_abi_version(void) { return 0; }
unsigned long long silcu_kernel_launches(void) { return g_launches; }
silcu_status silcu_synchronize(silcu_stream) { return SILCU_OK; }
silcu_status silcu_device_status(silcu_stream) { return SILCU_OK; }

#define BIN(NAME, T, EXPR)                                                                          \
  silcu_status silcu_##NAME(const T *a, size_t la, const T *b, size_t lb, T *o, size_t n, silcu_stream) { \
    return binary<T>(a, la, b, lb, o, n, [](T x, T y) -> T { return EXPR; });                       \
  }
BIN(add_f32, float, x + y)
BIN(sub_f32, float, x - y)
BIN(mul_f32, float, x * y)
BIN(div_f32, float, x / y)
BIN(pow_f32, float, std::pow(x, y))
BIN(add_i32, int32_t, int32_t(uint32_t(x) + uint32_t(y)))
BIN(sub_i32, int32_t, int32_t(uint32_t(x) - uint32_t(y)))
BIN(mul_i32, int32_t, int32_t(uint32_t(x) * uint32_t(y)))
BIN(div_i32, int32_t, y ? x / y : 0)
BIN(pow_i32, int32_t, int32_t(std::pow(double(x), double(y))))
#undef BIN

silcu_status silcu_sigmoid_f32(const float *in, float *out, size_t n, silcu_stream) {
  for (size_t i = 0; i < n; i++) out[i] = sigm(in[i]);
  g_launches++;
  return SILCU_OK;
}
silcu_status silcu_relu_f32(const float *in, float *out, size_t n, silcu_stream) {
  for (size_t i = 0; i < n; i++) out[i] = in[i] >= 0.0f ? in[i] : 0.0f;
  g_launches++;
  return SILCU_OK;
}
silcu_status silcu_sigmoid_backward_f32(const float *dout, const float *x, float *out, size_t n, silcu_stream) {
  for (size_t i = 0; i < n; i++) {
    const float s = sigm(x[i]);
    out[i] = (dout[i] * s) * (1.0f - s);
  }
  g_launches++;
  return SILCU_OK;
}
silcu_status silcu_bias_sigmoid_f32(float *d, const float *b, size_t n, size_t cols, silcu_stream) {
  for (size_t i = 0; i < n; i++) d[i] = sigm(d[i] + b[i % cols]);
  g_launches++;
  return SILCU_OK;
}
silcu_status silcu_affine_f32(const float *in, float *out, size_t n, float s, float o, int fused, silcu_stream) {
  for (size_t i = 0; i < n; i++) out[i] = fused ? std::fma(in[i], s, o) : in[i] * s + o;
  g_launches++;
  return SILCU_OK;
}

static silcu_status interpret(const silcu_program *p, const float *const *in, const size_t *lens, float *const *outs,
                              int n_outs, float *out, size_t n) {
  for (int j = 0; j < p->n_inputs; j++)
    if (!in[j] || !lens[j]) return fail("fused: input %d empty", j);
  for (size_t i = 0; i < n; i++) {
    float r[8] = {0};
    for (int pc = 0; pc < p->n_instr; pc++) {
      const silcu_instr &s = p->code[pc];
      const float x = r[s.a & 7], y = r[s.b & 7];
      float v = 0.0f;
      switch (s.op) {
        case SILCU_OP_STORE:
          if (s.b < 0 || s.b >= n_outs) return fail("fused: bad store");
          outs[s.b][i] = r[s.a & 7];
          continue;
        case SILCU_OP_LOAD: v = in[s.a][i % lens[s.a]]; break;
        case SILCU_OP_ADD: v = x + y; break;
        case SILCU_OP_SUB: v = x - y; break;
        case SILCU_OP_MUL: v = x * y; break;
        case SILCU_OP_DIV: v = x / y; break;
        case SILCU_OP_POW: v = std::pow(x, y); break;
        case SILCU_OP_AFFINE: v = x * s.imm0 + s.imm1; break;
        case SILCU_OP_AFFINE_FMA: v = std::fma(x, s.imm0, s.imm1); break;
        case SILCU_OP_SIGMOID: v = sigm(x); break;
        case SILCU_OP_RELU: v = x >= 0.0f ? x : 0.0f; break;
        case SILCU_OP_SIGMOID_BWD: {
          const float sg = sigm(y);
          v = (x * sg) * (1.0f - sg);
          break;
        }
        case SILCU_OP_RDIV_IMM: v = s.imm0 / x; break;
        default: return fail("fused: bad opcode");
      }
      r[s.dst & 7] = v;
    }
    if (out) out[i] = r[p->code[p->n_instr - 1].dst & 7];
  }
  g_launches++;
  return SILCU_OK;
}

silcu_status silcu_fused_f32(const silcu_program *p, const float *const *in, const size_t *lens, float *out, size_t n,
                             silcu_stream) {
  return interpret(p, in, lens, nullptr, 0, out, n);
}
silcu_status silcu_fused_multi_f32(const silcu_program *p, const float *const *in, const size_t *lens,
                                   float *const *outs, int n_outs, size_t n, silcu_stream) {
  return interpret(p, in, lens, outs, n_outs, nullptr, n);
}

size_t silcu_reduce_workspace_bytes(size_t) { return 0; }
silcu_status silcu_sum_f32(const float *in, size_t n, float *out, void *, size_t, silcu_stream) {
  double s = 0;
  for (size_t i = 0; i < n; i++) s += in[i];
  *out = float(s);
  g_launches++;
  return SILCU_OK;
}

silcu_status silcu_min_f32(const float *in, size_t n, float *out, void *, size_t, silcu_stream) {
  float m = in[0];
  for (size_t i = 1; i < n; i++) m = in[i] < m ? in[i] : m;
  *out = m;
  g_launches++;
  return SILCU_OK;
}
silcu_status silcu_max_f32(const float *in, size_t n, float *out, void *, size_t, silcu_stream) {
  float m = in[0];
  for (size_t i = 1; i < n; i++) m = in[i] > m ? in[i] : m;
  *out = m;
  g_launches++;
  return SILCU_OK;
}
silcu_status silcu_softmax_f32(const float *in, float *out, size_t rows, size_t cols, silcu_stream) {
  for (size_t r = 0; r < rows; r++) {
    const float *x = in + r * cols;
    float *y = out + r * cols;
    float m = x[0], s = 0.0f;
    for (size_t c = 1; c < cols; c++) m = x[c] > m ? x[c] : m;
    for (size_t c = 0; c < cols; c++) s += (y[c] = std::exp(x[c] - m));
    const float inv = 1.0f / s;
    for (size_t c = 0; c < cols; c++) y[c] *= inv;
  }
  g_launches++;
  return SILCU_OK;
}
silcu_status silcu_layer_norm_f32(const float *in, float *out, const float *g, const float *b, size_t rows,
                                  size_t cols, float eps, silcu_stream) {
  for (size_t r = 0; r < rows; r++) {
    const float *x = in + r * cols;
    float mu = 0.0f, ss = 0.0f;
    for (size_t c = 0; c < cols; c++) mu += x[c];
    mu /= float(cols);
    for (size_t c = 0; c < cols; c++) ss += (x[c] - mu) * (x[c] - mu);
    const float inv = 1.0f / std::sqrt(ss / float(cols) + eps);
    for (size_t c = 0; c < cols; c++) out[r * cols + c] = (x[c] - mu) * inv * g[c] + b[c];
  }
  g_launches++;
  return SILCU_OK;
}
silcu_status silcu_argmax_f32(const float *in, int32_t *out, size_t rows, size_t cols, void *, size_t, silcu_stream) {
  for (size_t r = 0; r < rows; r++) {
    float bv = 1.17549435e-38f;
    int32_t bi = 0;
    for (size_t c = 0; c < cols; c++)
      if (in[r * cols + c] > bv) bv = in[r * cols + c], bi = int32_t(c);
    out[r] = bi;
  }
  g_launches++;
  return SILCU_OK;
}
silcu_status silcu_sum_axis_f32(const float *in, float *out, size_t outer, size_t len, size_t inner, void *, size_t,
                                silcu_stream) {
  for (size_t o = 0; o < outer; o++)
    for (size_t i = 0; i < inner; i++) {
      double s = 0;
      for (size_t l = 0; l < len; l++) s += in[(o * len + l) * inner + i];
      out[o * inner + i] = float(s);
    }
  g_launches++;
  return SILCU_OK;
}
// Plain loops over the general GEMM arguments (fp32 operands only).
silcu_status silcu_sgemm_ex(const silcu_gemm_args *ap, void *, size_t, silcu_stream) {
  const silcu_gemm_args &a = *ap;
  if (!a.A || !a.B || !a.C) return fail("sgemm: the host double takes plain fp32 operands only");
  const int64_t bin = a.batch_inner > 1 ? a.batch_inner : 1;
  for (int64_t bo = 0; bo < a.batch; bo++)
    for (int64_t bi = 0; bi < bin; bi++) {
      const float *A = a.A + bo * a.stride_a + bi * a.stride_a_inner;
      const float *B = a.B + bo * a.stride_b + bi * a.stride_b_inner;
      float *C = a.C + bo * a.stride_c + bi * a.stride_c_inner;
      for (int64_t m = 0; m < a.M; m++)
        for (int64_t n = 0; n < a.N; n++) {
          double acc = 0;
          for (int64_t k = 0; k < a.K; k++)
            acc += double(a.trans_a ? A[k * a.lda + m] : A[m * a.lda + k]) *
                   double(a.trans_b ? B[n * a.ldb + k] : B[k * a.ldb + n]);
          float v = float(acc);
          if (a.alpha != 1.0f) v *= a.alpha;
          if (a.bias) v += a.bias[n % (a.bias_len > 0 ? a.bias_len : 1)];
          if (a.act == SILCU_ACT_RELU) v = v >= 0.0f ? v : 0.0f;
          else if (a.act == SILCU_ACT_SIGMOID) v = sigm(v);
          if (a.residual) v += a.residual[m * a.ldr + n];
          C[m * a.ldc + n] = v;
        }
    }
  g_launches++;
  return SILCU_OK;
}
size_t silcu_conv2d_workspace_bytes(uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t) { return 0; }
silcu_status silcu_conv2d_f32(const float *in, const float *w, float *out, uint32_t N, uint32_t H, uint32_t W,
                              uint32_t C, uint32_t K, uint32_t Co, void *, size_t, silcu_stream) {
  const long pad = long(K / 2);
  for (size_t m = 0; m < size_t(N) * H * W; m++) {
    const size_t n = m / (size_t(H) * W), sp = m % (size_t(H) * W), oh = sp / W, ow = sp % W;
    for (size_t co = 0; co < Co; co++) {
      double s = 0;
      for (size_t kh = 0; kh < K; kh++)
        for (size_t kw = 0; kw < K; kw++) {
          const long ih = long(oh + kh) - pad, iw = long(ow + kw) - pad;
          if (ih < 0 || ih >= long(H) || iw < 0 || iw >= long(W)) continue;
          for (size_t ci = 0; ci < C; ci++)
            s += double(in[((n * H + size_t(ih)) * W + size_t(iw)) * C + ci]) * double(w[((co * K + kh) * K + kw) * C + ci]);
        }
      out[m * Co + co] = float(s);
    }
  }
  g_launches++;
  return SILCU_OK;
}
silcu_status silcu_sum_axis_seq_f32(const float *in, float *out, size_t outer, size_t len, size_t inner, silcu_stream) {
  for (size_t o = 0; o < outer; o++)
    for (size_t i = 0; i < inner; i++) {
      float s = 0.0f;
      for (size_t l = 0; l < len; l++) s += in[(o * len + l) * inner + i];
      out[o * inner + i] = s;
    }
  g_launches++;
  return SILCU_OK;
}
size_t silcu_argmax_workspace_bytes(size_t, size_t) { return 0; }
size_t silcu_sum_axis_workspace_bytes(size_t, size_t, size_t) { return 0; }
size_t silcu_sgemm_workspace_bytes(const silcu_gemm_args *) { return 0; }
}

/* Test infrastructure only: the parity oracle.  Never linked into, loaded by
 * or called from the product path (silarray_b200/ and include/); only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg use it.
 *
 * A plain-C restatement of silarray's CPU backend for the hot path, one
 * function per reference routine, each citing the reference file:line it
 * follows.  Arithmetic is IEEE fp32 in the reference's evaluation order; the
 * file is compiled with -ffp-contract=off so no multiply-add is fused unless
 * the reference fuses it (cpu::affine's vfmaq_f32).
 *
 * Pinned against: (1) the reference's own doctest suite (test/test_array.cpp),
 * which passes 45/45 on the reference CPU build in oracle/_ref, and (2) that
 * build itself, function by function, in tests/test_oracle.py; the golden
 * vectors in tests/golden/ come from the reference build via
 * tests/golden/make_golden.py.
 *
 * Where the reference calls a closed library whose summation order is not
 * published (Accelerate vDSP_sve/vDSP_dotpr, cblas_sgemm), this file sums
 * sequentially in fp32 (vDSP stand-in) or, for GEMM, in fp64 rounded once.
 */
#include <float.h>
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

enum { ORC_ADD = 0, ORC_SUB = 1, ORC_MUL = 2, ORC_DIV = 3, ORC_POW = 4 };

/* cpu::add/sub/mul/div/pow<float> (include/cpu.h:76-237): every branch of
 * the vDSP fast paths computes out[i] = a[i % len_a] (op) b[i % len_b] over
 * the storage lengths; pow is powf (vvpowf / std::pow(float, float)). */
void orc_binary_f32(int op, const float *a, size_t la, const float *b,
                    size_t lb, float *out, size_t n) {
  for (size_t i = 0; i < n; i++) {
    float x = a[i % la], y = b[i % lb];
    switch (op) {
      case ORC_ADD: out[i] = x + y; break;
      case ORC_SUB: out[i] = x - y; break;
      case ORC_MUL: out[i] = x * y; break;
      case ORC_DIV: out[i] = x / y; break;
      default: out[i] = powf(x, y); break;
    }
  }
}

/* cpu::add..pow<int> (include/cpu.h:76-237, generic loops): 32-bit wrapping
 * arithmetic, truncating division, pow = (int)std::pow(double, double). */
void orc_binary_i32(int op, const int32_t *a, size_t la, const int32_t *b,
                    size_t lb, int32_t *out, size_t n) {
  for (size_t i = 0; i < n; i++) {
    int32_t x = a[i % la], y = b[i % lb];
    switch (op) {
      case ORC_ADD: out[i] = (int32_t)((uint32_t)x + (uint32_t)y); break;
      case ORC_SUB: out[i] = (int32_t)((uint32_t)x - (uint32_t)y); break;
      case ORC_MUL: out[i] = (int32_t)((uint32_t)x * (uint32_t)y); break;
      case ORC_DIV: out[i] = y ? x / y : 0; break;
      default: out[i] = (int32_t)pow((double)x, (double)y); break;
    }
  }
}

/* One scalar operation on an evaluated vector, as the lazy evaluator runs it
 * (include/array.h:1888-1940 folds it to out = x * scale + offset, and
 * 1989-2023 applies it):
 *   x + r  -> scale 1, offset r          x - r -> scale 1, offset -r
 *   x * r  -> scale r, offset 0          x / r -> scale 1/r, offset 0
 *   l + x  -> scale 1, offset l          l - x -> scale -1, offset l
 *   l * x  -> scale l, offset 0          l / x -> not affine: l / x[i]
 * Application (2003-2015): n >= 5,000,000 -> fmaf (NEON, cpu.h:329-350);
 * else the vDSP branch picked by which of scale/offset is trivial.
 * Because the evaluator visits nodes in topological order, every node's
 * inputs are already evaluated, so each scalar node is one such pass. */
void orc_scalar_op_f32(int op, float s, int left, const float *x, float *out,
                       size_t n) {
  float scale = 1.0f, offset = 0.0f;
  if (left && op == ORC_DIV) {
    for (size_t i = 0; i < n; i++) out[i] = s / x[i];
    return;
  }
  if (!left) {
    switch (op) {
      case ORC_ADD: offset = s; break;
      case ORC_SUB: offset = -s; break;
      case ORC_MUL: scale = s; offset = 0.0f * s; break;
      default: scale = 1.0f / s; offset = 0.0f / s; break;
    }
  } else {
    switch (op) {
      case ORC_ADD: offset = s; break;
      case ORC_SUB: scale = -1.0f; offset = s - 0.0f; break;
      default: scale = s; offset = 0.0f * s; break;
    }
  }
  if (n >= 5000000) {
    for (size_t i = 0; i < n; i++) out[i] = fmaf(x[i], scale, offset);
  } else if (scale == 1.0f && offset == 0.0f) {
    memcpy(out, x, n * sizeof(float));
  } else if (offset == 0.0f) {
    for (size_t i = 0; i < n; i++) out[i] = x[i] * scale;
  } else if (scale == 1.0f) {
    for (size_t i = 0; i < n; i++) out[i] = x[i] + offset;
  } else {
    for (size_t i = 0; i < n; i++) {
      volatile float p = x[i] * scale;
      out[i] = p + offset;
    }
  }
}

/* cpu::sigmoid (include/cpu.h:290-297): negate, expf, add 1, reciprocal. */
void orc_sigmoid_f32(const float *x, float *y, size_t n) {
  for (size_t i = 0; i < n; i++) {
    float t = expf(-x[i]);
    t = t + 1.0f;
    y[i] = 1.0f / t;
  }
}

/* cpu::relu (include/cpu.h:324-327): vDSP_vthres with threshold 0. */
void orc_relu_f32(const float *x, float *y, size_t n) {
  for (size_t i = 0; i < n; i++) y[i] = x[i] >= 0.0f ? x[i] : 0.0f;
}

/* cpu::sigmoid_backward (include/cpu.h:299-308): s = sigmoid(x),
 * out = dout * s * (1 - s), evaluated left to right. */
void orc_sigmoid_backward_f32(const float *dout, const float *x, float *y,
                              size_t n) {
  for (size_t i = 0; i < n; i++) {
    float t = expf(-x[i]);
    t = t + 1.0f;
    float s = 1.0f / t;
    float p = dout[i] * s;
    y[i] = p * (1.0f - s);
  }
}

/* cpu::bias_sigmoid (include/cpu.h:310-322): in place x += bias[i % cols],
 * then sigmoid. */
void orc_bias_sigmoid_f32(float *x, const float *bias, size_t n, size_t cols) {
  for (size_t i = 0; i < n; i++) {
    float v = x[i] + bias[i % cols];
    float t = expf(-v);
    t = t + 1.0f;
    x[i] = 1.0f / t;
  }
}

/* cpu::layer_norm (include/cpu.h:352-373), per row: mu = (sequential sum)/cols;
 * d = x - mu; ss = sequential sum of d*d; inv = 1/sqrtf(ss/cols + eps);
 * y = ((d * inv) * gamma) + beta. */
void orc_layer_norm_f32(const float *x, float *y, const float *g,
                        const float *b, size_t rows, size_t cols, float eps) {
  for (size_t r = 0; r < rows; r++) {
    const float *row = x + r * cols;
    float *o = y + r * cols;
    float s = 0.0f;
    for (size_t c = 0; c < cols; c++) s += row[c];
    float mu = s / (float)cols;
    float ss = 0.0f;
    for (size_t c = 0; c < cols; c++) {
      o[c] = row[c] + (-mu);
      volatile float p = o[c] * o[c];
      ss += p;
    }
    float inv = 1.0f / sqrtf(ss / (float)cols + eps);
    for (size_t c = 0; c < cols; c++) {
      float t = o[c] * inv;
      t = t * g[c];
      o[c] = t + b[c];
    }
  }
}

/* 2-D softmax, CPU branch (include/array.h:2139-2150): per row subtract the
 * row MIN (not the max), e = expf(x - min), s = sequential sum of e, then
 * e / s folded by the affine pass into e * (1/s). */
void orc_softmax_f32(const float *x, float *y, size_t rows, size_t cols) {
  for (size_t r = 0; r < rows; r++) {
    const float *row = x + r * cols;
    float *o = y + r * cols;
    float m = INFINITY;
    for (size_t c = 0; c < cols; c++)
      if (row[c] < m) m = row[c];
    float s = 0.0f;
    for (size_t c = 0; c < cols; c++) {
      o[c] = expf(row[c] - m);
      s += o[c];
    }
    float inv = 1.0f / s;
    for (size_t c = 0; c < cols; c++) o[c] = o[c] * inv;
  }
}

/* argmax, CPU branch (include/array.h:1728-1746): strict '>' so the first
 * index wins ties; the running maximum starts at FLT_MIN (the smallest
 * positive normal, numeric_limits<float>::min()), so a row whose values are
 * all <= FLT_MIN yields index 0. */
void orc_argmax_f32(const float *x, int32_t *idx, size_t rows, size_t cols) {
  for (size_t r = 0; r < rows; r++) {
    float m = FLT_MIN;
    size_t k = 0;
    for (size_t c = 0; c < cols; c++)
      if (x[r * cols + c] > m) { m = x[r * cols + c]; k = c; }
    idx[r] = (int32_t)k;
  }
}

/* argmax on int arrays (same loop; numeric_limits<int>::min() start). */
void orc_argmax_i32(const int32_t *x, int32_t *idx, size_t rows, size_t cols) {
  for (size_t r = 0; r < rows; r++) {
    int32_t m = INT32_MIN;
    size_t k = 0;
    for (size_t c = 0; c < cols; c++)
      if (x[r * cols + c] > m) { m = x[r * cols + c]; k = c; }
    idx[r] = (int32_t)k;
  }
}

/* array<float>::sum() CPU branch -> cpu::sum -> vDSP_sve (include/array.h:
 * 1526-1532, cpu.h:266-274): sequential fp32. */
float orc_sum_f32(const float *x, size_t n) {
  float s = 0.0f;
  for (size_t i = 0; i < n; i++) s += x[i];
  return s;
}

/* array<int>::sum(): std::accumulate in int (cpu.h:273), wrapping. */
int32_t orc_sum_i32(const int32_t *x, size_t n) {
  uint32_t s = 0;
  for (size_t i = 0; i < n; i++) s += (uint32_t)x[i];
  return (int32_t)s;
}

/* min()/max() CPU branch: vDSP_minvi / vDSP_maxvi over the storage
 * (include/array.h:1604-1609, 1634-1639). */
float orc_min_f32(const float *x, size_t n) {
  float m = INFINITY;
  for (size_t i = 0; i < n; i++)
    if (x[i] < m) m = x[i];
  return m;
}
float orc_max_f32(const float *x, size_t n) {
  float m = -INFINITY;
  for (size_t i = 0; i < n; i++)
    if (x[i] > m) m = x[i];
  return m;
}

/* sum(axis) on a contiguous array viewed as [outer, len, inner]
 * (include/array.h:2275-2319): axis 0 of a 2-D array uses cpu::sum_axis0
 * (row-by-row vDSP_vadd, cpu.h:276-288); every other case walks positions in
 * row-major order with tmp.at(p) += at(pos).  Both add the elements of one
 * output in increasing index order along the axis, in fp32. */
void orc_sum_axis_f32(const float *x, float *y, size_t outer, size_t len,
                      size_t inner) {
  for (size_t o = 0; o < outer; o++)
    for (size_t i = 0; i < inner; i++) {
      float s = 0.0f;
      for (size_t k = 0; k < len; k++) s += x[(o * len + k) * inner + i];
      y[o * inner + i] = s;
    }
}

void orc_sum_axis_i32(const int32_t *x, int32_t *y, size_t outer, size_t len,
                      size_t inner) {
  for (size_t o = 0; o < outer; o++)
    for (size_t i = 0; i < inner; i++) {
      uint32_t s = 0;
      for (size_t k = 0; k < len; k++) s += (uint32_t)x[(o * len + k) * inner + i];
      y[o * inner + i] = (int32_t)s;
    }
}

/* dot<float> (include/array.h:2632-2655): cblas_sgemm(RowMajor, tA, tB, ...)
 * with lda/ldb taken from the strides.  cblas' summation order is not
 * specified, so this restatement accumulates in fp64 and rounds once; the
 * parity tolerance (sqrt(K)-scaled) absorbs the order difference.
 * A is [M,K] (lda) or, when tA, stored [K,M]; B is [K,N] or, when tB, [N,K].
 * Rows [row0, row1) of C only, so large cases can be spot-checked. */
void orc_sgemm_rows(const float *A, const float *B, float *C, size_t M,
                    size_t N, size_t K, size_t lda, size_t ldb, int tA, int tB,
                    size_t row0, size_t row1) {
  (void)M;
  for (size_t i = row0; i < row1; i++)
    for (size_t j = 0; j < N; j++) {
      double s = 0.0;
      for (size_t k = 0; k < K; k++) {
        double a = tA ? A[k * lda + i] : A[i * lda + k];
        double b = tB ? B[j * ldb + k] : B[k * ldb + j];
        s += a * b;
      }
      C[(i - row0) * N + j] = (float)s;
    }
}

/* dot<int> (include/cpu.h:250-263): i-k-j loop, 32-bit wrapping. */
void orc_dot_i32(const int32_t *A, const int32_t *B, int32_t *C, size_t M,
                 size_t N, size_t K) {
  memset(C, 0, M * N * sizeof(int32_t));
  for (size_t i = 0; i < M; i++)
    for (size_t k = 0; k < K; k++) {
      uint32_t a = (uint32_t)A[i * K + k];
      for (size_t j = 0; j < N; j++)
        C[i * N + j] = (int32_t)((uint32_t)C[i * N + j] + a * (uint32_t)B[k * N + j]);
    }
}

/* conv2d (array::conv2d, include/array.h:1508-1519 and 2259-2273; gpu::conv2d,
 * include/gpu.h:815-833 with the padding K/2 of gpu.h:713, 1202-1204): NHWC
 * input [N,H,W,C], OHWI weight [C_out,K,K,C], stride 1, zero padding K/2,
 * NHWC output [N,H,W,C_out].  The reference has no CPU path for conv2d (its
 * benchmark notes "GPU only"), so this restates the GPU kernels' arithmetic:
 * a dot product over (kh, kw, ci) per output, accumulated in fp64 and
 * rounded once, like orc_sgemm_rows.  Rows [m0, m1) of the N*H*W output
 * pixels only. */
void orc_conv2d_f32(const float *in, const float *w, float *out, size_t N, size_t H, size_t W, size_t C,
                    size_t K, size_t C_out, size_t m0, size_t m1) {
  (void)N;
  const long pad = (long)(K / 2);
  for (size_t m = m0; m < m1; m++) {
    const size_t n = m / (H * W), sp = m % (H * W), oh = sp / W, ow = sp % W;
    for (size_t co = 0; co < C_out; co++) {
      double s = 0.0;
      for (size_t kh = 0; kh < K; kh++) {
        const long ih = (long)oh + (long)kh - pad;
        if (ih < 0 || ih >= (long)H) continue;
        for (size_t kw = 0; kw < K; kw++) {
          const long iw = (long)ow + (long)kw - pad;
          if (iw < 0 || iw >= (long)W) continue;
          const float *x = in + ((n * H + (size_t)ih) * W + (size_t)iw) * C;
          const float *f = w + ((co * K + kh) * K + kw) * C;
          for (size_t ci = 0; ci < C; ci++) s += (double)x[ci] * (double)f[ci];
        }
      }
      out[(m - m0) * C_out + co] = (float)s;
    }
  }
}

// conv2d as an implicit GEMM on the 3xTF32 tensor-core path.
//
// Semantics of the reference (array::conv2d, include/array.h:1508-1519, eval
// 2259-2273; gpu::conv2d, include/gpu.h:815-833 and the kernels of
// include/gpu_kernels.metal:1530-2077): input NHWC [N, H, W, C_in], weight
// OHWI [C_out, K, K, C_in], stride 1, zero padding K / 2 on every side,
// output NHWC [N, H, W, C_out], no bias:
//   out[n, oh, ow, co] = sum over (kh, kw, ci) of
//       in[n, oh + kh - K/2, ow + kw - K/2, ci] * w[co, kh, kw, ci]
// (terms outside the image are zero).  As a GEMM: M = N*H*W rows (output
// pixels), N = C_out, K_dim = K*K*C_in in (kh, kw, ci) order -- the weight
// rows [C_out, K_dim] are already the K-major B operand.
//
// One pass writes the patch matrix of the output pixels straight in the
// tensor-core operand format (exact tf32 split hi / lo, rows of K_dim padded
// to a multiple of 32 with zeros), so the GEMM reads it without a split
// pre-pass; the GEMM (tc_gemm.cu) splits the weight itself.  When the
// output rows are not 16-byte aligned (C_out % 4 != 0) or the problem is
// tiny, the patch matrix is written plain and the GEMM dispatcher picks the
// kernel.
#include <string.h>

#include "common.cuh"
#include "gemm_internal.cuh"
#include "tc_common.cuh"

namespace silcu {
namespace {

struct ConvShape {
  int64_t N, H, W, C, K, C_out, pad, M, Kd, Kp;
};

ConvShape conv_shape(uint32_t N, uint32_t H, uint32_t W, uint32_t C_in, uint32_t K, uint32_t C_out) {
  ConvShape s;
  s.N = N, s.H = H, s.W = W, s.C = C_in, s.K = K, s.C_out = C_out, s.pad = K / 2;
  s.M = s.N * s.H * s.W;
  s.Kd = s.K * s.K * s.C;
  s.Kp = (s.Kd + 31) / 32 * 32;
  return s;
}

bool conv_tc(const ConvShape &s) { return s.C_out % 4 == 0 && s.M >= 64 && s.C_out >= 32 && s.Kd >= 16; }

// Implicit GEMM (no patch matrix): the input is split once (hi / lo, NHWC)
// and the GEMM's A tiles are im2col TMA boxes of it, 16 channels of one
// filter tap per K block, so C_in must be a multiple of 16.
bool conv_implicit(const ConvShape &s) {
  return s.C % 16 == 0 && s.C_out % 4 == 0 && s.M >= 128 && s.C_out >= 32;
}

size_t conv_split_bytes(const ConvShape &s) { return (size_t(2) * s.M * s.C * sizeof(float) + 255) / 256 * 256; }

// One thread per 4 consecutive patch columns of one output pixel (a float4
// of hi and of lo when C_in % 4 == 0); columns past K_dim up to the padded
// row length are zeros.  SPLIT = 0 writes the plain patch matrix (row
// length K_dim).
template <bool SPLIT, bool VEC>
__global__ void __launch_bounds__(256) im2col_kernel(const float *__restrict__ in, float *__restrict__ hi,
                                                     float *__restrict__ lo, int64_t M, int64_t H, int64_t W,
                                                     int64_t C, int64_t K, int64_t pad, int64_t Kd, int64_t ld) {
  const int64_t q4 = ld / 4;
  const int64_t total = M * q4;
  for (int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += int64_t(gridDim.x) * blockDim.x) {
    const int64_t m = g / q4, k0 = (g - m * q4) * 4;
    const int64_t n = m / (H * W), sp = m - n * (H * W);
    const int64_t oh = sp / W, ow = sp - oh * W;
    float v[4];
    if (VEC && k0 < Kd) {  // C % 4 == 0: the 4 columns share (kh, kw)
      const int64_t kh = k0 / (K * C), r = k0 - kh * (K * C), kw = r / C, ci = r - kw * C;
      const int64_t ih = oh + kh - pad, iw = ow + kw - pad;
      float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
      if (ih >= 0 && ih < H && iw >= 0 && iw < W)
        f = __ldg(reinterpret_cast<const float4 *>(in + ((n * H + ih) * W + iw) * C + ci));
      v[0] = f.x, v[1] = f.y, v[2] = f.z, v[3] = f.w;
    } else {
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int64_t k = k0 + u;
        float x = 0.0f;
        if (k < Kd) {
          const int64_t kh = k / (K * C), r = k - kh * (K * C), kw = r / C, ci = r - kw * C;
          const int64_t ih = oh + kh - pad, iw = ow + kw - pad;
          if (ih >= 0 && ih < H && iw >= 0 && iw < W) x = __ldg(in + ((n * H + ih) * W + iw) * C + ci);
        }
        v[u] = x;
      }
    }
    if (SPLIT) {
      float h[4], l[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        h[u] = tc::tf32_rna(v[u]);
        l[u] = __fsub_rn(v[u], h[u]);
      }
      *reinterpret_cast<float4 *>(hi + m * ld + k0) = make_float4(h[0], h[1], h[2], h[3]);
      *reinterpret_cast<float4 *>(lo + m * ld + k0) = make_float4(l[0], l[1], l[2], l[3]);
    } else {
      for (int u = 0; u < 4; u++)
        if (k0 + u < Kd) hi[m * ld + k0 + u] = v[u];
    }
  }
}

silcu_gemm_args conv_gemm_args(const ConvShape &s, const float *weight, float *out) {
  silcu_gemm_args a;
  memset(&a, 0, sizeof(a));
  a.B = weight;  // [C_out, K_dim]: the K-major B operand
  a.C = out;
  a.M = s.M;
  a.N = s.C_out;
  a.ldb = s.Kd;
  a.ldc = s.C_out;
  a.trans_b = 1;
  a.batch = 1;
  a.alpha = 1.0f;
  a.algo = SILCU_GEMM_AUTO;
  return a;
}

}  // namespace
}  // namespace silcu

using namespace silcu;

extern "C" {

size_t silcu_conv2d_workspace_bytes(uint32_t N, uint32_t H, uint32_t W, uint32_t C_in, uint32_t K, uint32_t C_out) {
  const ConvShape s = conv_shape(N, H, W, C_in, K, C_out);
  silcu_gemm_args a = conv_gemm_args(s, nullptr, nullptr);
  size_t patch;
  if (conv_tc(s)) {
    patch = size_t(2) * s.M * s.Kp * sizeof(float);
    a.K = s.Kp;
    a.lda = s.Kp;
    a.A_hi = a.A_lo = reinterpret_cast<const float *>(16);  // layout only: split A
    a.algo = SILCU_GEMM_TC3XTF32;
    a.B = reinterpret_cast<const float *>(16);
    a.ldb = s.Kd;
    a.K = s.Kd;  // the GEMM sees K_dim; the split rows are padded
  } else {
    patch = size_t(s.M) * s.Kd * sizeof(float);
    a.K = s.Kd;
    a.lda = s.Kd;
    a.A = reinterpret_cast<const float *>(16);
    a.B = reinterpret_cast<const float *>(16);
  }
  patch = (patch + 255) / 256 * 256;
  size_t need = patch + silcu_sgemm_workspace_bytes(&a);
  if (conv_implicit(s)) {  // the implicit path: split input + the GEMM's B split / partials
    silcu_gemm_args g = conv_gemm_args(s, reinterpret_cast<const float *>(16), reinterpret_cast<float *>(16));
    g.A_hi = g.A_lo = reinterpret_cast<const float *>(16);
    g.K = s.Kd;
    g.lda = s.Kd;
    g.algo = SILCU_GEMM_TC3XTF32;
    const size_t imp = conv_split_bytes(s) + silcu_sgemm_workspace_bytes(&g);
    if (imp > need) need = imp;
  }
  return need;
}

silcu_status silcu_conv2d_f32(const float *input, const float *weight, float *output, uint32_t N, uint32_t H,
                              uint32_t W, uint32_t C_in, uint32_t K, uint32_t C_out, void *ws, size_t wsb,
                              silcu_stream stream) {
  if (!input || !weight || !output) return fail(SILCU_INVALID_ARGUMENT, "conv2d: null pointer");
  if (N == 0 || H == 0 || W == 0 || C_in == 0 || K == 0 || C_out == 0)
    return fail(SILCU_INVALID_ARGUMENT, "conv2d: empty extent");
  const ConvShape s = conv_shape(N, H, W, C_in, K, C_out);
  if (s.M > (int64_t(1) << 31) || s.Kp > (int64_t(1) << 24))
    return fail(SILCU_UNSUPPORTED, "conv2d: too large");
  const size_t need = silcu_conv2d_workspace_bytes(N, H, W, C_in, K, C_out);
  if (!ws || wsb < need) return fail(SILCU_WORKSPACE_TOO_SMALL, "conv2d: workspace %zu < %zu", wsb, need);
  cudaStream_t st = as_stream(stream);
  // the implicit path when the driver accepts the im2col map for this shape
  // (checked on a dummy encode; the patch-matrix path otherwise)
  CUtensorMap probe;
  const bool im2col_ok = conv_implicit(s) && aligned16(input) && aligned16(output) && aligned16(weight) &&
                         s.Kd % 4 == 0 &&
                         tc::make_im2col_map(&probe, input, s.N, s.H, s.W, s.C, int(s.pad), 16, 128,
                                         CU_TENSOR_MAP_SWIZZLE_64B);
  if (im2col_ok) {
    uint8_t *w8 = static_cast<uint8_t *>(ws);
    float *hi = reinterpret_cast<float *>(w8);
    float *lo = hi + s.M * s.C;
    silcu_status r = split_contiguous(input, uint64_t(s.M * s.C), hi, lo, st);  // [M, C] rows, C % 16 == 0
    if (r != SILCU_OK) return r;
    silcu_gemm_args a = conv_gemm_args(s, weight, output);
    a.A_hi = hi;
    a.A_lo = lo;
    a.K = s.Kd;
    a.lda = s.Kd;
    a.algo = SILCU_GEMM_TC3XTF32;
    TcConv cv;
    cv.in_hi = hi;
    cv.in_lo = lo;
    cv.N = s.N, cv.H = s.H, cv.W = s.W, cv.C = s.C, cv.Kf = s.K, cv.pad = s.pad;
    const size_t sb = conv_split_bytes(s);
    return tc_run(a, w8 + sb, wsb - sb, st, &cv);
  }
  const bool tc = conv_tc(s);
  const bool vec = (s.C % 4 == 0) && aligned16(input);
  uint8_t *w8 = static_cast<uint8_t *>(ws);
  float *hi = reinterpret_cast<float *>(w8);
  float *lo = tc ? hi + s.M * s.Kp : nullptr;
  size_t patch = tc ? size_t(2) * s.M * s.Kp * sizeof(float) : size_t(s.M) * s.Kd * sizeof(float);
  patch = (patch + 255) / 256 * 256;
  const int64_t ld = tc ? s.Kp : (s.Kd + 3) / 4 * 4;
  const int64_t threads = s.M * (ld / 4);
  int64_t grid = (threads + 255) / 256;
  const int64_t cap = int64_t(sm_count()) * 16;
  if (grid > cap) grid = cap;
  if (tc) {
    if (vec)
      im2col_kernel<true, true><<<unsigned(grid), 256, 0, st>>>(input, hi, lo, s.M, s.H, s.W, s.C, s.K, s.pad, s.Kd, ld);
    else
      im2col_kernel<true, false><<<unsigned(grid), 256, 0, st>>>(input, hi, lo, s.M, s.H, s.W, s.C, s.K, s.pad, s.Kd, ld);
  } else {
    // plain rows of K_dim (the last thread of a row stops at K_dim)
    im2col_kernel<false, false><<<unsigned(grid), 256, 0, st>>>(input, hi, nullptr, s.M, s.H, s.W, s.C, s.K, s.pad,
                                                               s.Kd, ld);
  }
  silcu_status r = check_launch("conv2d(im2col)");
  if (r != SILCU_OK) return r;
  silcu_gemm_args a = conv_gemm_args(s, weight, output);
  a.K = s.Kd;
  if (tc) {
    a.A_hi = hi;
    a.A_lo = lo;
    a.lda = s.Kp;
    a.algo = SILCU_GEMM_TC3XTF32;
  } else {
    a.A = hi;
    a.lda = ld;
  }
  return silcu_sgemm_ex(&a, w8 + patch, wsb - patch, stream);
}

}  // extern "C"

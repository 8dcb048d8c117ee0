// GEMM family on CUDA cores and the dispatcher of silcu_sgemm_ex.
//
//   ffma_gemm   128x128x8 tiles, 256 threads, 8x8 outputs per thread, fp32
//               FFMA.  Handles every stride/transpose/batch/tail case and is
//               the accuracy reference for the tensor-core path.
//   skinny_gemm M <= 16 rows per CTA (GEMV at M = 1): each thread streams
//               float4 columns of W with K split across warps and CTAs, so W
//               is read from HBM once; partials are combined in a fixed order.
//   tensor-core 3xTF32 tcgen05 path lives in tc_gemm.cu.
#include <string.h>

#include "common.cuh"
#include "gemm_internal.cuh"

namespace silcu {
namespace {

// ------------------------------------------------------------------ epilogue
struct Epi {
  float alpha;
  const float *bias;
  int64_t bias_len;
  int act;
  const float *residual;
  int64_t ldr;
};

__device__ __forceinline__ float apply_epi(const Epi &e, float acc, int64_t row, int64_t col,
                                           int64_t roff = 0) {
  float v = acc;
  if (e.alpha != 1.0f) v = __fmul_rn(v, e.alpha);
  if (e.bias) v = __fadd_rn(v, __ldg(e.bias + (col % e.bias_len)));
  if (e.act == SILCU_ACT_RELU) v = v >= 0.0f ? v : 0.0f;
  else if (e.act == SILCU_ACT_SIGMOID) v = sigmoid_ref(v);
  if (e.residual) v = __fadd_rn(v, __ldg(e.residual + roff + row * e.ldr + col));
  return v;
}

// ------------------------------------------------------------------ FFMA GEMM
constexpr int FBM = 128, FBN = 128, FBK = 8;

struct FfmaArgs {
  const float *A, *B;
  float *C;
  int64_t M, N, K, lda, ldb, ldc;
  int ta, tb;
  int64_t sa, sb, sc;
  int64_t bin, sa_in, sb_in, sc_in;  // inner batch level
  Epi epi;
};

__device__ __forceinline__ float load_a(const FfmaArgs &p, const float *A, int64_t m, int64_t k) {
  if (m >= p.M || k >= p.K) return 0.0f;
  return p.ta ? A[k * p.lda + m] : A[m * p.lda + k];
}
__device__ __forceinline__ float load_b(const FfmaArgs &p, const float *B, int64_t k, int64_t n) {
  if (n >= p.N || k >= p.K) return 0.0f;
  return p.tb ? B[n * p.ldb + k] : B[k * p.ldb + n];
}

__global__ void __launch_bounds__(256) ffma_gemm(const FfmaArgs p) {
  __shared__ float As[2][FBK][FBM];
  __shared__ float Bs[2][FBK][FBN];
  const int64_t bo = blockIdx.z / p.bin, bi = blockIdx.z % p.bin;
  const float *A = p.A + bo * p.sa + bi * p.sa_in;
  const float *B = p.B + bo * p.sb + bi * p.sb_in;
  const int64_t coff = bo * p.sc + bi * p.sc_in;
  float *C = p.C + coff;
  const int64_t m0 = int64_t(blockIdx.y) * FBM, n0 = int64_t(blockIdx.x) * FBN;
  const int t = threadIdx.x;
  const int tx = t % 16, ty = t / 16;
  // Loader mapping: 1024 elements per operand tile, 4 per thread.
  // A tile [FBM x FBK]: non-transposed reads run along k (contiguous), the
  // transposed case along m; either way the index math keeps a warp on few
  // cache lines.
  float ra[4], rb[4];
  auto fetch = [&](int64_t k0) {
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int e = t + u * 256;
      int mm, kk;
      if (p.ta) { mm = e % FBM; kk = e / FBM; } else { kk = e % FBK; mm = e / FBK; }
      ra[u] = load_a(p, A, m0 + mm, k0 + kk);
      int nn, kb;
      if (p.tb) { kb = e % FBK; nn = e / FBK; } else { nn = e % FBN; kb = e / FBN; }
      rb[u] = load_b(p, B, k0 + kb, n0 + nn);
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int e = t + u * 256;
      int mm, kk;
      if (p.ta) { mm = e % FBM; kk = e / FBM; } else { kk = e % FBK; mm = e / FBK; }
      As[buf][kk][mm] = ra[u];
      int nn, kb;
      if (p.tb) { kb = e % FBK; nn = e / FBK; } else { nn = e % FBN; kb = e / FBN; }
      Bs[buf][kb][nn] = rb[u];
    }
  };
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;

  const int64_t nk = (p.K + FBK - 1) / FBK;
  fetch(0);
  stash(0);
  __syncthreads();
  for (int64_t kt = 0; kt < nk; kt++) {
    const int buf = kt & 1;
    if (kt + 1 < nk) fetch((kt + 1) * FBK);
#pragma unroll
    for (int kk = 0; kk < FBK; kk++) {
      float a[8], b[8];
      const float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][64 + tx * 4]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
      b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (kt + 1 < nk) {
      stash(buf ^ 1);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int64_t row = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (row >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int64_t col = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (col < p.N) C[row * p.ldc + col] = apply_epi(p.epi, acc[i][j], row, col, coff);
    }
  }
}

// ------------------------------------------------------- skinny GEMM / GEMV
// CTA = 8 warps over one 128-column tile; lane l owns columns 4l..4l+3.
// Warps split the CTA's K chunk round-robin; CTAs (grid.y) split K further.
// Each thread keeps MR float4 accumulators (MR rows of X).
template <int MR>
__global__ void __launch_bounds__(256) skinny_gemm(const float *__restrict__ X, int64_t ldx,
                                                   const float *__restrict__ W, int64_t ldw,
                                                   float *__restrict__ out, int64_t ldo, int64_t M,
                                                   int64_t N, int64_t K, int64_t kchunk,
                                                   float *__restrict__ part, Epi epi) {
  __shared__ float red[MR][128];
  extern __shared__ float xs[];  // [MR][kchunk]
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t c0 = int64_t(blockIdx.x) * 128 + lane * 4;
  const int64_t k0 = int64_t(blockIdx.y) * kchunk;
  const int64_t k1 = k0 + kchunk < K ? k0 + kchunk : K;
  const int64_t m0 = int64_t(blockIdx.z) * MR;
  const int kn = int(k1 - k0);
  for (int e = threadIdx.x; e < MR * kn; e += 256) {
    const int r = e / kn, kk = e % kn;
    xs[r * kchunk + kk] = (m0 + r < M) ? X[(m0 + r) * ldx + k0 + kk] : 0.0f;
  }
  for (int e = threadIdx.x; e < MR * 128; e += 256) red[e / 128][e % 128] = 0.0f;
  __syncthreads();
  float4 acc[MR];
#pragma unroll
  for (int r = 0; r < MR; r++) acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
  const bool full = c0 + 4 <= N;
  int kk = w;
  for (; kk + 24 < kn; kk += 32) {
    float4 wv[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const float *src = W + (k0 + kk + u * 8) * ldw + c0;
      if (full) wv[u] = __ldg(reinterpret_cast<const float4 *>(src));
      else {
        wv[u].x = c0 < N ? src[0] : 0.f; wv[u].y = c0 + 1 < N ? src[1] : 0.f;
        wv[u].z = c0 + 2 < N ? src[2] : 0.f; wv[u].w = c0 + 3 < N ? src[3] : 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; u++)
#pragma unroll
      for (int r = 0; r < MR; r++) {
        const float x = xs[r * kchunk + kk + u * 8];
        acc[r].x = fmaf(x, wv[u].x, acc[r].x);
        acc[r].y = fmaf(x, wv[u].y, acc[r].y);
        acc[r].z = fmaf(x, wv[u].z, acc[r].z);
        acc[r].w = fmaf(x, wv[u].w, acc[r].w);
      }
  }
  for (; kk < kn; kk += 8) {
    const float *src = W + (k0 + kk) * ldw + c0;
    float4 wv;
    if (full) wv = __ldg(reinterpret_cast<const float4 *>(src));
    else {
      wv.x = c0 < N ? src[0] : 0.f; wv.y = c0 + 1 < N ? src[1] : 0.f;
      wv.z = c0 + 2 < N ? src[2] : 0.f; wv.w = c0 + 3 < N ? src[3] : 0.f;
    }
#pragma unroll
    for (int r = 0; r < MR; r++) {
      const float x = xs[r * kchunk + kk];
      acc[r].x = fmaf(x, wv.x, acc[r].x);
      acc[r].y = fmaf(x, wv.y, acc[r].y);
      acc[r].z = fmaf(x, wv.z, acc[r].z);
      acc[r].w = fmaf(x, wv.w, acc[r].w);
    }
  }
  // Combine the 8 warps in warp order (deterministic).
  for (int ww = 0; ww < 8; ww++) {
    if (w == ww) {
#pragma unroll
      for (int r = 0; r < MR; r++) {
        red[r][lane * 4 + 0] += acc[r].x;
        red[r][lane * 4 + 1] += acc[r].y;
        red[r][lane * 4 + 2] += acc[r].z;
        red[r][lane * 4 + 3] += acc[r].w;
      }
    }
    __syncthreads();
  }
  for (int e = threadIdx.x; e < MR * 128; e += 256) {
    const int r = e / 128, c = e % 128;
    const int64_t row = m0 + r, col = int64_t(blockIdx.x) * 128 + c;
    if (row >= M || col >= N) continue;
    if (part) part[(int64_t(blockIdx.y) * M + row) * N + col] = red[r][c];
    else out[row * ldo + col] = apply_epi(epi, red[r][c], row, col);
  }
}

__global__ void __launch_bounds__(256) skinny_finish(const float *__restrict__ part, int splits,
                                                     float *__restrict__ out, int64_t ldo, int64_t M,
                                                     int64_t N, Epi epi) {
  const int64_t j = int64_t(blockIdx.x) * 256 + threadIdx.x;
  if (j >= M * N) return;
  const int64_t row = j / N, col = j % N;
  float s = 0.0f;
  for (int sp = 0; sp < splits; sp++) s += part[int64_t(sp) * M * N + j];
  out[row * ldo + col] = apply_epi(epi, s, row, col);
}

struct SkinnyPlan {
  int mr, splits;
  int64_t kchunk;
};

SkinnyPlan skinny_plan(int64_t M, int64_t N, int64_t K) {
  SkinnyPlan pl;
  pl.mr = M == 1 ? 1 : (M <= 4 ? 4 : (M <= 8 ? 8 : 16));
  const int64_t col_tiles = (N + 127) / 128;
  const int64_t m_tiles = (M + pl.mr - 1) / pl.mr;
  const int64_t target = int64_t(sm_count()) * 6;
  int64_t sp = (target + col_tiles * m_tiles - 1) / (col_tiles * m_tiles);
  const int64_t max_sp = K / 64 > 0 ? K / 64 : 1;
  if (sp > max_sp) sp = max_sp;
  if (sp < 1) sp = 1;
  int64_t kchunk = (K + sp - 1) / sp;
  kchunk = (kchunk + 31) / 32 * 32;
  // keep the X tile in shared memory within 64 KB
  const int64_t max_chunk = (64 * 1024) / (4 * pl.mr);
  if (kchunk > max_chunk) kchunk = max_chunk / 32 * 32;
  pl.kchunk = kchunk;
  pl.splits = int((K + kchunk - 1) / kchunk);
  if (pl.splits < 1) pl.splits = 1;
  return pl;
}

template <int MR>
void launch_skinny(const SkinnyPlan &pl, const float *X, int64_t ldx, const float *W, int64_t ldw, float *out,
                   int64_t ldo, int64_t M, int64_t N, int64_t K, float *part, const Epi &epi,
                   cudaStream_t s) {
  dim3 grid(uint32_t((N + 127) / 128), uint32_t(pl.splits), uint32_t((M + MR - 1) / MR));
  const size_t smem = size_t(MR) * pl.kchunk * sizeof(float);
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(skinny_gemm<MR>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
    configured = true;
  }
  skinny_gemm<MR><<<grid, 256, smem, s>>>(X, ldx, W, ldw, out, ldo, M, N, K, pl.kchunk,
                                          pl.splits > 1 ? part : nullptr, epi);
  if (pl.splits > 1) {
    const int64_t total = M * N;
    skinny_finish<<<uint32_t((total + 255) / 256), 256, 0, s>>>(part, pl.splits, out, ldo, M, N, epi);
  }
}

bool skinny_eligible(const silcu_gemm_args &a) {
  return a.M <= 64 && !a.trans_a && !a.trans_b && a.batch == 1 && a.batch_inner <= 1 && (a.ldb % 4 == 0) &&
         aligned16(a.B) && a.K >= 1;
}

Epi make_epi(const silcu_gemm_args &a) {
  Epi e;
  e.alpha = a.alpha;
  e.bias = a.bias;
  e.bias_len = a.bias_len > 0 ? a.bias_len : 1;
  e.act = a.act;
  e.residual = a.residual;
  e.ldr = a.ldr;
  return e;
}

silcu_status validate(const silcu_gemm_args &a) {
  const bool has_a = a.A || (a.A_hi && a.A_lo), has_b = a.B || (a.B_hi && a.B_lo);
  const bool has_c = a.C || (a.C_hi && a.C_lo);
  if (!has_a || !has_b || !has_c) return fail(SILCU_INVALID_ARGUMENT, "sgemm: null pointer");
  const bool any_split = a.A_hi || a.A_lo || a.B_hi || a.B_lo || a.C_hi || a.C_lo;
  if (any_split && a.algo == SILCU_GEMM_FFMA)
    return fail(SILCU_UNSUPPORTED, "sgemm: split operands need the tensor-core path");
  if (a.M < 0 || a.N < 0 || a.K < 0 || a.batch < 1 || a.batch_inner < 0)
    return fail(SILCU_INVALID_ARGUMENT, "sgemm: negative extent or batch < 1");
  if (a.bias && a.bias_len <= 0) return fail(SILCU_INVALID_ARGUMENT, "sgemm: bias_len <= 0");
  if (a.M > 0 && a.N > 0) {
    if (a.ldc < a.N) return fail(SILCU_INVALID_ARGUMENT, "sgemm: ldc < N");
    if (a.K > 0) {
      if ((a.trans_a ? a.lda < a.M : a.lda < a.K)) return fail(SILCU_INVALID_ARGUMENT, "sgemm: lda too small");
      if ((a.trans_b ? a.ldb < a.K : a.ldb < a.N)) return fail(SILCU_INVALID_ARGUMENT, "sgemm: ldb too small");
    }
  }
  if (a.algo < 0 || a.algo > SILCU_GEMM_TC3XTF32) return fail(SILCU_INVALID_ARGUMENT, "sgemm: bad algo");
  return SILCU_OK;
}

}  // namespace

int gemm_path(const silcu_gemm_args &a) {
  if (a.A_hi || a.A_lo || a.B_hi || a.B_lo || a.C_hi || a.C_lo) return kPathTc;
  if (a.algo == SILCU_GEMM_FFMA) return kPathFfma;
  if (a.algo == SILCU_GEMM_TC3XTF32) return kPathTc;
  if (skinny_eligible(a)) return kPathSkinny;
  const double nb = double(a.batch) * double(a.batch_inner > 1 ? a.batch_inner : 1);
  if (a.M >= 64 && a.N >= 32 && a.K >= 32 && double(a.M) * a.N * a.K * nb >= double(1 << 22))
    return kPathTc;
  return kPathFfma;
}

}  // namespace silcu

using namespace silcu;

extern "C" {

size_t silcu_sgemm_workspace_bytes(const silcu_gemm_args *a) {
  if (!a) return 0;
  switch (gemm_path(*a)) {
    case kPathTc: return tc_workspace_bytes(*a);
    case kPathSkinny: {
      SkinnyPlan pl = skinny_plan(a->M, a->N, a->K);
      return pl.splits > 1 ? size_t(pl.splits) * a->M * a->N * sizeof(float) : 0;
    }
    default: return 0;
  }
}

silcu_status silcu_sgemm_ex(const silcu_gemm_args *ap, void *ws, size_t wsb, silcu_stream stream) {
  if (!ap) return fail(SILCU_INVALID_ARGUMENT, "sgemm: null args");
  const silcu_gemm_args &a = *ap;
  silcu_status st = validate(a);
  if (st != SILCU_OK) return st;
  if (a.M == 0 || a.N == 0) return SILCU_OK;
  cudaStream_t s = as_stream(stream);
  const Epi epi = make_epi(a);
  const int path = gemm_path(a);
  if (path == kPathTc) return tc_run(a, ws, wsb, s);
  if (path == kPathSkinny) {
    SkinnyPlan pl = skinny_plan(a.M, a.N, a.K);
    const size_t need = pl.splits > 1 ? size_t(pl.splits) * a.M * a.N * sizeof(float) : 0;
    if (need && (!ws || wsb < need))
      return fail(SILCU_WORKSPACE_TOO_SMALL, "sgemm(skinny): workspace %zu < %zu", wsb, need);
    float *part = static_cast<float *>(ws);
    switch (pl.mr) {
      case 1: launch_skinny<1>(pl, a.A, a.lda, a.B, a.ldb, a.C, a.ldc, a.M, a.N, a.K, part, epi, s); break;
      case 4: launch_skinny<4>(pl, a.A, a.lda, a.B, a.ldb, a.C, a.ldc, a.M, a.N, a.K, part, epi, s); break;
      case 8: launch_skinny<8>(pl, a.A, a.lda, a.B, a.ldb, a.C, a.ldc, a.M, a.N, a.K, part, epi, s); break;
      default: launch_skinny<16>(pl, a.A, a.lda, a.B, a.ldb, a.C, a.ldc, a.M, a.N, a.K, part, epi, s); break;
    }
    return check_launch("sgemm(skinny)", pl.splits > 1 ? 2 : 1);
  }
  const int64_t bin = a.batch_inner > 1 ? a.batch_inner : 1;
  if (a.batch * bin > 65535) return fail(SILCU_UNSUPPORTED, "sgemm(ffma): batch > 65535");
  if ((a.M + FBM - 1) / FBM > 65535) return fail(SILCU_UNSUPPORTED, "sgemm(ffma): M too large");
  FfmaArgs p{a.A, a.B, a.C, a.M, a.N, a.K, a.lda, a.ldb, a.ldc, a.trans_a, a.trans_b,
             a.stride_a, a.stride_b, a.stride_c, bin, a.stride_a_inner, a.stride_b_inner,
             a.stride_c_inner, epi};
  dim3 grid(uint32_t((a.N + FBN - 1) / FBN), uint32_t((a.M + FBM - 1) / FBM), uint32_t(a.batch * bin));
  ffma_gemm<<<grid, 256, 0, s>>>(p);
  return check_launch("sgemm(ffma)");
}

static silcu_gemm_args base_args(const float *A, const float *B, float *C, uint32_t M, uint32_t N, uint32_t K,
                                 uint32_t lda, uint32_t ldb, int ta, int tb) {
  silcu_gemm_args a;
  memset(&a, 0, sizeof(a));
  a.A = A; a.B = B; a.C = C;
  a.M = M; a.N = N; a.K = K;
  a.lda = lda; a.ldb = ldb; a.ldc = N;
  a.trans_a = ta; a.trans_b = tb;
  a.batch = 1;
  a.alpha = 1.0f;
  a.algo = SILCU_GEMM_AUTO;
  return a;
}

silcu_status silcu_sgemm(const float *A, const float *B, float *C, uint32_t M, uint32_t N, uint32_t K,
                         uint32_t lda, uint32_t ldb, int ta, int tb, void *ws, size_t wsb, silcu_stream s) {
  silcu_gemm_args a = base_args(A, B, C, M, N, K, lda, ldb, ta, tb);
  return silcu_sgemm_ex(&a, ws, wsb, s);
}

silcu_status silcu_sgemm_batched(const float *A, const float *B, float *C, uint32_t M, uint32_t N, uint32_t K,
                                 uint32_t lda, uint32_t ldb, uint32_t batch, uint64_t sa, uint64_t sb,
                                 uint64_t sc, void *ws, size_t wsb, silcu_stream s) {
  silcu_gemm_args a = base_args(A, B, C, M, N, K, lda, ldb, 0, 0);
  a.batch = batch;
  a.stride_a = int64_t(sa); a.stride_b = int64_t(sb); a.stride_c = int64_t(sc);
  return silcu_sgemm_ex(&a, ws, wsb, s);
}

silcu_status silcu_sgemm_bias(const float *A, const float *B, float *C, const float *bias, uint32_t bias_len,
                              uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb, void *ws,
                              size_t wsb, silcu_stream s) {
  silcu_gemm_args a = base_args(A, B, C, M, N, K, lda, ldb, 0, 0);
  a.bias = bias;
  a.bias_len = bias_len;
  return silcu_sgemm_ex(&a, ws, wsb, s);
}

silcu_status silcu_sgemm_bias_sigmoid(const float *A, const float *B, float *C, const float *bias,
                                      uint32_t bias_len, uint32_t M, uint32_t N, uint32_t K, uint32_t lda,
                                      uint32_t ldb, void *ws, size_t wsb, silcu_stream s) {
  silcu_gemm_args a = base_args(A, B, C, M, N, K, lda, ldb, 0, 0);
  a.bias = bias;
  a.bias_len = bias_len;
  a.act = SILCU_ACT_SIGMOID;
  return silcu_sgemm_ex(&a, ws, wsb, s);
}

size_t silcu_sgemv_workspace_bytes(uint32_t N, uint32_t K) {
  SkinnyPlan pl = skinny_plan(1, N, K);
  return pl.splits > 1 ? size_t(pl.splits) * N * sizeof(float) : 0;
}

silcu_status silcu_sgemv(const float *x, const float *W, float *y, const float *bias, uint32_t N, uint32_t K,
                         void *ws, size_t wsb, silcu_stream s) {
  silcu_gemm_args a = base_args(x, W, y, 1, N, K, K, N, 0, 0);
  a.bias = bias;
  a.bias_len = N;
  return silcu_sgemm_ex(&a, ws, wsb, s);
}

}  // extern "C"

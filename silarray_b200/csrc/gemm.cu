// GEMM family on CUDA cores and the dispatcher of silcu_sgemm_ex.
//
//   ffma_gemm   128x128x8 tiles, 256 threads, 8x8 outputs per thread, fp32
//               FFMA.  Handles every stride/transpose/batch/tail case and is
//               the accuracy reference for the tensor-core path.
//   gemv_kernel  M = 1: float4 streams of W, K slices combined in a thread
//                block cluster through distributed shared memory (HBM-bound).
//   small_m_gemm 2 <= M <= 64: 4x4 register micro-tiles over a cp.async ring,
//                split K combined in a cluster the same way.
//   Both sum in a fixed order, so results are deterministic.
//   tensor-core 3xTF32 tcgen05 path lives in tc_gemm.cu.
#include <stdlib.h>
#include <string.h>

#include <cooperative_groups.h>

#include "common.cuh"
#include "gemm_internal.cuh"

namespace silcu {
namespace {

// ------------------------------------------------------------------ epilogue
using Epi = SkinnyEpi;

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

// ------------------------------------------------------- small M / GEMV
// Small M (2..64): register-blocked FFMA with split K.  A CTA computes an
// MT x 64 tile of C over one K slice with 4*MT threads, each a 4 x 4
// micro-tile (64 FMAs per eight 128-bit shared loads).  K runs in stages of
// 32 through a kSmStages-deep cp.async ring: the W stage (32 x 64) and the X
// stage (MT x 32, rows padded to 36 floats) are 16-byte copies, zero-filled
// past N, past M and past the slice.  The slices of a tile run as one cluster
// and combine in rank order through distributed shared memory; with more
// slices than the cluster holds, each cluster writes a partial that
// partial_finish adds in order.
constexpr int kSmCols = 64;
constexpr int kSmStage = 32;
constexpr int kSmStages = 4;
constexpr int kSmXPitch = kSmStage + 4;

template <int MT>
constexpr size_t small_m_smem() {
  return size_t(kSmStages) * (kSmStage * kSmCols + MT * kSmXPitch) * sizeof(float);
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src, int bytes) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void cp_async4(void *dst, const void *src, int bytes) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(d), "l"(src), "r"(bytes) : "memory");
}

template <int MT>
__global__ void __launch_bounds__(4 * MT) small_m_gemm(const float *__restrict__ X, int64_t ldx,
                                                       const float *__restrict__ W, int64_t ldw,
                                                       float *__restrict__ out, int64_t ldo, int64_t M,
                                                       int64_t N, int64_t K, int64_t kchunk,
                                                       float *__restrict__ part, Epi epi) {
  namespace cg = cooperative_groups;
  constexpr int T = 4 * MT;
  extern __shared__ float4 sm_small[];
  float *wbase = reinterpret_cast<float *>(sm_small);        // [kSmStages][32][64]
  float *xbase = wbase + kSmStages * kSmStage * kSmCols;      // [kSmStages][MT][36]
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const int64_t col0 = int64_t(blockIdx.x) * kSmCols, m0 = int64_t(blockIdx.z) * MT;
  const int64_t k0 = int64_t(blockIdx.y) * kchunk;
  const int64_t kend = k0 + kchunk < K ? k0 + kchunk : K;
  const int nst = kend > k0 ? int((kend - k0 + kSmStage - 1) / kSmStage) : 0;
  const bool xvec = (ldx % 4) == 0 && (reinterpret_cast<uintptr_t>(X) & 15) == 0;

  auto load_stage = [&](int st) {
    const int buf = st % kSmStages;
    const int64_t kb = k0 + int64_t(st) * kSmStage;
    float *wsb = wbase + buf * kSmStage * kSmCols;
    for (int i = tid; i < kSmStage * (kSmCols / 4); i += T) {
      const int kk = i / (kSmCols / 4), q = i % (kSmCols / 4);
      const int64_t k = kb + kk, col = col0 + 4 * q;
      int bytes = 0;
      if (k < kend) {
        const int64_t left = N - col;
        bytes = left >= 4 ? 16 : (left > 0 ? int(left) * 4 : 0);
      }
      cp_async16(wsb + kk * kSmCols + 4 * q, bytes ? W + k * ldw + col : W, bytes);
    }
    float *xsb = xbase + buf * MT * kSmXPitch;
    for (int i = tid; i < MT * (kSmStage / 4); i += T) {
      const int r = i / (kSmStage / 4), q = i % (kSmStage / 4);
      const int64_t row = m0 + r, k = kb + 4 * q;
      const int64_t left = row < M ? kend - k : 0;
      const float *src = X + row * ldx + k;
      float *dst = xsb + r * kSmXPitch + 4 * q;
      if (xvec) {
        const int bytes = left >= 4 ? 16 : (left > 0 ? int(left) * 4 : 0);
        cp_async16(dst, bytes ? src : X, bytes);
      } else {
#pragma unroll
        for (int u = 0; u < 4; u++) cp_async4(dst + u, u < left ? src + u : X, u < left ? 4 : 0);
      }
    }
  };

  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
#pragma unroll
  for (int st = 0; st < kSmStages - 1; st++) {
    if (st < nst) load_stage(st);
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  }
  for (int st = 0; st < nst; st++) {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(kSmStages - 2) : "memory");
    __syncthreads();  // stage st landed for every thread; stage st-1's buffer is free
    if (st + kSmStages - 1 < nst) load_stage(st + kSmStages - 1);
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    const int buf = st % kSmStages;
    const float *wsb = wbase + buf * kSmStage * kSmCols;
    const float *xsb = xbase + buf * MT * kSmXPitch;
#pragma unroll
    for (int k4 = 0; k4 < kSmStage / 4; k4++) {
      float a[4][4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float4 f = *reinterpret_cast<const float4 *>(xsb + (4 * ty + i) * kSmXPitch + 4 * k4);
        a[i][0] = f.x; a[i][1] = f.y; a[i][2] = f.z; a[i][3] = f.w;
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const float4 b = *reinterpret_cast<const float4 *>(wsb + (4 * k4 + u) * kSmCols + 4 * tx);
        const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
          for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i][u], bv[j], acc[i][j]);
      }
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  __syncthreads();
  // CTA tile into shared memory (the ring is free), then the cluster combine.
  float *red = wbase;  // MT x 64 <= kSmStages x 32 x 64
#pragma unroll
  for (int i = 0; i < 4; i++)
    *reinterpret_cast<float4 *>(&red[(4 * ty + i) * kSmCols + 4 * tx]) =
        make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
  cg::cluster_group cl = cg::this_cluster();
  cl.sync();
  const int CL = int(cl.num_blocks()), q = int(cl.block_rank());
  constexpr int E = MT * kSmCols;
  const int per = E / CL;
  const int64_t g = blockIdx.y / CL;
  for (int e = q * per + tid; e < (q + 1) * per; e += T) {
    float v = 0.0f;
    for (int j = 0; j < CL; j++) v += cl.map_shared_rank(red, j)[e];
    const int64_t row = m0 + e / kSmCols, col = col0 + e % kSmCols;
    if (row >= M || col >= N) continue;
    if (part) part[(g * M + row) * N + col] = v;
    else out[row * ldo + col] = apply_epi(epi, v, row, col);
  }
  cl.sync();
}

// GEMV (M = 1): a CTA owns 128 columns (lane l holds 4, float4 loads) and a
// slice of K; warp w takes rows w, w+8, ... of the slice, U float4 loads in
// flight per thread from a pointer stepped by 8 rows (U = 16 with up to 2
// CTAs per SM when the grid is small, so more bytes are in flight per SM;
// U = 8 with up to 4 CTAs per SM otherwise: measured 4096 x 4096 14.9 ->
// 12.7 us with U = 16, while 16384 x 4096 runs 43.9 us with U = 8, 53 with 16).  x is read
// through the read-only cache (one broadcast per warp and row).  The 8 warps
// combine in warp order in shared memory, then the CL consecutive slices of a
// cluster combine in rank order through distributed shared memory; with more
// than CL slices, each cluster writes a partial that partial_finish adds in
// order.
template <int kGemvUnroll>
__global__ void __launch_bounds__(256, kGemvUnroll >= 16 ? 2 : 4) gemv_kernel(const float *__restrict__ x, const float *__restrict__ W,
                                                   int64_t ldw, float *__restrict__ out, int64_t N, int64_t K,
                                                   int64_t kchunk, float *__restrict__ part, Epi epi) {
  namespace cg = cooperative_groups;
  __shared__ float4 wsum[8][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t c0 = int64_t(blockIdx.x) * 128 + lane * 4;
  const int64_t k0 = int64_t(blockIdx.y) * kchunk;
  const int64_t k1 = k0 + kchunk < K ? k0 + kchunk : K;
  const bool vec = c0 + 4 <= N;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  const float *p = W + (k0 + w) * ldw + c0;
  const int64_t step = 8 * ldw;
  int64_t k = k0 + w;
  for (; k + 8 * (kGemvUnroll - 1) < k1; k += 8 * kGemvUnroll) {
    float4 wv[kGemvUnroll];
    float xv[kGemvUnroll];
    if (vec) {
#pragma unroll
      for (int u = 0; u < kGemvUnroll; u++) wv[u] = __ldg(reinterpret_cast<const float4 *>(p + u * step));
    } else {
#pragma unroll
      for (int u = 0; u < kGemvUnroll; u++) {
        const float *q = p + u * step;
        wv[u] = make_float4(c0 < N ? q[0] : 0.f, c0 + 1 < N ? q[1] : 0.f, c0 + 2 < N ? q[2] : 0.f, 0.f);
      }
    }
#pragma unroll
    for (int u = 0; u < kGemvUnroll; u++) xv[u] = __ldg(x + k + 8 * u);
#pragma unroll
    for (int u = 0; u < kGemvUnroll; u++) {
      acc.x = fmaf(xv[u], wv[u].x, acc.x);
      acc.y = fmaf(xv[u], wv[u].y, acc.y);
      acc.z = fmaf(xv[u], wv[u].z, acc.z);
      acc.w = fmaf(xv[u], wv[u].w, acc.w);
    }
    p += kGemvUnroll * step;
  }
  for (; k < k1; k += 8, p += step) {
    float4 wv;
    if (vec) wv = __ldg(reinterpret_cast<const float4 *>(p));
    else wv = make_float4(c0 < N ? p[0] : 0.f, c0 + 1 < N ? p[1] : 0.f, c0 + 2 < N ? p[2] : 0.f, 0.f);
    const float xv = __ldg(x + k);
    acc.x = fmaf(xv, wv.x, acc.x);
    acc.y = fmaf(xv, wv.y, acc.y);
    acc.z = fmaf(xv, wv.z, acc.z);
    acc.w = fmaf(xv, wv.w, acc.w);
  }
  wsum[w][lane] = acc;
  __syncthreads();
  float *tile = reinterpret_cast<float *>(&wsum[0][0]);  // 128 column sums after the warp combine
  if (w == 0) {
    float4 v = wsum[0][lane];
#pragma unroll
    for (int j = 1; j < 8; j++) {
      const float4 t = wsum[j][lane];
      v.x += t.x; v.y += t.y; v.z += t.z; v.w += t.w;
    }
    __syncwarp();
    wsum[0][lane] = v;
  }
  // The cluster's CTAs are consecutive K slices of this column tile: rank q
  // adds columns [q*128/CL, (q+1)*128/CL) over the ranks in order.
  cg::cluster_group cl = cg::this_cluster();
  cl.sync();
  const int CL = int(cl.num_blocks()), q = int(cl.block_rank());
  const int per = 128 / CL;
  if (int(threadIdx.x) < per) {
    const int c = q * per + threadIdx.x;
    float v = 0.0f;
    for (int j = 0; j < CL; j++) v += cl.map_shared_rank(tile, j)[c];
    const int64_t col = int64_t(blockIdx.x) * 128 + c;
    if (col < N) {
      if (part) part[int64_t(blockIdx.y / CL) * N + col] = v;
      else out[col] = apply_epi(epi, v, 0, col);
    }
  }
  cl.sync();
}

__global__ void __launch_bounds__(256) partial_finish(const float *__restrict__ part, int groups,
                                                     float *__restrict__ out, int64_t ldo, int64_t M,
                                                     int64_t N, Epi epi) {
  const int64_t j = int64_t(blockIdx.x) * 256 + threadIdx.x;
  if (j >= M * N) return;
  const int64_t row = j / N, col = j % N;
  // Loads batched 16 at a time (independent, in flight together); the adds
  // keep group order.
  const int64_t stride = M * N;
  float s = 0.0f;
  for (int g0 = 0; g0 < groups; g0 += 16) {
    float v[16];
#pragma unroll
    for (int u = 0; u < 16; u++) v[u] = g0 + u < groups ? part[int64_t(g0 + u) * stride + j] : 0.0f;
#pragma unroll
    for (int u = 0; u < 16; u++)
      if (g0 + u < groups) s += v[u];
  }
  out[row * ldo + col] = apply_epi(epi, s, row, col);
}

struct SmallMPlan {
  int mt, cluster, groups;  // K slices = cluster * groups; groups > 1 needs the finish pass
  int64_t kchunk;
};

int env_int(const char *name, int lo, int hi, int dflt) {
  const char *e = getenv(name);
  const int x = e ? atoi(e) : dflt;
  return x >= lo && x <= hi ? x : dflt;
}

// Cluster of 8 slices (4 for 64-row tiles, whose CTAs are 256 threads); for
// tiles of up to 32 rows, enough cluster groups for about 3 CTAs per SM (a CTA's life is short and
// latency-bound, so more CTAs in flight is faster), but slices of at least
// 128 k, and at most 1024 k (more become groups).  Measured: 32x768x4096
// 14.5 -> 13.1 us, 8x4096x4096 30.7 -> 27.0 us against a 16-CTA cluster.
// SILCU_SMALLM_CLUSTER and SILCU_SMALLM_GROUPS override, for tuning.
SmallMPlan small_m_plan(int64_t M, int64_t N, int64_t K) {
  SmallMPlan pl;
  pl.mt = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
  const int64_t tiles = (N + kSmCols - 1) / kSmCols * ((M + pl.mt - 1) / pl.mt);
  static const int forced_cl = env_int("SILCU_SMALLM_CLUSTER", 1, 16, 0);
  static const int forced_groups = env_int("SILCU_SMALLM_GROUPS", 1, 64, 0);
  pl.cluster = forced_cl ? forced_cl : (pl.mt == 64 ? 4 : 8);
  const int64_t cl = pl.cluster;
  int64_t groups = (K + cl * 1024 - 1) / (cl * 1024);
  // (64-row tiles are FMA-bound with 256-thread CTAs: extra groups only add partials.)
  const int64_t want = pl.mt == 64 ? 1 : (3 * int64_t(sm_count()) + tiles * cl - 1) / (tiles * cl);
  const int64_t cap = K / (cl * 128);
  const int64_t more = want < cap ? want : cap;
  if (groups < more) groups = more;
  if (forced_groups) groups = forced_groups;
  if (groups < 1) groups = 1;
  int64_t kchunk = (K + groups * pl.cluster - 1) / (groups * pl.cluster);
  kchunk = (kchunk + kSmStage - 1) / kSmStage * kSmStage;
  pl.kchunk = kchunk;
  pl.groups = int((K + kchunk * pl.cluster - 1) / (kchunk * pl.cluster));
  if (pl.groups < 1) pl.groups = 1;
  return pl;
}

size_t small_m_part_bytes(const SmallMPlan &pl, int64_t M, int64_t N) {
  return pl.groups > 1 ? size_t(pl.groups) * M * N * sizeof(float) : 0;
}

template <int MT>
cudaError_t launch_small_m(const SmallMPlan &pl, const float *X, int64_t ldx, const float *W, int64_t ldw,
                           float *out, int64_t ldo, int64_t M, int64_t N, int64_t K, float *part,
                           const Epi &epi, cudaStream_t s) {
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaFuncSetAttribute(small_m_gemm<MT>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    cudaFuncSetAttribute(small_m_gemm<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(small_m_smem<MT>()));
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(uint32_t((N + kSmCols - 1) / kSmCols), uint32_t(pl.groups * pl.cluster),
                     uint32_t((M + MT - 1) / MT));
  cfg.blockDim = dim3(4 * MT);
  cfg.dynamicSmemBytes = small_m_smem<MT>();
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = unsigned(pl.cluster);
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  float *p = pl.groups > 1 ? part : nullptr;
  cudaError_t e = cudaLaunchKernelEx(&cfg, small_m_gemm<MT>, X, ldx, W, ldw, out, ldo, M, N, K, pl.kchunk, p, epi);
  if (e != cudaSuccess) return e;
  if (pl.groups > 1) {
    const int64_t total = M * N;
    partial_finish<<<uint32_t((total + 255) / 256), 256, 0, s>>>(part, pl.groups, out, ldo, M, N, epi);
  }
  return cudaSuccess;
}

struct GemvPlan {
  int cluster, groups;  // K slices = cluster * groups; groups > 1 needs the finish pass
  int64_t kchunk;
};

// Cluster size for the K slices: 8, or 16 when 8 slices per column tile
// would leave SMs idle (environment SILCU_GEMV_CLUSTER = 1/2/4/8/16
// overrides, for tuning).
int gemv_cluster(int64_t tiles, int64_t K) {
  static const int forced = [] {
    const char *e = getenv("SILCU_GEMV_CLUSTER");
    const int x = e ? atoi(e) : 0;
    return (x == 1 || x == 2 || x == 4 || x == 8 || x == 16) ? x : 0;
  }();
  if (forced) return forced;
  return (tiles * 8 < sm_count() && K >= 16 * 64) ? 16 : 8;
}

// One cluster group while the slices stay <= 1024 rows; multiples of 64 rows.
GemvPlan gemv_plan(int64_t N, int64_t K) {
  GemvPlan pl;
  pl.cluster = gemv_cluster((N + 127) / 128, K);
  int64_t groups = (K + int64_t(pl.cluster) * 1024 - 1) / (int64_t(pl.cluster) * 1024);
  if (groups < 1) groups = 1;
  int64_t kchunk = (K + groups * pl.cluster - 1) / (groups * pl.cluster);
  kchunk = (kchunk + 63) / 64 * 64;
  pl.kchunk = kchunk;
  pl.groups = int((K + kchunk * pl.cluster - 1) / (kchunk * pl.cluster));
  if (pl.groups < 1) pl.groups = 1;
  return pl;
}

size_t gemv_part_bytes(const GemvPlan &pl, int64_t N) {
  return pl.groups > 1 ? size_t(pl.groups) * N * sizeof(float) : 0;
}

cudaError_t launch_gemv(const GemvPlan &pl, const float *x, const float *W, int64_t ldw, float *out, int64_t N,
                        int64_t K, float *part, const Epi &epi, cudaStream_t s) {
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (pl.cluster > 8 && dev >= 0 && dev < 64 && !configured[dev]) {
    cudaFuncSetAttribute(gemv_kernel<8>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    cudaFuncSetAttribute(gemv_kernel<16>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    configured[dev] = true;
  }
  const int64_t ctas = (N + 127) / 128 * int64_t(pl.groups) * pl.cluster;
  const bool deep = ctas <= 2 * int64_t(sm_count());
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(uint32_t((N + 127) / 128), uint32_t(pl.groups * pl.cluster));
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = unsigned(pl.cluster);
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  float *p = pl.groups > 1 ? part : nullptr;
  cudaError_t e = deep ? cudaLaunchKernelEx(&cfg, gemv_kernel<16>, x, W, ldw, out, N, K, pl.kchunk, p, epi)
                       : cudaLaunchKernelEx(&cfg, gemv_kernel<8>, x, W, ldw, out, N, K, pl.kchunk, p, epi);
  if (e != cudaSuccess) return e;
  if (pl.groups > 1)
    partial_finish<<<uint32_t((N + 255) / 256), 256, 0, s>>>(part, pl.groups, out, N, 1, N, epi);
  return cudaSuccess;
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
      if (a->M == 1) return gemv_part_bytes(gemv_plan(a->N, a->K), a->N);
      if (skinny_tma_eligible(*a)) return 0;
      return small_m_part_bytes(small_m_plan(a->M, a->N, a->K), a->M, a->N);
    }
    default: return 0;
  }
}

silcu_status silcu_sgemm_plan(const silcu_gemm_args *a, silcu_gemm_plan *plan) {
  if (!a || !plan) return fail(SILCU_INVALID_ARGUMENT, "sgemm_plan: null argument");
  silcu_gemm_plan p = {};
  p.path = gemm_path(*a);
  p.ksplit = 1;
  if (p.path == kPathTc) tc_describe(*a, &p);
  *plan = p;
  return SILCU_OK;
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
  if (path == kPathSkinny && a.M == 1) {
    const GemvPlan pl = gemv_plan(a.N, a.K);
    const size_t need = gemv_part_bytes(pl, a.N);
    if (need && (!ws || wsb < need))
      return fail(SILCU_WORKSPACE_TOO_SMALL, "sgemm(gemv): workspace %zu < %zu", wsb, need);
    const cudaError_t e = launch_gemv(pl, a.A, a.B, a.ldb, a.C, a.N, a.K, static_cast<float *>(ws), epi, s);
    if (e != cudaSuccess) return fail(SILCU_CUDA_ERROR, "sgemm(gemv): %s", cudaGetErrorString(e));
    return check_launch("sgemm(gemv)", pl.groups > 1 ? 2 : 1);
  }
  if (path == kPathSkinny && skinny_tma_eligible(a)) return skinny_tma_run(a, epi, s);
  if (path == kPathSkinny) {
    const SmallMPlan pl = small_m_plan(a.M, a.N, a.K);
    const size_t need = small_m_part_bytes(pl, a.M, a.N);
    if (need && (!ws || wsb < need))
      return fail(SILCU_WORKSPACE_TOO_SMALL, "sgemm(small M): workspace %zu < %zu", wsb, need);
    float *part = static_cast<float *>(ws);
    cudaError_t e;
    switch (pl.mt) {
      case 16: e = launch_small_m<16>(pl, a.A, a.lda, a.B, a.ldb, a.C, a.ldc, a.M, a.N, a.K, part, epi, s); break;
      case 32: e = launch_small_m<32>(pl, a.A, a.lda, a.B, a.ldb, a.C, a.ldc, a.M, a.N, a.K, part, epi, s); break;
      default: e = launch_small_m<64>(pl, a.A, a.lda, a.B, a.ldb, a.C, a.ldc, a.M, a.N, a.K, part, epi, s); break;
    }
    if (e != cudaSuccess) return fail(SILCU_CUDA_ERROR, "sgemm(small M): %s", cudaGetErrorString(e));
    return check_launch("sgemm(small M)", pl.groups > 1 ? 2 : 1);
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
  return gemv_part_bytes(gemv_plan(N, K), N);
}

silcu_status silcu_sgemv(const float *x, const float *W, float *y, const float *bias, uint32_t N, uint32_t K,
                         void *ws, size_t wsb, silcu_stream s) {
  silcu_gemm_args a = base_args(x, W, y, 1, N, K, K, N, 0, 0);
  a.bias = bias;
  a.bias_len = N;
  return silcu_sgemm_ex(&a, ws, wsb, s);
}

}  // extern "C"

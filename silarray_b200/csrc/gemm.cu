// GEMM family on CUDA cores and the dispatcher of silcu_sgemm_ex.
//
//   ffma_gemm   128x128x8 tiles, 256 threads, 8x8 outputs per thread, fp32
//               FFMA.  Handles every stride/transpose/batch/tail case and is
//               the accuracy reference for the tensor-core path.
//   skinny_gemm M <= 64 (GEMV at M = 1): each thread streams 2-4 columns of
//               W with K split across warps and CTAs, so W is read from HBM
//               once; partials are combined in a fixed order.
//   tensor-core 3xTF32 tcgen05 path lives in tc_gemm.cu.
#include <stdlib.h>
#include <string.h>

#include <cooperative_groups.h>

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
// HBM-bound: W is streamed once.  A CTA (8 warps) owns a tile of 32*CPL
// columns (lane l holds CPL consecutive columns), MR rows of X and one K
// slice; its warps take the slice's k round-robin with UNROLL W loads in
// flight per thread, the first batch issued before X's slice is staged
// (transposed, [k][m], so the MR values of one k are broadcast loads).  The
// K slices of a tile run as one 8-CTA cluster and are combined through
// distributed shared memory in rank order; with more than 8 slices per tile,
// G cluster groups write partials that skinny_finish adds in group order.
// Every sum has a fixed order, so results are deterministic.
constexpr int kSkinnyCluster = 8;
constexpr int kSkinnyMaxChunk = 256;  // K per CTA at most

template <int MR, int CPL, int UNROLL>
__global__ void __cluster_dims__(1, kSkinnyCluster, 1) __launch_bounds__(256, MR <= 8 ? 4 : 1)
    skinny_gemm(const float *__restrict__ X, int64_t ldx, const float *__restrict__ W, int64_t ldw,
                float *__restrict__ out, int64_t ldo, int64_t M, int64_t N, int64_t K, int64_t kchunk,
                float *__restrict__ part, Epi epi) {
  namespace cg = cooperative_groups;
  constexpr int COLS = 32 * CPL, E = MR * COLS;
  extern __shared__ float4 smem4[];
  float *wred = reinterpret_cast<float *>(smem4);  // [8][E] per-warp sums
  float *red = wred + 8 * E;                       // [E] CTA sum (read by the cluster)
  float *xs = red + E;                             // [kchunk][MR]
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t col0 = int64_t(blockIdx.x) * COLS;
  const int64_t c0 = col0 + lane * CPL;
  const int64_t k0 = int64_t(blockIdx.y) * kchunk;
  const int64_t kend = k0 + kchunk < K ? k0 + kchunk : K;
  const int kn = kend > k0 ? int(kend - k0) : 0;
  const int64_t m0 = int64_t(blockIdx.z) * MR;
  const bool full = c0 + CPL <= N && ((reinterpret_cast<uintptr_t>(W + c0) & (4 * CPL - 1)) == 0);
  auto loadw = [&](int kk, float (&wv)[CPL]) {
    if (kk >= kn) {
#pragma unroll
      for (int c = 0; c < CPL; c++) wv[c] = 0.0f;
      return;
    }
    const float *src = W + (k0 + kk) * ldw + c0;
    if (full) {
      if constexpr (CPL == 4) {
        const float4 f = __ldg(reinterpret_cast<const float4 *>(src));
        wv[0] = f.x; wv[1] = f.y; wv[2] = f.z; wv[3] = f.w;
      } else if constexpr (CPL == 2) {
        const float2 f = __ldg(reinterpret_cast<const float2 *>(src));
        wv[0] = f.x; wv[1] = f.y;
      } else {
        wv[0] = __ldg(src);
      }
    } else {
#pragma unroll
      for (int c = 0; c < CPL; c++) wv[c] = c0 + c < N ? src[c] : 0.0f;
    }
  };
  float acc[MR][CPL];
#pragma unroll
  for (int r = 0; r < MR; r++)
#pragma unroll
    for (int c = 0; c < CPL; c++) acc[r][c] = 0.0f;
  auto fma_row = [&](int kk, const float (&wv)[CPL]) {
    const float *xr = xs + kk * MR;
    constexpr int V = MR >= 4 ? 4 : 1;
#pragma unroll
    for (int r = 0; r < MR; r += V) {
      float xv[4];
      if constexpr (V == 4) {
        const float4 f = *reinterpret_cast<const float4 *>(xr + r);
        xv[0] = f.x; xv[1] = f.y; xv[2] = f.z; xv[3] = f.w;
      } else {
        xv[0] = xr[r];
      }
#pragma unroll
      for (int q = 0; q < V; q++)
#pragma unroll
        for (int c = 0; c < CPL; c++) acc[r + q][c] = fmaf(xv[q], wv[c], acc[r + q][c]);
    }
  };
  // First W batch in flight while X's slice is staged.
  float wv[UNROLL][CPL];
#pragma unroll
  for (int u = 0; u < UNROLL; u++) loadw(w + 8 * u, wv[u]);
  // X slice: thread e loads 4 consecutive k of row e % MR (16-byte loads when
  // aligned), XB loads in flight per thread; the [k][m] stores of a warp hit
  // consecutive rows, so they are free of bank conflicts.
  {
    constexpr int XB = 8;
    const int k4n = int(kchunk) / 4;  // the whole slice, zero past kn
    const bool xvec = (ldx % 4) == 0 && (reinterpret_cast<uintptr_t>(X) & 15) == 0;
    for (int base = threadIdx.x; base < MR * k4n; base += 256 * XB) {
      float v[XB][4];
#pragma unroll
      for (int u = 0; u < XB; u++) {
        const int e = base + u * 256, r = e % MR, kk = (e / MR) * 4;
        const float *src = X + (m0 + r) * ldx + k0 + kk;
        if (e < MR * k4n && m0 + r < M) {
          if (xvec && kk + 4 <= kn) {
            const float4 f = __ldg(reinterpret_cast<const float4 *>(src));
            v[u][0] = f.x; v[u][1] = f.y; v[u][2] = f.z; v[u][3] = f.w;
          } else {
#pragma unroll
            for (int i = 0; i < 4; i++) v[u][i] = kk + i < kn ? src[i] : 0.0f;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 4; i++) v[u][i] = 0.0f;
        }
      }
#pragma unroll
      for (int u = 0; u < XB; u++) {
        const int e = base + u * 256, r = e % MR, kk = (e / MR) * 4;
        if (e < MR * k4n)
#pragma unroll
          for (int i = 0; i < 4; i++) xs[(kk + i) * MR + r] = v[u][i];
      }
    }
  }
  __syncthreads();
  // kchunk is a multiple of 8 * UNROLL and X's slice is zero past kn, so the
  // loop needs no guards (W loads past kn return 0).
  for (int kk = w; kk < kchunk; kk += 8 * UNROLL) {
    if (kk > w) {
#pragma unroll
      for (int u = 0; u < UNROLL; u++) loadw(kk + 8 * u, wv[u]);
    }
#pragma unroll
    for (int u = 0; u < UNROLL; u++) fma_row(kk + 8 * u, wv[u]);
  }
#pragma unroll
  for (int r = 0; r < MR; r++)
#pragma unroll
    for (int c = 0; c < CPL; c++) wred[w * E + r * COLS + lane * CPL + c] = acc[r][c];
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += 256) {
    float v = wred[e];
#pragma unroll
    for (int ww = 1; ww < 8; ww++) v += wred[ww * E + e];
    red[e] = v;
  }
  cg::cluster_group cl = cg::this_cluster();
  cl.sync();
  // Rank q of the cluster finishes elements [q*E/8, (q+1)*E/8) of the tile.
  const int q = int(cl.block_rank());
  const int64_t g = blockIdx.y / kSkinnyCluster;
  for (int e = q * (E / kSkinnyCluster) + threadIdx.x; e < (q + 1) * (E / kSkinnyCluster); e += 256) {
    float v = 0.0f;
#pragma unroll
    for (int j = 0; j < kSkinnyCluster; j++) v += cl.map_shared_rank(red, j)[e];
    const int r = e / COLS, c = e % COLS;
    const int64_t row = m0 + r, col = col0 + c;
    if (row >= M || col >= N) continue;
    if (part) part[(g * M + row) * N + col] = v;
    else out[row * ldo + col] = apply_epi(epi, v, row, col);
  }
  cl.sync();  // peers' shared memory stays valid until every rank has read it
}

// GEMV (M = 1): a CTA owns 128 columns (lane l holds 4, float4 loads) and a
// slice of K; warp w takes rows w, w+8, ... of the slice, GEMV_UNROLL float4
// loads in flight per thread from a pointer stepped by 8 rows.  x is read
// through the read-only cache (one broadcast per warp and row).  The 8 warps
// combine in warp order in shared memory, then the CL consecutive slices of a
// cluster combine in rank order through distributed shared memory; with more
// than CL slices, each cluster writes a partial that skinny_finish adds in
// order.
constexpr int kGemvUnroll = 8;

__global__ void __launch_bounds__(256, 4) gemv_kernel(const float *__restrict__ x, const float *__restrict__ W,
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

__global__ void __launch_bounds__(256) skinny_finish(const float *__restrict__ part, int groups,
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

struct SkinnyPlan {
  int mr, cpl, groups;  // groups: cluster groups along K (> 1 needs the finish pass)
  int64_t kchunk;       // K per CTA
};

int skinny_unroll(int mr) { return mr == 32 ? 4 : 8; }

SkinnyPlan skinny_plan(int64_t M, int64_t N, int64_t K) {
  SkinnyPlan pl;
  if (M <= 8) { pl.mr = 8; pl.cpl = 2; }
  else if (M <= 16) { pl.mr = 16; pl.cpl = 1; }
  else { pl.mr = 32; pl.cpl = 1; }
  // Slices of 256 k: few enough CTAs that the per-CTA costs
  // (X staging, cluster combine) stay small, long enough chains of W loads
  // per warp to keep HBM busy.
  const int64_t step = 8 * skinny_unroll(pl.mr);
  const int64_t target = kSkinnyMaxChunk;
  int64_t groups = (K + target * kSkinnyCluster - 1) / (target * kSkinnyCluster);
  if (groups < 1) groups = 1;
  int64_t kchunk = (K + groups * kSkinnyCluster - 1) / (groups * kSkinnyCluster);
  kchunk = (kchunk + step - 1) / step * step;
  pl.kchunk = kchunk;
  pl.groups = int((K + kchunk * kSkinnyCluster - 1) / (kchunk * kSkinnyCluster));
  if (pl.groups < 1) pl.groups = 1;
  return pl;
}

size_t skinny_part_bytes(const SkinnyPlan &pl, int64_t M, int64_t N) {
  return pl.groups > 1 ? size_t(pl.groups) * M * N * sizeof(float) : 0;
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
    cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    configured[dev] = true;
  }
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
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_kernel, x, W, ldw, out, N, K, pl.kchunk, p, epi);
  if (e != cudaSuccess) return e;
  if (pl.groups > 1)
    skinny_finish<<<uint32_t((N + 255) / 256), 256, 0, s>>>(part, pl.groups, out, N, 1, N, epi);
  return cudaSuccess;
}

template <int MR, int CPL, int UNROLL>
void launch_skinny(const SkinnyPlan &pl, const float *X, int64_t ldx, const float *W, int64_t ldw, float *out,
                   int64_t ldo, int64_t M, int64_t N, int64_t K, float *part, const Epi &epi,
                   cudaStream_t s) {
  constexpr int COLS = 32 * CPL;
  dim3 grid(uint32_t((N + COLS - 1) / COLS), uint32_t(pl.groups * kSkinnyCluster),
            uint32_t((M + MR - 1) / MR));
  const size_t smem = (size_t(9) * MR * COLS + size_t(MR) * pl.kchunk) * sizeof(float);
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaFuncSetAttribute(skinny_gemm<MR, CPL, UNROLL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         int((9 * MR * COLS + MR * kSkinnyMaxChunk) * sizeof(float)));
    configured[dev] = true;
  }
  skinny_gemm<MR, CPL, UNROLL><<<grid, 256, smem, s>>>(X, ldx, W, ldw, out, ldo, M, N, K, pl.kchunk,
                                                       pl.groups > 1 ? part : nullptr, epi);
  if (pl.groups > 1) {
    const int64_t total = M * N;
    skinny_finish<<<uint32_t((total + 255) / 256), 256, 0, s>>>(part, pl.groups, out, ldo, M, N, epi);
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
      if (a->M == 1) return gemv_part_bytes(gemv_plan(a->N, a->K), a->N);
      SkinnyPlan pl = skinny_plan(a->M, a->N, a->K);
      return skinny_part_bytes(pl, a->M, a->N);
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
  if (path == kPathSkinny && a.M == 1) {
    const GemvPlan pl = gemv_plan(a.N, a.K);
    const size_t need = gemv_part_bytes(pl, a.N);
    if (need && (!ws || wsb < need))
      return fail(SILCU_WORKSPACE_TOO_SMALL, "sgemm(gemv): workspace %zu < %zu", wsb, need);
    const cudaError_t e = launch_gemv(pl, a.A, a.B, a.ldb, a.C, a.N, a.K, static_cast<float *>(ws), epi, s);
    if (e != cudaSuccess) return fail(SILCU_CUDA_ERROR, "sgemm(gemv): %s", cudaGetErrorString(e));
    return check_launch("sgemm(gemv)", pl.groups > 1 ? 2 : 1);
  }
  if (path == kPathSkinny) {
    SkinnyPlan pl = skinny_plan(a.M, a.N, a.K);
    const size_t need = skinny_part_bytes(pl, a.M, a.N);
    if (need && (!ws || wsb < need))
      return fail(SILCU_WORKSPACE_TOO_SMALL, "sgemm(skinny): workspace %zu < %zu", wsb, need);
    float *part = static_cast<float *>(ws);
    switch (pl.mr) {
      case 8: launch_skinny<8, 2, 8>(pl, a.A, a.lda, a.B, a.ldb, a.C, a.ldc, a.M, a.N, a.K, part, epi, s); break;
      case 16: launch_skinny<16, 1, 8>(pl, a.A, a.lda, a.B, a.ldb, a.C, a.ldc, a.M, a.N, a.K, part, epi, s); break;
      default: launch_skinny<32, 1, 4>(pl, a.A, a.lda, a.B, a.ldb, a.C, a.ldc, a.M, a.N, a.K, part, epi, s); break;
    }
    return check_launch("sgemm(skinny)", pl.groups > 1 ? 2 : 1);
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

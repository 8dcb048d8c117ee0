// Skinny GEMM, C[M, N] = X[M, K] . W[K, N] for 2 <= M <= 32 (the "small
// batch" of the reference's linear layers, include/array.h:1375-1416): an
// HBM-bound stream of W in which every W element feeds M FMAs.
//
// Design (one wave, everything requested up front):
//   * the grid is (column blocks of 64) x (C slices of K); the C CTAs of a
//     column block form one thread-block cluster, and C is chosen with the
//     occupancy API so that every CTA of the grid is resident at once;
//   * at start, one thread issues TMA tile loads of the CTA's whole W slice
//     and X slice into shared memory (per chunk of 32 k: a 64-column x 32-row
//     W box and a 32-k x R-row X box, zero-filled past K, N and M): ~100-200
//     KB in flight per SM, the whole matrix requested in the first
//     microseconds; each chunk has its own mbarrier, so the FMAs start on the
//     first chunk while the rest streams in;
//   * 256 threads: lane l owns columns 2l, 2l+1 of the block for all R rows
//     (R = 16 or 32; 2R accumulators), warp w takes k = 4w..4w+3 of every
//     32-k chunk; per 4 k a thread does 8R FMAs for R broadcast 128-bit X
//     loads and four 64-bit W loads;
//   * the 8 warps' partials meet in shared memory in a fixed tree, then the
//     C CTAs of the cluster add their partials in rank order through
//     distributed shared memory (each CTA finishes 1/C of the tile) and
//     apply the epilogue: alpha, bias, activation, residual, in the
//     reference's order.
// Every sum runs in a fixed order, so results are deterministic.  All waits
// are bounded (tc::mbar_wait); no multicast.
#include <cooperative_groups.h>
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "gemm_internal.cuh"
#include "tc_common.cuh"

namespace silcu {
namespace {

constexpr int kCols = 64;     // columns per CTA
constexpr int kChunk = 32;    // k rows per mbarrier
constexpr int kThreads = 256;
constexpr int kMaxChunks = 32;  // kslice <= 1024
constexpr int kHead = 1024;     // mbarriers ahead of the data

template <int R>
size_t smem_bytes(int kslice) {
  const size_t data = size_t(kslice) * (kCols + R) * sizeof(float);
  const size_t red = size_t(4 + 1) * R * kCols * sizeof(float);  // tree scratch + CTA partial
  return kHead + (data > red ? data : red);
}

struct __align__(64) SkinnyMaps {
  CUtensorMap w;  // W [K rows, N cols], boxes of 64 cols x 32 rows
  CUtensorMap x;  // X [M rows, K cols], boxes of 32 k x R rows
};

template <int R>
__global__ void __launch_bounds__(kThreads, 2)
    skinny_gemm(const __grid_constant__ SkinnyMaps maps, float *__restrict__ out, int64_t ldo, int M, int64_t N,
                int64_t K, int kslice, SkinnyEpi epi, int *err) {
  namespace cg = cooperative_groups;
  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm);  // [c] = chunk c (W and X boxes)
  float *Ws = reinterpret_cast<float *>(sm + kHead);  // [kslice][64]
  float *Xs = Ws + size_t(kslice) * kCols;           // per chunk c: [R][32] at c * R * 32
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t col0 = int64_t(blockIdx.x) * kCols;
  const int64_t k0 = int64_t(blockIdx.y) * kslice;
  const int kn = int(k0 + kslice <= K ? kslice : (K > k0 ? K - k0 : 0));  // k rows of this slice
  const int nch = (kn + kChunk - 1) / kChunk;
  constexpr uint32_t kChunkBytes = uint32_t(kChunk) * (kCols + R) * 4;

  if (tid == 0) {
    for (int c = 0; c < nch; c++) tc::mbar_init(tc::smem_u32(bars + c), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0) {
    // The whole slice at once: one W box and one X box per chunk (boxes past
    // K or N read as zeros and still count their full size).
    for (int c = 0; c < nch; c++) {
      const uint32_t bar = tc::smem_u32(bars + c);
      tc::mbar_expect_tx(bar, kChunkBytes);
      const int kc = int(k0) + c * kChunk;
      tc::tma_load_4d(tc::smem_u32(Ws + size_t(c) * kChunk * kCols), &maps.w, bar, int(col0), kc, 0, 0);
      tc::tma_load_4d(tc::smem_u32(Xs + size_t(c) * R * kChunk), &maps.x, bar, kc, 0, 0, 0);
    }
  }

  float acc[R][2];
#pragma unroll
  for (int r = 0; r < R; r++) acc[r][0] = acc[r][1] = 0.0f;
  bool ok = true;
  for (int c = 0; c < nch; c++) {
    ok = tc::mbar_wait(tc::smem_u32(bars + c), 0, err, 62);
    if (!ok) break;
    const int kk = 4 * warp;  // this warp's 4 k of the chunk (zeros past the slice end)
    const float *wr = Ws + (size_t(c) * kChunk + kk) * kCols + 2 * lane;
    float w[4][2];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const float2 v = *reinterpret_cast<const float2 *>(wr + u * kCols);
      w[u][0] = v.x;
      w[u][1] = v.y;
    }
    const float *xr = Xs + size_t(c) * R * kChunk + kk;
#pragma unroll
    for (int r = 0; r < R; r++) {
      const float4 x = *reinterpret_cast<const float4 *>(xr + r * kChunk);
      acc[r][0] = fmaf(x.x, w[0][0], acc[r][0]);
      acc[r][1] = fmaf(x.x, w[0][1], acc[r][1]);
      acc[r][0] = fmaf(x.y, w[1][0], acc[r][0]);
      acc[r][1] = fmaf(x.y, w[1][1], acc[r][1]);
      acc[r][0] = fmaf(x.z, w[2][0], acc[r][0]);
      acc[r][1] = fmaf(x.z, w[2][1], acc[r][1]);
      acc[r][0] = fmaf(x.w, w[3][0], acc[r][0]);
      acc[r][1] = fmaf(x.w, w[3][1], acc[r][1]);
    }
  }
  // Rows >= M are zeros (the X boxes are zero-filled past M) and are never
  // stored.  The tree below sums warps in a fixed order.
  __syncthreads();  // all FMAs done: the data region becomes the tree scratch
  float *tree = reinterpret_cast<float *>(sm + kHead);  // [4][R][64]
  float *part = tree + 4 * R * kCols;                   // [R][64] CTA partial
  for (int half = 4; half >= 1; half >>= 1) {
    if (warp >= half && warp < 2 * half) {
      float *dst = tree + size_t(warp - half) * R * kCols;
#pragma unroll
      for (int r = 0; r < R; r++)
        *reinterpret_cast<float2 *>(dst + r * kCols + 2 * lane) = make_float2(acc[r][0], acc[r][1]);
    }
    __syncthreads();
    if (warp < half) {
      const float *src = tree + size_t(warp) * R * kCols;
#pragma unroll
      for (int r = 0; r < R; r++) {
        const float2 v = *reinterpret_cast<const float2 *>(src + r * kCols + 2 * lane);
        acc[r][0] += v.x;
        acc[r][1] += v.y;
      }
    }
    __syncthreads();
  }
  if (warp == 0) {
#pragma unroll
    for (int r = 0; r < R; r++)
      *reinterpret_cast<float2 *>(part + r * kCols + 2 * lane) = make_float2(acc[r][0], acc[r][1]);
  }
  cg::cluster_group cl = cg::this_cluster();
  cl.sync();  // every CTA's partial is complete
  const int C = int(cl.num_blocks()), q = int(cl.block_rank());
  constexpr int E = R * kCols;
  const int per = (E + C - 1) / C;
  const bool good = ok && *reinterpret_cast<volatile int *>(err) == 0;
  for (int e = q * per + tid; e < (q + 1) * per && e < E; e += kThreads) {
    const int r = e / kCols, cc = e % kCols;
    if (r >= M || col0 + cc >= N || !good) continue;
    float v = 0.0f;
    for (int j = 0; j < C; j++) v += cl.map_shared_rank(part, j)[e];
    const int64_t row = r, col = col0 + cc;
    if (epi.alpha != 1.0f) v = __fmul_rn(v, epi.alpha);
    if (epi.bias) v = __fadd_rn(v, __ldg(epi.bias + (col % epi.bias_len)));
    if (epi.act == SILCU_ACT_RELU) v = v >= 0.0f ? v : 0.0f;
    else if (epi.act == SILCU_ACT_SIGMOID) v = sigmoid_ref(v);
    if (epi.residual) v = __fadd_rn(v, __ldg(epi.residual + row * epi.ldr + col));
    out[row * ldo + col] = v;
  }
  cl.sync();  // peers keep their shared memory until everyone has read it
}

struct SkinnyPlan {
  int R, C, kslice;
  size_t smem;
};

template <int R>
bool configure(int C, size_t smem) {
  static bool done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !done[dev]) {
    cudaFuncSetAttribute(skinny_gemm<R>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    cudaFuncSetAttribute(skinny_gemm<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    done[dev] = true;
  }
  (void)C;
  (void)smem;
  return true;
}

// Resident clusters of C CTAs with `smem` bytes each (0 if unknown).
template <int R>
int resident_ctas(int C, size_t smem) {
  configure<R>(C, smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, unsigned(C), 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = unsigned(C);
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, skinny_gemm<R>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n * C;
}

// The cluster size C (K slices per column block) with the shortest
// estimated time: time ~ (work per CTA) x (CTAs per SM), all CTAs resident
// (otherwise a second wave doubles it); slices of at least 64 k.
template <int R>
SkinnyPlan plan_for(int64_t N, int64_t K) {
  const int64_t cb = (N + kCols - 1) / kCols;
  const int sms = sm_count();
  SkinnyPlan best{R, 0, 0, 0};
  double best_cost = 1e300;
  for (int C = 16; C >= 1; C--) {
    int64_t ks = (K + C - 1) / C;
    ks = (ks + kChunk - 1) / kChunk * kChunk;
    if (ks > int64_t(kChunk) * kMaxChunks) continue;
    if (C > 1 && ks < 64) continue;
    if ((K + ks - 1) / ks < C) continue;  // every slice non-empty
    const size_t smem = smem_bytes<R>(int(ks));
    if (smem > 227 * 1024) continue;
    const int64_t ctas = cb * C;
    const int cap = resident_ctas<R>(C, smem);
    if (cap <= 0) continue;
    const double waves = double((ctas + cap - 1) / cap);
    const double per_sm = double((ctas + sms - 1) / sms);
    const double cost = double(ks) * per_sm * waves + 2.0 * C;  // + the cluster combine
    if (cost < best_cost) {
      best_cost = cost;
      best = SkinnyPlan{R, C, int(ks), smem};
    }
  }
  return best;
}

template <int R>
silcu_status run(const silcu_gemm_args &a, const SkinnyEpi &epi, cudaStream_t s) {
  struct Key {
    int64_t N, K;
    int dev;
  };
  static Key keys[16];
  static SkinnyPlan plans[16];
  static int n_cached = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  SkinnyPlan pl{R, 0, 0, 0};
  for (int i = 0; i < n_cached; i++)
    if (keys[i].N == a.N && keys[i].K == a.K && keys[i].dev == dev) pl = plans[i];
  if (pl.C == 0) {
    pl = plan_for<R>(a.N, a.K);
    if (pl.C == 0) return fail(SILCU_UNSUPPORTED, "sgemm(skinny): no launchable plan");
    const int slot = n_cached < 16 ? n_cached++ : int(a.K % 16);
    keys[slot] = Key{a.N, a.K, dev};
    plans[slot] = pl;
  }
  configure<R>(pl.C, pl.smem);
  int *err = device_error_ptr();
  if (!err) return fail(SILCU_CUDA_ERROR, "sgemm(skinny): no device error word");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned((a.N + kCols - 1) / kCols), unsigned(pl.C), 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = unsigned(pl.C);
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  SkinnyMaps maps;
  const CUtensorMapSwizzle none = CU_TENSOR_MAP_SWIZZLE_NONE;
  if (!tc::make_map4(&maps.w, a.B, a.N, a.K, a.ldb, 1, 0, 1, 0, kCols, kChunk, none) ||
      !tc::make_map4(&maps.x, a.A, a.K, a.M, a.lda, 1, 0, 1, 0, kChunk, R, none))
    return fail(SILCU_CUDA_ERROR, "sgemm(skinny): cuTensorMapEncodeTiled failed");
  cudaError_t e = cudaLaunchKernelEx(&cfg, skinny_gemm<R>, maps, a.C, int64_t(a.ldc), int(a.M), int64_t(a.N),
                                     int64_t(a.K), pl.kslice, epi, err);
  if (e != cudaSuccess) return fail(SILCU_CUDA_ERROR, "sgemm(skinny): %s", cudaGetErrorString(e));
  return check_launch("sgemm(skinny)");
}

}  // namespace

bool skinny_tma_eligible(const silcu_gemm_args &a) {
  static const int off = [] {
    const char *e = getenv("SILCU_SKINNY_TMA");
    return e && atoi(e) == 0;
  }();
  if (off) return false;
  // tensor maps need 16-byte aligned bases and row strides (lda, ldb
  // multiples of 4 floats); the boxes' x coordinates (col0, k) are multiples
  // of 32 floats.
  return a.M >= 2 && a.M <= 32 && !a.trans_a && !a.trans_b && a.batch == 1 && a.batch_inner <= 1 &&
         a.lda % 4 == 0 && a.ldb % 4 == 0 && aligned16(a.A) && aligned16(a.B) &&
         a.K >= 64 && a.K <= int64_t(16) * kChunk * kMaxChunks && (!a.residual || a.ldr >= a.N);
}

silcu_status skinny_tma_run(const silcu_gemm_args &a, const SkinnyEpi &epi, cudaStream_t s) {
  return a.M <= 16 ? run<16>(a, epi, s) : run<32>(a, epi, s);
}

}  // namespace silcu

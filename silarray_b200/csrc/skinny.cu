// Skinny GEMM, C[M, N] = X[M, K] . W[K, N] for 2 <= M <= 32 (the "small
// batch" of the reference's linear layers, include/array.h:1375-1416): an
// HBM-bound stream of W in which every W element feeds M FMAs.
//
// Design (one wave, everything requested up front):
//   * the grid is (column blocks of BW = 32 or 64) x (C slices of K); the C
//     CTAs of a column block form one thread-block cluster; BW and C are
//     chosen with the occupancy API so that every CTA is resident at once,
//     preferably two per SM (16 warps), with the FMA work spread evenly;
//   * at start, one thread issues TMA tile loads of the CTA's whole W slice
//     and X slice into shared memory (per chunk of CH k: a BW-column x CH-row
//     W box of 8 KB and a CH-k x R-row X box, zero-filled past K, N and M):
//     the whole matrix is requested in the first microseconds; each chunk has
//     its own mbarrier, so the FMAs start on the first chunk while the rest
//     streams in;
//   * 256 threads: a thread owns 2 columns for all R rows (R = 16 or 32; 2R
//     accumulators) and 4 k of every chunk (warp w, and for BW = 32 the two
//     half-warps, take different k); per 4 k a thread does 8R FMAs for R
//     broadcast 128-bit X loads and four 64-bit W loads;
//   * the partials of the half-warps (shuffle) and of the 8 warps (shared
//     memory, a fixed tree) meet, then the C CTAs of the cluster add theirs
//     in rank order through distributed shared memory (each CTA finishes 1/C
//     of the tile) and apply the epilogue: alpha, bias, activation, residual,
//     in the reference's order.
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

constexpr int kThreads = 256;
constexpr int kMaxChunks = 32;
constexpr int kHead = 1024;  // mbarriers ahead of the data

// k rows per chunk: 8 warps x 4 k x (64 / BW) half-warps; the W box is 8 KB.
template <int BW>
__host__ __device__ constexpr int chunk_k() {
  return 8 * 4 * (64 / BW);
}

template <int R, int BW>
size_t smem_bytes(int kslice) {
  const size_t data = size_t(kslice) * (BW + R) * sizeof(float);
  const size_t red = size_t(4 + 1) * R * BW * sizeof(float);  // tree scratch + CTA partial
  return kHead + (data > red ? data : red);
}

struct __align__(64) SkinnyMaps {
  CUtensorMap w;  // W [K rows, N cols], boxes of BW cols x CH rows
  CUtensorMap x;  // X [M rows, K cols], boxes of CH k x R rows
};

template <int R, int BW>
__global__ void __launch_bounds__(kThreads, 2)
    skinny_gemm(const __grid_constant__ SkinnyMaps maps, float *__restrict__ out, int64_t ldo, int M, int64_t N,
                int64_t K, int kslice, SkinnyEpi epi, int *err) {
  namespace cg = cooperative_groups;
  constexpr int CH = chunk_k<BW>();
  constexpr int HL = 32 / (64 / BW);  // lanes per half-warp group (32 or 16)
  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm);  // [c] = chunk c (W and X boxes)
  float *Ws = reinterpret_cast<float *>(sm + kHead);  // per chunk c: [CH][BW] at c * CH * BW
  float *Xs = Ws + size_t(kslice) * BW;              // per chunk c: [R][CH] at c * R * CH
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int half = lane / HL, cl_lane = lane % HL;
  const int64_t col0 = int64_t(blockIdx.x) * BW;
  const int64_t k0 = int64_t(blockIdx.y) * kslice;
  const int kn = int(k0 + kslice <= K ? kslice : (K > k0 ? K - k0 : 0));  // k rows of this slice
  const int nch = (kn + CH - 1) / CH;
  constexpr uint32_t kChunkBytes = uint32_t(CH) * (BW + R) * 4;

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
      const int kc = int(k0) + c * CH;
      tc::tma_load_4d(tc::smem_u32(Ws + size_t(c) * CH * BW), &maps.w, bar, int(col0), kc, 0, 0);
      tc::tma_load_4d(tc::smem_u32(Xs + size_t(c) * R * CH), &maps.x, bar, kc, 0, 0, 0);
    }
  }

  float acc[R][2];
#pragma unroll
  for (int r = 0; r < R; r++) acc[r][0] = acc[r][1] = 0.0f;
  bool ok = true;
  const int kk = 4 * ((64 / BW) * warp + half);  // this thread's 4 k of every chunk
  for (int c = 0; c < nch; c++) {
    ok = tc::mbar_wait(tc::smem_u32(bars + c), 0, err, 62);
    if (!ok) break;
    const float *wr = Ws + (size_t(c) * CH + kk) * BW + 2 * cl_lane;
    float w[4][2];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const float2 v = *reinterpret_cast<const float2 *>(wr + u * BW);
      w[u][0] = v.x;
      w[u][1] = v.y;
    }
    const float *xr = Xs + size_t(c) * R * CH + kk;
#pragma unroll
    for (int r = 0; r < R; r++) {
      const float4 x = *reinterpret_cast<const float4 *>(xr + r * CH);
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
  // The two half-warps of a BW = 32 CTA hold partials of the same outputs:
  // the lower half adds the upper's (fixed order).
  if constexpr (BW == 32) {
#pragma unroll
    for (int r = 0; r < R; r++) {
      acc[r][0] += __shfl_down_sync(0xffffffffu, acc[r][0], 16);
      acc[r][1] += __shfl_down_sync(0xffffffffu, acc[r][1], 16);
    }
  }
  // Rows >= M are zeros (the X boxes are zero-filled past M) and are never
  // stored.  The tree below sums warps in a fixed order.
  __syncthreads();  // all FMAs done: the data region becomes the tree scratch
  float *tree = reinterpret_cast<float *>(sm + kHead);  // [4][R][BW]
  float *part = tree + 4 * R * BW;                      // [R][BW] CTA partial
  const bool writer = half == 0;
  for (int h = 4; h >= 1; h >>= 1) {
    if (warp >= h && warp < 2 * h && writer) {
      float *dst = tree + size_t(warp - h) * R * BW;
#pragma unroll
      for (int r = 0; r < R; r++)
        *reinterpret_cast<float2 *>(dst + r * BW + 2 * cl_lane) = make_float2(acc[r][0], acc[r][1]);
    }
    __syncthreads();
    if (warp < h && writer) {
      const float *src = tree + size_t(warp) * R * BW;
#pragma unroll
      for (int r = 0; r < R; r++) {
        const float2 v = *reinterpret_cast<const float2 *>(src + r * BW + 2 * cl_lane);
        acc[r][0] += v.x;
        acc[r][1] += v.y;
      }
    }
    __syncthreads();
  }
  if (warp == 0 && writer) {
#pragma unroll
    for (int r = 0; r < R; r++)
      *reinterpret_cast<float2 *>(part + r * BW + 2 * cl_lane) = make_float2(acc[r][0], acc[r][1]);
  }
  cg::cluster_group cl = cg::this_cluster();
  cl.sync();  // every CTA's partial is complete
  const int C = int(cl.num_blocks()), q = int(cl.block_rank());
  constexpr int E = R * BW;
  const int per = (E + C - 1) / C;
  const bool good = ok && *reinterpret_cast<volatile int *>(err) == 0;
  for (int e = q * per + tid; e < (q + 1) * per && e < E; e += kThreads) {
    const int r = e / BW, cc = e % BW;
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
  int BW, C, kslice;
  size_t smem;
};

template <int R, int BW>
void configure() {
  static bool done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !done[dev]) {
    cudaFuncSetAttribute(skinny_gemm<R, BW>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    cudaFuncSetAttribute(skinny_gemm<R, BW>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    done[dev] = true;
  }
}

// Resident CTAs of the grid in clusters of C with `smem` bytes each (0 if
// the occupancy query fails, e.g. without a device).
template <int R, int BW>
int resident_ctas(int C, size_t smem) {
  configure<R, BW>();
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
  if (cudaOccupancyMaxActiveClusters(&n, skinny_gemm<R, BW>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n * C;
}

// Estimated time of one configuration in FMA rows (per SM: CTAs on the
// busiest SM x k rows x columns), x2 per extra wave, x1.4 when an SM holds
// a single CTA (8 warps hide less latency).
template <int R, int BW>
void consider(int64_t N, int64_t K, SkinnyPlan &best, double &best_cost) {
  constexpr int CH = chunk_k<BW>();
  const int64_t cb = (N + BW - 1) / BW;
  const int sms = sm_count();
  const char *fc = getenv("SILCU_SKINNY_C");
  const int force_c = fc ? atoi(fc) : 0;
  for (int C = 16; C >= 1; C--) {
    if (force_c && C != force_c) continue;
    int64_t ks = (K + C - 1) / C;
    ks = (ks + CH - 1) / CH * CH;
    if (ks / CH > kMaxChunks) continue;
    if ((K + ks - 1) / ks < C) continue;  // every slice non-empty
    const size_t smem = smem_bytes<R, BW>(int(ks));
    if (smem > 227 * 1024) continue;
    const int64_t ctas = cb * C;
    const int cap = resident_ctas<R, BW>(C, smem);
    if (cap <= 0) continue;
    const int64_t live = ctas < cap ? ctas : cap;
    const double waves = double((ctas + cap - 1) / cap);
    const double per_sm = double((live + sms - 1) / sms);
    const double cost = waves * per_sm * double(ks) * BW * (per_sm < 2 ? 1.4 : 1.0) + 64.0 * C;
    if (cost < best_cost) {
      best_cost = cost;
      best = SkinnyPlan{BW, C, int(ks), smem};
    }
  }
}

// SILCU_SKINNY_BW (32 / 64) and SILCU_SKINNY_C (1..16) restrict the choice (tuning).
template <int R>
SkinnyPlan plan_for(int64_t N, int64_t K) {
  SkinnyPlan best{0, 0, 0, 0};
  double best_cost = 1e300;
  const char *bw = getenv("SILCU_SKINNY_BW");
  const int force_bw = bw ? atoi(bw) : 0;
  if (force_bw != 32) consider<R, 64>(N, K, best, best_cost);
  if (force_bw != 64) consider<R, 32>(N, K, best, best_cost);
  return best;
}

// Plans are cached per (N, K, device): the occupancy queries cost ~10 us.
template <int R>
SkinnyPlan cached_plan(int64_t N, int64_t K) {
  struct Key {
    int64_t N, K;
    int dev;
  };
  static Key keys[32];
  static SkinnyPlan plans[32];
  static int n_cached = 0, next = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  for (int i = 0; i < n_cached; i++)
    if (keys[i].N == N && keys[i].K == K && keys[i].dev == dev) return plans[i];
  const SkinnyPlan pl = plan_for<R>(N, K);
  const int slot = n_cached < 32 ? n_cached++ : (next++ & 31);
  keys[slot] = Key{N, K, dev};
  plans[slot] = pl;
  return pl;
}

template <int R, int BW>
silcu_status launch(const silcu_gemm_args &a, const SkinnyPlan &pl, const SkinnyEpi &epi, cudaStream_t s) {
  configure<R, BW>();
  int *err = device_error_ptr();
  if (!err) return fail(SILCU_CUDA_ERROR, "sgemm(skinny): no device error word");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned((a.N + BW - 1) / BW), unsigned(pl.C), 1);
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
  constexpr int CH = chunk_k<BW>();
  if (!tc::make_map4(&maps.w, a.B, a.N, a.K, a.ldb, 1, 0, 1, 0, BW, CH, none) ||
      !tc::make_map4(&maps.x, a.A, a.K, a.M, a.lda, 1, 0, 1, 0, CH, R, none))
    return fail(SILCU_CUDA_ERROR, "sgemm(skinny): cuTensorMapEncodeTiled failed");
  cudaError_t e = cudaLaunchKernelEx(&cfg, skinny_gemm<R, BW>, maps, a.C, int64_t(a.ldc), int(a.M),
                                     int64_t(a.N), int64_t(a.K), pl.kslice, epi, err);
  if (e != cudaSuccess) return fail(SILCU_CUDA_ERROR, "sgemm(skinny): %s", cudaGetErrorString(e));
  return check_launch("sgemm(skinny)");
}

template <int R>
silcu_status run(const silcu_gemm_args &a, const SkinnyEpi &epi, cudaStream_t s) {
  const SkinnyPlan pl = cached_plan<R>(a.N, a.K);
  if (pl.C == 0) return fail(SILCU_UNSUPPORTED, "sgemm(skinny): no launchable plan");
  return pl.BW == 32 ? launch<R, 32>(a, pl, epi, s) : launch<R, 64>(a, pl, epi, s);
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
         a.lda % 4 == 0 && a.ldb % 4 == 0 && aligned16(a.A) && aligned16(a.B) && a.K >= 64 &&
         (!a.residual || a.ldr >= a.N) &&
         (a.M <= 16 ? cached_plan<16>(a.N, a.K).C : cached_plan<32>(a.N, a.K).C) > 0;
}

silcu_status skinny_tma_run(const silcu_gemm_args &a, const SkinnyEpi &epi, cudaStream_t s) {
  return a.M <= 16 ? run<16>(a, epi, s) : run<32>(a, epi, s);
}

}  // namespace silcu

// Reductions: whole-array sum/min/max/argmax, row-wise softmax / layer_norm /
// argmax, and sum over an axis.  All HBM-bound; each input byte is read once.
//
// Whole-array reductions use a fixed grid (a multiple of the SM count) whose
// CTAs write one partial each into the caller's workspace, then a one-CTA
// finish kernel combines the partials in index order, so results are
// deterministic for a given GPU.
//
// Row ops keep the whole row on chip (each thread's VPT float4 in registers,
// or, for rows of 4K-32K columns, the row in shared memory by one bulk copy
// per CTA), so softmax and layer_norm read HBM once and write once (the
// reference reads the row 2-3 times: include/gpu_kernels.metal:1316-1467).
#include <atomic>
#include <stdlib.h>
#include <cooperative_groups.h>
#include <float.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace silcu {
namespace {


// ------------------------------------------------------------- block reduce
template <int NT, typename T, typename F>
__device__ __forceinline__ T block_reduce(T v, T *smem, F op) {
  constexpr int NW = NT / 32;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (NW == 1) return v;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) smem[w] = v;
  __syncthreads();
  T r = smem[0];
#pragma unroll
  for (int i = 1; i < NW; i++) r = op(r, smem[i]);  // broadcast reads, fixed order
  __syncthreads();  // smem is reused by the next reduction
  return r;
}

// Row reduction: a whole warp per row (WARP) or the whole CTA.
template <int NT, bool WARP, typename T, typename F>
__device__ __forceinline__ T row_reduce(T v, T *smem, F op) {
  if (WARP) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
  }
  return block_reduce<NT>(v, smem, op);
}

struct Add {
  template <typename T>
  __device__ T operator()(T a, T b) const { return a + b; }
};
struct Max {
  __device__ float operator()(float a, float b) const { return fmaxf(a, b); }
  __device__ unsigned long long operator()(unsigned long long a, unsigned long long b) const {
    return a > b ? a : b;
  }
};

// Orderable encoding of a float: unsigned compare == float compare.
__device__ __forceinline__ uint32_t ord(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unord(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}
// Argmax key: larger value wins, then the smaller index.  Only values above
// FLT_MIN are candidates (include/array.h:1733-1740 starts its running max at
// numeric_limits<float>::min() and compares with a strict '>'); NaN never is.
__device__ __forceinline__ unsigned long long amax_key(float v, uint64_t idx) {
  if (!(v > FLT_MIN)) return 0ull;
  return (uint64_t(ord(v)) << 32) | uint64_t(0xFFFFFFFFu - uint32_t(idx));
}

// ---------------------------------------------------- whole-array reductions
constexpr int kRedThreads = 512;
constexpr int kRedCtasPerSm = 4;
constexpr int kMaxPartials = 4096;

enum RedKind { kSum = 0, kMinK = 1, kMaxK = 2, kSumI = 3, kArgmax = 4 };

template <int KIND>
struct RedT;
template <> struct RedT<kSum> { using T = double; };
template <> struct RedT<kMinK> { using T = float; };
template <> struct RedT<kMaxK> { using T = float; };
template <> struct RedT<kSumI> { using T = uint32_t; };
template <> struct RedT<kArgmax> { using T = unsigned long long; };

template <int KIND>
__device__ __forceinline__ typename RedT<KIND>::T red_identity() {
  if (KIND == kMinK) return __int_as_float(0x7f800000);   // +inf
  if (KIND == kMaxK) return __int_as_float(0xff800000);   // -inf
  return 0;
}

template <int KIND, typename T>
__device__ __forceinline__ T red_op(T a, T b) {
  if (KIND == kMinK) return fminf(a, b);
  if (KIND == kMaxK) return fmaxf(a, b);
  if (KIND == kArgmax) return a > b ? a : b;
  return a + b;
}

template <int KIND, typename In>
__device__ __forceinline__ typename RedT<KIND>::T red_elem(In v, uint64_t idx) {
  if (KIND == kSum) return double(v);
  if (KIND == kSumI) return uint32_t(v);
  if (KIND == kArgmax) return amax_key(float(v), idx);
  return float(v);
}

template <int KIND, typename In>
__global__ void __launch_bounds__(kRedThreads) reduce_partials(const In *__restrict__ in, uint64_t n,
                                                               typename RedT<KIND>::T *__restrict__ part) {
  using T = typename RedT<KIND>::T;
  __shared__ T smem[kRedThreads / 32];
  T acc = red_identity<KIND>();
  const uint64_t tid = uint64_t(blockIdx.x) * kRedThreads + threadIdx.x;
  const uint64_t nthreads = uint64_t(gridDim.x) * kRedThreads;
  const bool vec = (reinterpret_cast<uintptr_t>(in) & 15) == 0;
  const uint64_t n4 = vec ? n / 4 : 0;
  // 4 independent 16-byte loads in flight per thread per iteration.
  uint64_t i = tid;
  for (; i + 3 * nthreads < n4; i += 4 * nthreads) {
    float4 f[4];
#pragma unroll
    for (int u = 0; u < 4; u++) f[u] = __ldcs(reinterpret_cast<const float4 *>(in) + i + u * nthreads);
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const In *e = reinterpret_cast<const In *>(&f[u]);
      const uint64_t base = (i + u * nthreads) * 4;
#pragma unroll
      for (int k = 0; k < 4; k++) acc = red_op<KIND>(acc, red_elem<KIND>(e[k], base + k));
    }
  }
  for (; i < n4; i += nthreads) {
    float4 f = __ldcs(reinterpret_cast<const float4 *>(in) + i);
    const In *e = reinterpret_cast<const In *>(&f);
#pragma unroll
    for (int k = 0; k < 4; k++) acc = red_op<KIND>(acc, red_elem<KIND>(e[k], i * 4 + k));
  }
  for (uint64_t j = n4 * 4 + tid; j < n; j += nthreads) acc = red_op<KIND>(acc, red_elem<KIND>(in[j], j));
  // block reduce
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc = red_op<KIND>(acc, __shfl_xor_sync(0xffffffffu, acc, o));
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) smem[w] = acc;
  __syncthreads();
  if (w == 0) {
    T r = lane < kRedThreads / 32 ? smem[lane] : red_identity<KIND>();
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) r = red_op<KIND>(r, __shfl_xor_sync(0xffffffffu, r, o));
    if (lane == 0) part[blockIdx.x] = r;
  }
}

template <int KIND, typename Out>
__global__ void __launch_bounds__(1024) reduce_finish(const typename RedT<KIND>::T *__restrict__ part,
                                                      int nparts, Out *__restrict__ out,
                                                      float *__restrict__ out_value,
                                                      const float *__restrict__ in) {
  using T = typename RedT<KIND>::T;
  __shared__ T smem[32];
  T acc = red_identity<KIND>();
  for (int i = threadIdx.x; i < nparts; i += 1024) acc = red_op<KIND>(acc, part[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc = red_op<KIND>(acc, __shfl_xor_sync(0xffffffffu, acc, o));
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) smem[w] = acc;
  __syncthreads();
  if (w == 0) {
    T r = smem[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) r = red_op<KIND>(r, __shfl_xor_sync(0xffffffffu, r, o));
    if (lane == 0) {
      if (KIND == kSum) {
        *reinterpret_cast<float *>(out) = float(r);
      } else if (KIND == kArgmax) {
        const unsigned long long key = (unsigned long long)r;
        const int64_t idx = key ? int64_t(0xFFFFFFFFu - uint32_t(key & 0xFFFFFFFFu)) : 0;
        *reinterpret_cast<int64_t *>(out) = idx;
        if (out_value) *out_value = key ? unord(uint32_t(key >> 32)) : in[0];
      } else {
        *out = Out(r);
      }
    }
  }
}

// Small float sums (n <= kSeqSumMax) are added sequentially in fp32, in index
// order, exactly as the reference's CPU sum (vDSP_sve / std::accumulate,
// include/cpu.h:266-274) does, so they match it bit for bit; larger sums
// accumulate in fp64 and round once.
constexpr int kSeqSumMax = 4096;

__global__ void __launch_bounds__(256) sum_seq_small(const float *__restrict__ in, int n, float *out) {
  __shared__ float buf[kSeqSumMax];
  for (int i = threadIdx.x; i < n; i += 256) buf[i] = in[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int i = 0; i < n; i++) s = __fadd_rn(s, buf[i]);
    *out = s;
  }
}

int red_grid(uint64_t n) {
  uint64_t want = (n + kRedThreads * 16 - 1) / (kRedThreads * 16);
  uint64_t cap = uint64_t(sm_count()) * kRedCtasPerSm;
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  if (want > kMaxPartials) want = kMaxPartials;
  return int(want);
}

template <int KIND, typename In, typename Out>
silcu_status run_reduce(const char *name, const In *in, size_t n, Out *out, float *out_value,
                        void *ws, size_t ws_bytes, silcu_stream stream) {
  using T = typename RedT<KIND>::T;
  if (!in || !out) return fail(SILCU_INVALID_ARGUMENT, "%s: null pointer", name);
  if (n == 0) return fail(SILCU_INVALID_ARGUMENT, "%s: empty input", name);
  if (KIND == kArgmax && n > 0xFFFFFFFFull) return fail(SILCU_UNSUPPORTED, "%s: n >= 2^32", name);
  const int g = red_grid(n);
  if (!ws || ws_bytes < size_t(g) * sizeof(T))
    return fail(SILCU_WORKSPACE_TOO_SMALL, "%s: workspace %zu < %zu", name, ws_bytes, size_t(g) * sizeof(T));
  T *part = static_cast<T *>(ws);
  cudaStream_t s = as_stream(stream);
  reduce_partials<KIND, In><<<g, kRedThreads, 0, s>>>(in, n, part);
  reduce_finish<KIND, Out><<<1, 1024, 0, s>>>(part, g, out, out_value, reinterpret_cast<const float *>(in));
  return check_launch(name, 2);
}

// ------------------------------------------------------------------ row ops
enum RowOp { kSoftmax = 0, kLayerNorm = 1, kRowArgmax = 2, kRowSum = 3 };

struct RowArgs {
  const float *in;
  float *out;
  float *out_lo;  // when set, out / out_lo receive the exact tf32 split (hi, lo) of the result
  int32_t *idx;
  const float *gamma, *beta;
  uint32_t rows, cols;
  float eps;
  int *err = nullptr;  // device error word of the bounded waits (TMA-staged kernel)
};

__device__ __forceinline__ float tf32_hi(float x) {
  uint32_t h;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
  return __uint_as_float(h);
}

// Stores four results of row `row`, float4 index c: plain, or split into
// hi/lo for a consumer on the tensor cores.
__device__ __forceinline__ void row_store4(const RowArgs &a, uint32_t row, uint32_t c, float4 o) {
  float4 *dst = reinterpret_cast<float4 *>(a.out + size_t(row) * a.cols);
  if (!a.out_lo) {
    __stcs(dst + c, o);
    return;
  }
  float4 h = make_float4(tf32_hi(o.x), tf32_hi(o.y), tf32_hi(o.z), tf32_hi(o.w));
  float4 l = make_float4(__fsub_rn(o.x, h.x), __fsub_rn(o.y, h.y), __fsub_rn(o.z, h.z), __fsub_rn(o.w, h.w));
  __stcs(dst + c, h);
  __stcs(reinterpret_cast<float4 *>(a.out_lo + size_t(row) * a.cols) + c, l);
}

__device__ __forceinline__ void row_store1(const RowArgs &a, size_t i, float o) {
  if (!a.out_lo) {
    a.out[i] = o;
    return;
  }
  const float h = tf32_hi(o);
  a.out[i] = h;
  a.out_lo[i] = __fsub_rn(o, h);
}

// The row cached in registers: VPT float4 per thread.  WARP: one warp per
// row, 8 rows per CTA of 256 threads (short rows, shuffle-only reductions);
// otherwise one CTA of NT threads per row.
// Requires cols % 4 == 0 and 16-byte aligned rows; cols <= (WARP ? 32 : NT) * VPT * 4.
template <int OP, int NT, int VPT, bool WARP>
__global__ void __launch_bounds__(WARP ? 256 : NT) row_kernel(const RowArgs a) {
  __shared__ float sf[NT / 32];
  __shared__ unsigned long long sk[NT / 32];
  const uint32_t c4 = a.cols / 4;
  const int t = WARP ? (threadIdx.x & 31) : threadIdx.x;
  const uint32_t rows_per_cta = WARP ? 8u : 1u;
  const uint32_t row0 = WARP ? blockIdx.x * 8u + (threadIdx.x >> 5) : blockIdx.x;
  for (uint32_t row = row0; row < a.rows; row += gridDim.x * rows_per_cta) {
    const float4 *src = reinterpret_cast<const float4 *>(a.in + size_t(row) * a.cols);
    float4 v[VPT];
#pragma unroll
    for (int j = 0; j < VPT; j++) {
      const uint32_t c = t + j * NT;
      v[j] = c < c4 ? __ldcs(src + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (OP == kSoftmax) {
      float m = __int_as_float(0xff800000);
#pragma unroll
      for (int j = 0; j < VPT; j++)
        if (t + j * NT < c4) m = fmaxf(m, fmaxf(fmaxf(v[j].x, v[j].y), fmaxf(v[j].z, v[j].w)));
      m = row_reduce<NT, WARP>(m, sf, Max());
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < VPT; j++) {
        if (t + j * NT < c4) {
          v[j].x = expf(__fsub_rn(v[j].x, m));
          v[j].y = expf(__fsub_rn(v[j].y, m));
          v[j].z = expf(__fsub_rn(v[j].z, m));
          v[j].w = expf(__fsub_rn(v[j].w, m));
          s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
        }
      }
      s = row_reduce<NT, WARP>(s, sf, Add());
      const float inv = __frcp_rn(s);
#pragma unroll
      for (int j = 0; j < VPT; j++) {
        const uint32_t c = t + j * NT;
        if (c < c4)
          row_store4(a, row, c, make_float4(__fmul_rn(v[j].x, inv), __fmul_rn(v[j].y, inv),
                                            __fmul_rn(v[j].z, inv), __fmul_rn(v[j].w, inv)));
      }
    } else if (OP == kLayerNorm) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < VPT; j++) s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
      s = row_reduce<NT, WARP>(s, sf, Add());
      const float mu = __fdiv_rn(s, float(a.cols));
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < VPT; j++) {
        if (t + j * NT < c4) {
          v[j].x = __fsub_rn(v[j].x, mu);
          v[j].y = __fsub_rn(v[j].y, mu);
          v[j].z = __fsub_rn(v[j].z, mu);
          v[j].w = __fsub_rn(v[j].w, mu);
          ss += (__fmul_rn(v[j].x, v[j].x) + __fmul_rn(v[j].y, v[j].y)) +
                (__fmul_rn(v[j].z, v[j].z) + __fmul_rn(v[j].w, v[j].w));
        }
      }
      ss = row_reduce<NT, WARP>(ss, sf, Add());
      const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(a.cols)), a.eps)));
      const float4 *g4 = reinterpret_cast<const float4 *>(a.gamma);
      const float4 *b4 = reinterpret_cast<const float4 *>(a.beta);
#pragma unroll
      for (int j = 0; j < VPT; j++) {
        const uint32_t c = t + j * NT;
        if (c < c4) {
          const float4 g = __ldg(g4 + c), b = __ldg(b4 + c);
          float4 o;
          o.x = __fadd_rn(__fmul_rn(__fmul_rn(v[j].x, inv), g.x), b.x);
          o.y = __fadd_rn(__fmul_rn(__fmul_rn(v[j].y, inv), g.y), b.y);
          o.z = __fadd_rn(__fmul_rn(__fmul_rn(v[j].z, inv), g.z), b.z);
          o.w = __fadd_rn(__fmul_rn(__fmul_rn(v[j].w, inv), g.w), b.w);
          row_store4(a, row, c, o);
        }
      }
    } else if (OP == kRowSum) {
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < VPT; j++) sum += (v[j].x + v[j].y) + (v[j].z + v[j].w);
      sum = row_reduce<NT, WARP>(sum, sf, Add());
      if (t == 0) a.out[row] = sum;
    } else {  // argmax: each thread scans its elements in increasing index
      // order with the reference's rule (running max starts at FLT_MIN,
      // strict '>'), then one 64-bit key per thread settles value and index.
      float bv = FLT_MIN;
      int32_t bi = -1;
#pragma unroll
      for (int j = 0; j < VPT; j++) {
        const uint32_t c = t + j * NT;
        if (c < c4) {
          const int32_t base = int32_t(c * 4);
          if (v[j].x > bv) { bv = v[j].x; bi = base; }
          if (v[j].y > bv) { bv = v[j].y; bi = base + 1; }
          if (v[j].z > bv) { bv = v[j].z; bi = base + 2; }
          if (v[j].w > bv) { bv = v[j].w; bi = base + 3; }
        }
      }
      unsigned long long best = bi >= 0 ? amax_key(bv, uint32_t(bi)) : 0ull;
      best = row_reduce<NT, WARP>(best, sk, Max());
      if (t == 0) a.idx[row] = best ? int32_t(0xFFFFFFFFu - uint32_t(best & 0xFFFFFFFFu)) : 0;
    }
  }
}

// Long rows from shared memory: a cluster of CL CTAs per row (CL = 1: one
// CTA), each CTA's column part brought in by one bulk copy (completing on an
// mbarrier) and read from shared memory in every pass, so a CTA needs few
// registers and an SM holds as many rows in flight as its shared memory
// fits.  Softmax keeps exp(x - max) in place for the final scaling.
template <int OP, int CL, int NT>
__global__ void __launch_bounds__(NT) row_smem_kernel(const RowArgs a) {
  extern __shared__ __align__(128) float4 rs[];  // cols / CL floats
  __shared__ __align__(8) uint64_t full;
  namespace cg = cooperative_groups;
  __shared__ float sf[NT / 32];
  __shared__ unsigned long long sk[NT / 32];
  __shared__ float xf[2][CL];                 // slot, source rank
  __shared__ unsigned long long xk[CL];
  const int t = threadIdx.x;
  uint32_t rank = 0;
  if constexpr (CL > 1) rank = cg::this_cluster().block_rank();
  const uint32_t row = blockIdx.x / CL;
  const uint32_t part = a.cols / 4 / CL;  // float4 per CTA
  const uint32_t c0 = rank * part;
  const uint32_t bar = tc::smem_u32(&full);
  if (t == 0) {
    tc::mbar_init(bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tc::mbar_expect_tx(bar, part * 16);
    const float *src = a.in + size_t(row) * a.cols + size_t(c0) * 4;
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     tc::smem_u32(rs)),
                 "l"(src), "r"(part * 16), "r"(bar)
                 : "memory");
  }
  // Cluster peers must have started before anyone writes into their shared
  // memory: arrive now, wait just before the first exchange.
  if constexpr (CL > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  __syncthreads();
  // A failed wait (error word set) computes on whatever is in shared memory
  // and the copy may still land later: after SILCU_TIMEOUT the outputs are
  // undefined and the caller must treat the device as failed (the host reads
  // the status).  Every thread waits, so none reads early.
  tc::mbar_wait(bar, 0, a.err, 41);
  bool started = false;
  // Cluster exchange, push form: every CTA writes its partial into slot
  // [slot][rank] of every CTA of the cluster, one cluster barrier, then each
  // combines its local copies in rank order (the same result everywhere).
  // No CTA reads another's shared memory, so none has to wait for its peers
  // before leaving; each slot is written once per CTA.
  auto cl_combine = [&](float x, int slot, bool is_max) {
    if constexpr (CL > 1) {
      cg::cluster_group cl = cg::this_cluster();
      if (!started) asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
      started = true;
      if (t < CL) *cl.map_shared_rank(&xf[slot][rank], uint32_t(t)) = x;
      cl.sync();
      float r = is_max ? __int_as_float(0xff800000) : 0.f;
#pragma unroll
      for (int q = 0; q < CL; q++) r = is_max ? fmaxf(r, xf[slot][q]) : r + xf[slot][q];
      return r;
    }
    return x;
  };
  if (OP == kSoftmax) {
    float m = __int_as_float(0xff800000);
    for (uint32_t c = t; c < part; c += NT) {
      const float4 v = rs[c];
      m = fmaxf(m, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
    }
    m = cl_combine(block_reduce<NT>(m, sf, Max()), 0, true);
    float s = 0.f;
    for (uint32_t c = t; c < part; c += NT) {
      float4 v = rs[c];
      v.x = expf(__fsub_rn(v.x, m));
      v.y = expf(__fsub_rn(v.y, m));
      v.z = expf(__fsub_rn(v.z, m));
      v.w = expf(__fsub_rn(v.w, m));
      s += (v.x + v.y) + (v.z + v.w);
      rs[c] = v;  // this thread's own element: no barrier needed before it is read back
    }
    s = cl_combine(block_reduce<NT>(s, sf, Add()), 1, false);
    const float inv = __frcp_rn(s);
    for (uint32_t c = t; c < part; c += NT) {
      const float4 v = rs[c];
      row_store4(a, row, c0 + c,
                 make_float4(__fmul_rn(v.x, inv), __fmul_rn(v.y, inv), __fmul_rn(v.z, inv), __fmul_rn(v.w, inv)));
    }
  } else if (OP == kLayerNorm) {
    float s = 0.f;
    for (uint32_t c = t; c < part; c += NT) {
      const float4 v = rs[c];
      s += (v.x + v.y) + (v.z + v.w);
    }
    s = cl_combine(block_reduce<NT>(s, sf, Add()), 0, false);
    const float mu = __fdiv_rn(s, float(a.cols));
    float ss = 0.f;
    for (uint32_t c = t; c < part; c += NT) {
      const float4 v = rs[c];
      const float dx = __fsub_rn(v.x, mu), dy = __fsub_rn(v.y, mu), dz = __fsub_rn(v.z, mu),
                  dw = __fsub_rn(v.w, mu);
      ss += (__fmul_rn(dx, dx) + __fmul_rn(dy, dy)) + (__fmul_rn(dz, dz) + __fmul_rn(dw, dw));
    }
    ss = cl_combine(block_reduce<NT>(ss, sf, Add()), 1, false);
    const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(a.cols)), a.eps)));
    const float4 *g4 = reinterpret_cast<const float4 *>(a.gamma);
    const float4 *b4 = reinterpret_cast<const float4 *>(a.beta);
    for (uint32_t c = t; c < part; c += NT) {
      const float4 v = rs[c];
      const float4 g = __ldg(g4 + c0 + c), b = __ldg(b4 + c0 + c);
      float4 o;
      o.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.x, mu), inv), g.x), b.x);
      o.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.y, mu), inv), g.y), b.y);
      o.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.z, mu), inv), g.z), b.z);
      o.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.w, mu), inv), g.w), b.w);
      row_store4(a, row, c0 + c, o);
    }
  } else if (OP == kRowSum) {
    float s = 0.f;
    for (uint32_t c = t; c < part; c += NT) {
      const float4 v = rs[c];
      s += (v.x + v.y) + (v.z + v.w);
    }
    s = cl_combine(block_reduce<NT>(s, sf, Add()), 0, false);
    if (rank == 0 && t == 0) a.out[row] = s;
  } else {
    float bv = FLT_MIN;
    int32_t bi = -1;
    for (uint32_t c = t; c < part; c += NT) {
      const float4 v = rs[c];
      const int32_t base = int32_t((c0 + c) * 4);
      if (v.x > bv) { bv = v.x; bi = base; }
      if (v.y > bv) { bv = v.y; bi = base + 1; }
      if (v.z > bv) { bv = v.z; bi = base + 2; }
      if (v.w > bv) { bv = v.w; bi = base + 3; }
    }
    unsigned long long best = bi >= 0 ? amax_key(bv, uint32_t(bi)) : 0ull;
    best = block_reduce<NT>(best, sk, Max());
    if constexpr (CL > 1) {  // push to rank 0 only: it alone writes the index
      cg::cluster_group cl = cg::this_cluster();
      asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
      if (t == 0) *cl.map_shared_rank(&xk[rank], 0u) = best;
      cl.sync();
      if (rank == 0 && t == 0) {
#pragma unroll
        for (int q = 0; q < CL; q++) best = best > xk[q] ? best : xk[q];
      }
    }
    if (rank == 0 && t == 0) a.idx[row] = best ? int32_t(0xFFFFFFFFu - uint32_t(best & 0xFFFFFFFFu)) : 0;
  }
}

// Long rows: a cluster of CL CTAs shares one row (each holds 1/CL of it in
// registers); partial maxima / sums / argmax keys meet through distributed
// shared memory, summed in cluster-rank order on every CTA (deterministic).
// With small CTAs several rows are in flight per SM, which a single
// 1024-thread CTA per row cannot do.  Requires cols % (4 * CL) == 0.
template <int OP, int VPT, int CL, int NT>
__global__ void __launch_bounds__(NT) row_cluster_kernel(const RowArgs a) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  constexpr int kClusterCtas = CL;
  __shared__ float sf[NT / 32];
  __shared__ unsigned long long sk[NT / 32];
  __shared__ float xf[2];
  __shared__ unsigned long long xk;
  const int t = threadIdx.x;
  const uint32_t rank = cl.block_rank();
  const uint32_t row = blockIdx.x / kClusterCtas;
  const uint32_t part = a.cols / 4 / kClusterCtas;  // float4 per CTA
  const uint32_t c0 = rank * part;
  const float4 *src = reinterpret_cast<const float4 *>(a.in + size_t(row) * a.cols);
  float4 v[VPT];
#pragma unroll
  for (int j = 0; j < VPT; j++) {
    const uint32_t c = t + j * NT;
    v[j] = c < part ? __ldcs(src + c0 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  auto cl_sum = [&](float x, int slot) {
    x = block_reduce<NT>(x, sf, Add());
    if (t == 0) xf[slot] = x;
    cl.sync();
    float r = 0.f;
#pragma unroll
    for (int q = 0; q < kClusterCtas; q++) r += *cl.map_shared_rank(&xf[slot], q);
    return r;
  };
  if (OP == kSoftmax) {
    float m = __int_as_float(0xff800000);
#pragma unroll
    for (int j = 0; j < VPT; j++)
      if (t + j * NT < part) m = fmaxf(m, fmaxf(fmaxf(v[j].x, v[j].y), fmaxf(v[j].z, v[j].w)));
    m = block_reduce<NT>(m, sf, Max());
    if (t == 0) xf[0] = m;
    cl.sync();
#pragma unroll
    for (int q = 0; q < kClusterCtas; q++) m = fmaxf(m, *cl.map_shared_rank(&xf[0], q));
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; j++) {
      if (t + j * NT < part) {
        v[j].x = expf(__fsub_rn(v[j].x, m));
        v[j].y = expf(__fsub_rn(v[j].y, m));
        v[j].z = expf(__fsub_rn(v[j].z, m));
        v[j].w = expf(__fsub_rn(v[j].w, m));
        s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
      }
    }
    s = cl_sum(s, 1);
    const float inv = __frcp_rn(s);
#pragma unroll
    for (int j = 0; j < VPT; j++) {
      const uint32_t c = t + j * NT;
      if (c < part)
        row_store4(a, row, c0 + c, make_float4(__fmul_rn(v[j].x, inv), __fmul_rn(v[j].y, inv),
                                               __fmul_rn(v[j].z, inv), __fmul_rn(v[j].w, inv)));
    }
  } else if (OP == kLayerNorm) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; j++) s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    s = cl_sum(s, 0);
    const float mu = __fdiv_rn(s, float(a.cols));
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; j++) {
      if (t + j * NT < part) {
        v[j].x = __fsub_rn(v[j].x, mu);
        v[j].y = __fsub_rn(v[j].y, mu);
        v[j].z = __fsub_rn(v[j].z, mu);
        v[j].w = __fsub_rn(v[j].w, mu);
        ss += (__fmul_rn(v[j].x, v[j].x) + __fmul_rn(v[j].y, v[j].y)) +
              (__fmul_rn(v[j].z, v[j].z) + __fmul_rn(v[j].w, v[j].w));
      }
    }
    ss = cl_sum(ss, 1);
    const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(a.cols)), a.eps)));
    const float4 *g4 = reinterpret_cast<const float4 *>(a.gamma);
    const float4 *b4 = reinterpret_cast<const float4 *>(a.beta);
#pragma unroll
    for (int j = 0; j < VPT; j++) {
      const uint32_t c = t + j * NT;
      if (c < part) {
        const float4 g = __ldg(g4 + c0 + c), b = __ldg(b4 + c0 + c);
        float4 o;
        o.x = __fadd_rn(__fmul_rn(__fmul_rn(v[j].x, inv), g.x), b.x);
        o.y = __fadd_rn(__fmul_rn(__fmul_rn(v[j].y, inv), g.y), b.y);
        o.z = __fadd_rn(__fmul_rn(__fmul_rn(v[j].z, inv), g.z), b.z);
        o.w = __fadd_rn(__fmul_rn(__fmul_rn(v[j].w, inv), g.w), b.w);
        row_store4(a, row, c0 + c, o);
      }
    }
  } else if (OP == kRowSum) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; j++) s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    s = cl_sum(s, 0);
    if (rank == 0 && t == 0) a.out[row] = s;
  } else {
    float bv = FLT_MIN;
    int32_t bi = -1;
#pragma unroll
    for (int j = 0; j < VPT; j++) {
      const uint32_t c = t + j * NT;
      if (c < part) {
        const int32_t base = int32_t((c0 + c) * 4);
        if (v[j].x > bv) { bv = v[j].x; bi = base; }
        if (v[j].y > bv) { bv = v[j].y; bi = base + 1; }
        if (v[j].z > bv) { bv = v[j].z; bi = base + 2; }
        if (v[j].w > bv) { bv = v[j].w; bi = base + 3; }
      }
    }
    unsigned long long best = bi >= 0 ? amax_key(bv, uint32_t(bi)) : 0ull;
    best = block_reduce<NT>(best, sk, Max());
    if (t == 0) xk = best;
    cl.sync();
    if (rank == 0 && t == 0) {
#pragma unroll
      for (int q = 0; q < kClusterCtas; q++) {
        const unsigned long long k = *cl.map_shared_rank(&xk, q);
        best = best > k ? best : k;
      }
      a.idx[row] = best ? int32_t(0xFFFFFFFFu - uint32_t(best & 0xFFFFFFFFu)) : 0;
    }
  }
  cl.sync();  // peers may still be reading this CTA's exchange slots
}

// Generic fallback: any cols (no alignment requirement), re-reads the row
// from global memory (the second read hits L2 for rows up to a few MB).
template <int OP>
__global__ void __launch_bounds__(512) row_kernel_generic(const RowArgs a) {
  constexpr int NT = 512;
  __shared__ float sf[NT / 32];
  __shared__ unsigned long long sk[NT / 32];
  const int t = threadIdx.x;
  for (uint32_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const float *src = a.in + size_t(row) * a.cols;
    if (OP == kSoftmax) {
      float m = __int_as_float(0xff800000);
      for (uint32_t c = t; c < a.cols; c += NT) m = fmaxf(m, src[c]);
      m = block_reduce<NT>(m, sf, Max());
      float s = 0.f;
      for (uint32_t c = t; c < a.cols; c += NT) s += expf(__fsub_rn(src[c], m));
      s = block_reduce<NT>(s, sf, Add());
      const float inv = __frcp_rn(s);
      for (uint32_t c = t; c < a.cols; c += NT)
        row_store1(a, size_t(row) * a.cols + c, __fmul_rn(expf(__fsub_rn(src[c], m)), inv));
    } else if (OP == kLayerNorm) {
      float s = 0.f;
      for (uint32_t c = t; c < a.cols; c += NT) s += src[c];
      s = block_reduce<NT>(s, sf, Add());
      const float mu = __fdiv_rn(s, float(a.cols));
      float ss = 0.f;
      for (uint32_t c = t; c < a.cols; c += NT) {
        const float d = __fsub_rn(src[c], mu);
        ss += __fmul_rn(d, d);
      }
      ss = block_reduce<NT>(ss, sf, Add());
      const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(a.cols)), a.eps)));
      for (uint32_t c = t; c < a.cols; c += NT)
        row_store1(a, size_t(row) * a.cols + c,
                   __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(src[c], mu), inv), a.gamma[c]), a.beta[c]));
    } else {
      unsigned long long best = 0ull;
      for (uint32_t c = t; c < a.cols; c += NT) {
        const unsigned long long k = amax_key(src[c], c);
        best = best > k ? best : k;
      }
      best = block_reduce<NT>(best, sk, Max());
      if (t == 0) a.idx[row] = best ? int32_t(0xFFFFFFFFu - uint32_t(best & 0xFFFFFFFFu)) : 0;
    }
  }
}

template <int OP, int NT, int VPT>
void launch_row(const RowArgs &a, cudaStream_t s) {
  uint32_t g = a.rows;
  row_kernel<OP, NT, VPT, false><<<g, NT, 0, s>>>(a);
}

template <int OP, int VPT>
void launch_row_warp(const RowArgs &a, cudaStream_t s) {
  uint32_t g = (a.rows + 7) / 8;
  row_kernel<OP, 32, VPT, true><<<g, 256, 0, s>>>(a);
}

template <int OP, int VPT, int CL, int NT>
cudaError_t launch_cluster_cfg(const RowArgs &a, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.rows * CL);
  cfg.blockDim = dim3(NT);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CL;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, row_cluster_kernel<OP, VPT, CL, NT>, a);
}

// Rows of 8K-32K columns: CL CTAs of NT threads share a row, VPT float4 per
// thread (cols = 4 * VPT * NT * CL).  SILCU_ROW_LONG = 2 / 4 / 8 picks the
// cluster size (tuning; default 4).
template <int OP>
cudaError_t launch_row_cluster(const RowArgs &a, cudaStream_t s) {
  static const int cl = [] {
    const char *e = getenv("SILCU_ROW_LONG");
    const int v = e ? atoi(e) : 4;
    return (v == 2 || v == 4 || v == 8) ? v : 4;
  }();
  const bool wide = a.cols > 16384;
  if (cl == 2) return wide ? launch_cluster_cfg<OP, 8, 2, 512>(a, s) : launch_cluster_cfg<OP, 4, 2, 512>(a, s);
  if (cl == 8) return wide ? launch_cluster_cfg<OP, 8, 8, 128>(a, s) : launch_cluster_cfg<OP, 4, 8, 128>(a, s);
  return wide ? launch_cluster_cfg<OP, 8, 4, 256>(a, s) : launch_cluster_cfg<OP, 4, 4, 256>(a, s);
}

// One cluster (CTA) per row, the row part in dynamic shared memory.
template <int OP, int CL, int NT>
cudaError_t launch_smem(RowArgs a, cudaStream_t s) {
  auto kern = row_smem_kernel<OP, CL, NT>;
  a.err = device_error_ptr();
  if (!a.err) return cudaErrorUnknown;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.rows * CL);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = size_t(a.cols / CL) * 4;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CL;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

// Rows of 4K-32K columns (multiples of 64): softmax, layer_norm and argmax
// from shared memory, one CTA per row up to 8K columns and a 2-CTA cluster
// above (measured at 4096 x 8192: 0.95 / 0.87 / 0.90 of HBM against
// 0.93 / 0.79 / 0.89 with the row in registers; at 4096 x 32768
// 0.77 / 0.74 / 0.82 against 0.69 / 0.64 / 0.76; clusters of 4: 0.76 /
// 0.74 / 0.80); the row sum from registers (0.97 / 0.98 against 0.94 /
// 0.77).  SILCU_ROW_IMPL = 0 / 1 forces registers / shared memory,
// SILCU_ROW_SMEM_CL = 4 the larger cluster (tuning).
template <int OP>
cudaError_t launch_row_long(const RowArgs &a, cudaStream_t s) {
  static const int impl = [] {
    const char *e = getenv("SILCU_ROW_IMPL");
    return e ? atoi(e) : -1;
  }();
  static const int cl = [] {  // cluster size of the shared-memory kernel above 8K columns
    const char *e = getenv("SILCU_ROW_SMEM_CL");
    const int v = e ? atoi(e) : 2;
    return v == 4 ? 4 : 2;
  }();
  const bool smem = impl == 1 || (impl != 0 && OP != kRowSum);
  if (smem) {
    if (a.cols <= 8192) return launch_smem<OP, 1, 256>(a, s);
    return cl == 4 ? launch_smem<OP, 4, 256>(a, s) : launch_smem<OP, 2, 512>(a, s);
  }
  if (a.cols <= 8192) {
    launch_row<OP, 512, 4>(a, s);
    return cudaSuccess;
  }
  return launch_row_cluster<OP>(a, s);
}

template <int OP>
silcu_status run_rows(const char *name, const RowArgs &a, silcu_stream stream) {
  if (a.rows == 0 || a.cols == 0) return SILCU_OK;
  cudaStream_t s = as_stream(stream);
  const bool vec = (a.cols % 4 == 0) && aligned16(a.in) && (!a.out || aligned16(a.out) || OP == kRowSum) &&
                   (!a.out_lo || aligned16(a.out_lo)) &&
                   (OP != kLayerNorm || (aligned16(a.gamma) && aligned16(a.beta)));
  const uint32_t c = a.cols;
  if (vec && c <= 128) launch_row_warp<OP, 1>(a, s);
  else if (vec && c <= 256) launch_row_warp<OP, 2>(a, s);
  else if (vec && c <= 512) launch_row_warp<OP, 4>(a, s);
  else if (vec && c <= 1024) launch_row_warp<OP, 8>(a, s);
  else if (vec && c <= 2048) launch_row<OP, 256, 2>(a, s);
  else if (vec && c <= 4096) launch_row<OP, 256, 4>(a, s);
  else if (vec && c <= 32768 && (c % 64 == 0) && a.rows <= 0x1FFFFFFFu) {
    const cudaError_t e = launch_row_long<OP>(a, s);
    if (e != cudaSuccess) return fail(SILCU_CUDA_ERROR, "%s: launch: %s", name, cudaGetErrorString(e));
  } else if (vec && c <= 16384) launch_row<OP, 512, 8>(a, s);
  else if (vec && c <= 32768) launch_row<OP, 1024, 8>(a, s);
  else row_kernel_generic<OP><<<a.rows < 65535u * 16 ? a.rows : 65535u * 16, 512, 0, s>>>(a);
  return check_launch(name);
}

// ------------------------------------------- split-row argmax (few long rows)
__global__ void __launch_bounds__(512) argmax_split_partials(const float *__restrict__ in, uint64_t cols,
                                                             uint32_t splits, unsigned long long *part) {
  __shared__ unsigned long long sk[16];
  const uint32_t row = blockIdx.y, sp = blockIdx.x;
  const uint64_t chunk = (cols + splits - 1) / splits;
  const uint64_t c0 = sp * chunk, c1 = c0 + chunk < cols ? c0 + chunk : cols;
  const float *src = in + uint64_t(row) * cols;
  unsigned long long best = 0ull;
  for (uint64_t c = c0 + threadIdx.x; c < c1; c += 512) {
    const unsigned long long k = amax_key(__ldcs(src + c), c);
    best = best > k ? best : k;
  }
  best = block_reduce<512>(best, sk, Max());
  if (threadIdx.x == 0) part[uint64_t(row) * splits + sp] = best;
}

__global__ void argmax_split_finish(const unsigned long long *part, uint32_t rows, uint32_t splits,
                                    int32_t *out) {
  const uint32_t row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  unsigned long long best = 0ull;
  for (uint32_t s = 0; s < splits; s++) {
    const unsigned long long k = part[uint64_t(row) * splits + s];
    best = best > k ? best : k;
  }
  out[row] = best ? int32_t(0xFFFFFFFFu - uint32_t(best & 0xFFFFFFFFu)) : 0;
}

uint32_t argmax_splits(size_t rows, size_t cols) {
  const size_t target = size_t(sm_count()) * 8;
  if (rows >= target || cols < 8192) return 1;
  size_t s = (target + rows - 1) / rows;
  const size_t max_s = cols / 4096;
  if (s > max_s) s = max_s;
  if (s < 1) s = 1;
  if (s > 65535) s = 65535;
  return uint32_t(s);
}

// ------------------------------------------------------------- sum over axis
// Rows (inner == 1): one warp per row for short rows, else one CTA per row.
__global__ void __launch_bounds__(256) sum_rows_kernel(const float *__restrict__ in, float *__restrict__ out,
                                                       uint64_t rows, uint64_t cols, bool vec) {
  __shared__ float sf[8];
  for (uint64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float *src = in + row * cols;
    float s = 0.f;
    if (vec) {
      const float4 *s4 = reinterpret_cast<const float4 *>(src);
      for (uint64_t c = threadIdx.x; c < cols / 4; c += 256) {
        const float4 f = __ldcs(s4 + c);
        s += (f.x + f.y) + (f.z + f.w);
      }
    } else {
      for (uint64_t c = threadIdx.x; c < cols; c += 256) s += src[c];
    }
    s = block_reduce<256>(s, sf, Add());
    if (threadIdx.x == 0) out[row] = s;
  }
}

__global__ void __launch_bounds__(256) sum_rows_warp_kernel(const float *__restrict__ in,
                                                            float *__restrict__ out, uint64_t rows,
                                                            uint64_t cols) {
  const uint64_t warp = (uint64_t(blockIdx.x) * 256 + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float *src = in + warp * cols;
  float s = 0.f;
  for (uint64_t c = lane; c < cols; c += 32) s += src[c];
  s = warp_sum(s);
  if (lane == 0) out[warp] = s;
}

// Columns (inner > 1): thread per inner index, rows of the axis split into
// `splits` chunks whose partials land in the workspace; a second pass adds
// the chunks in order.
__global__ void __launch_bounds__(256) sum_cols_kernel(const float *__restrict__ in, float *__restrict__ dst,
                                                       uint64_t outer, uint64_t len, uint64_t inner,
                                                       uint32_t splits) {
  const uint64_t i = uint64_t(blockIdx.x) * 256 + threadIdx.x;
  const uint64_t o = blockIdx.y;
  const uint32_t sp = blockIdx.z;
  if (i >= inner) return;
  const uint64_t chunk = (len + splits - 1) / splits;
  const uint64_t k0 = sp * chunk, k1 = k0 + chunk < len ? k0 + chunk : len;
  const float *src = in + o * len * inner + i;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  uint64_t k = k0;
  for (; k + 4 <= k1; k += 4) {
    s0 += __ldcs(src + (k + 0) * inner);
    s1 += __ldcs(src + (k + 1) * inner);
    s2 += __ldcs(src + (k + 2) * inner);
    s3 += __ldcs(src + (k + 3) * inner);
  }
  for (; k < k1; k++) s0 += __ldcs(src + k * inner);
  dst[(uint64_t(sp) * outer + o) * inner + i] = (s0 + s1) + (s2 + s3);
}

__global__ void __launch_bounds__(256) sum_cols_finish(const float *__restrict__ part, float *__restrict__ out,
                                                       uint64_t total, uint32_t splits) {
  const uint64_t j = uint64_t(blockIdx.x) * 256 + threadIdx.x;
  if (j >= total) return;
  float s = 0.f;
  for (uint32_t sp = 0; sp < splits; sp++) s += part[uint64_t(sp) * total + j];
  out[j] = s;
}

uint32_t col_splits(size_t outer, size_t len, size_t inner) {
  const size_t blocks = ((inner + 255) / 256) * outer;
  const size_t target = size_t(sm_count()) * 8;
  if (blocks >= target) return 1;
  size_t s = (target + blocks - 1) / blocks;
  const size_t max_s = len / 16 > 0 ? len / 16 : 1;
  if (s > max_s) s = max_s;
  if (s > 65535) s = 65535;
  return uint32_t(s < 1 ? 1 : s);
}

}  // namespace
}  // namespace silcu

using namespace silcu;

extern "C" {

size_t silcu_reduce_workspace_bytes(size_t n) {
  (void)n;
  return size_t(kMaxPartials) * 8;
}

silcu_status silcu_sum_f32(const float *in, size_t n, float *out, void *ws, size_t wsb, silcu_stream s) {
  if (in && out && n > 0 && n <= size_t(kSeqSumMax)) {
    sum_seq_small<<<1, 256, 0, as_stream(s)>>>(in, int(n), out);
    return check_launch("sum_f32");
  }
  return run_reduce<kSum, float, float>("sum_f32", in, n, out, nullptr, ws, wsb, s);
}
silcu_status silcu_min_f32(const float *in, size_t n, float *out, void *ws, size_t wsb, silcu_stream s) {
  return run_reduce<kMinK, float, float>("min_f32", in, n, out, nullptr, ws, wsb, s);
}
silcu_status silcu_max_f32(const float *in, size_t n, float *out, void *ws, size_t wsb, silcu_stream s) {
  return run_reduce<kMaxK, float, float>("max_f32", in, n, out, nullptr, ws, wsb, s);
}
silcu_status silcu_sum_i32(const int32_t *in, size_t n, int32_t *out, void *ws, size_t wsb, silcu_stream s) {
  return run_reduce<kSumI, int32_t, int32_t>("sum_i32", in, n, out, nullptr, ws, wsb, s);
}
silcu_status silcu_argmax_all_f32(const float *in, size_t n, int64_t *out_index, float *out_value, void *ws,
                                  size_t wsb, silcu_stream s) {
  return run_reduce<kArgmax, float, int64_t>("argmax_all_f32", in, n, out_index, out_value, ws, wsb, s);
}

silcu_status silcu_softmax_f32(const float *in, float *out, size_t rows, size_t cols, silcu_stream s) {
  if (rows && cols && (!in || !out)) return fail(SILCU_INVALID_ARGUMENT, "softmax: null pointer");
  if (rows > 0xFFFFFFFFull || cols > 0xFFFFFFFFull) return fail(SILCU_UNSUPPORTED, "softmax: dims >= 2^32");
  RowArgs a{in, out, nullptr, nullptr, nullptr, nullptr, uint32_t(rows), uint32_t(cols), 0.f};
  return run_rows<kSoftmax>("softmax", a, s);
}

silcu_status silcu_layer_norm_f32(const float *in, float *out, const float *gamma, const float *beta,
                                  size_t rows, size_t cols, float eps, silcu_stream s) {
  if (rows && cols && (!in || !out || !gamma || !beta))
    return fail(SILCU_INVALID_ARGUMENT, "layer_norm: null pointer");
  if (rows > 0xFFFFFFFFull || cols > 0xFFFFFFFFull) return fail(SILCU_UNSUPPORTED, "layer_norm: dims >= 2^32");
  RowArgs a{in, out, nullptr, nullptr, gamma, beta, uint32_t(rows), uint32_t(cols), eps};
  return run_rows<kLayerNorm>("layer_norm", a, s);
}

silcu_status silcu_softmax_split_f32(const float *in, float *out_hi, float *out_lo, size_t rows, size_t cols,
                                     silcu_stream s) {
  if (rows && cols && (!in || !out_hi || !out_lo)) return fail(SILCU_INVALID_ARGUMENT, "softmax_split: null pointer");
  if (rows > 0xFFFFFFFFull || cols > 0xFFFFFFFFull) return fail(SILCU_UNSUPPORTED, "softmax_split: dims >= 2^32");
  RowArgs a{in, out_hi, out_lo, nullptr, nullptr, nullptr, uint32_t(rows), uint32_t(cols), 0.f};
  return run_rows<kSoftmax>("softmax_split", a, s);
}

silcu_status silcu_layer_norm_split_f32(const float *in, float *out_hi, float *out_lo, const float *gamma,
                                        const float *beta, size_t rows, size_t cols, float eps, silcu_stream s) {
  if (rows && cols && (!in || !out_hi || !out_lo || !gamma || !beta))
    return fail(SILCU_INVALID_ARGUMENT, "layer_norm_split: null pointer");
  if (rows > 0xFFFFFFFFull || cols > 0xFFFFFFFFull) return fail(SILCU_UNSUPPORTED, "layer_norm_split: dims >= 2^32");
  RowArgs a{in, out_hi, out_lo, nullptr, gamma, beta, uint32_t(rows), uint32_t(cols), eps};
  return run_rows<kLayerNorm>("layer_norm_split", a, s);
}

size_t silcu_argmax_workspace_bytes(size_t rows, size_t cols) {
  const uint32_t sp = argmax_splits(rows, cols);
  return sp > 1 ? rows * sp * sizeof(unsigned long long) : 0;
}

silcu_status silcu_argmax_f32(const float *in, int32_t *out, size_t rows, size_t cols, void *ws, size_t wsb,
                              silcu_stream stream) {
  if (rows == 0) return SILCU_OK;
  if (!in || !out) return fail(SILCU_INVALID_ARGUMENT, "argmax: null pointer");
  if (cols == 0) return fail(SILCU_INVALID_ARGUMENT, "argmax: empty rows");
  if (rows > 65535u || cols > 0xFFFFFFFFull) {
    if (rows > 0xFFFFFFFFull || cols > 0xFFFFFFFFull) return fail(SILCU_UNSUPPORTED, "argmax: dims >= 2^32");
  }
  const uint32_t sp = argmax_splits(rows, cols);
  if (sp > 1) {
    const size_t need = rows * sp * sizeof(unsigned long long);
    if (!ws || wsb < need) return fail(SILCU_WORKSPACE_TOO_SMALL, "argmax: workspace %zu < %zu", wsb, need);
    cudaStream_t s = as_stream(stream);
    argmax_split_partials<<<dim3(sp, uint32_t(rows)), 512, 0, s>>>(in, cols, sp,
                                                                   static_cast<unsigned long long *>(ws));
    argmax_split_finish<<<uint32_t((rows + 255) / 256), 256, 0, s>>>(
        static_cast<const unsigned long long *>(ws), uint32_t(rows), sp, out);
    return check_launch("argmax(split)", 2);
  }
  RowArgs a{in, nullptr, nullptr, out, nullptr, nullptr, uint32_t(rows), uint32_t(cols), 0.f};
  return run_rows<kRowArgmax>("argmax", a, stream);
}

size_t silcu_sum_axis_workspace_bytes(size_t outer, size_t len, size_t inner) {
  if (inner == 1) return 0;
  const uint32_t sp = col_splits(outer, len, inner);
  return sp > 1 ? size_t(sp) * outer * inner * sizeof(float) : 0;
}

// Sum over an axis in the reference CPU loop's order (include/array.h:
// 2303-2317: every output accumulates its inputs sequentially in fp32, in
// increasing index along the axis): one thread per output, so the result is
// bit-identical to the reference.  Outputs along `inner` are consecutive
// threads (coalesced loads); with inner == 1 a thread walks its contiguous
// row with 16-byte loads, four sequential adds each.
__global__ void __launch_bounds__(128) sum_axis_seq_kernel(const float *__restrict__ in, float *__restrict__ out,
                                                          uint64_t outer, uint64_t len, uint64_t inner, int vec) {
  const uint64_t total = outer * inner;
  for (uint64_t g = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += uint64_t(gridDim.x) * blockDim.x) {
    const uint64_t o = g / inner, i = g - o * inner;
    const float *p = in + o * len * inner + i;
    float s = 0.0f;
    if (vec) {  // inner == 1, len % 4 == 0, 16-byte aligned rows
      // 16 loads in flight per thread (one thread per row leaves few threads
      // to hide memory latency with), then their 64 adds in order.
      const float4 *p4 = reinterpret_cast<const float4 *>(p);
      const uint64_t n4 = len / 4;
      uint64_t k = 0;
      for (; k + 16 <= n4; k += 16) {
        float4 v[16];
#pragma unroll
        for (int u = 0; u < 16; u++) v[u] = __ldg(p4 + k + u);
#pragma unroll
        for (int u = 0; u < 16; u++) s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v[u].x), v[u].y), v[u].z), v[u].w);
      }
      for (; k < n4; k++) {
        const float4 v = __ldg(p4 + k);
        s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v.x), v.y), v.z), v.w);
      }
    } else {
      for (uint64_t k = 0; k < len; k++) s = __fadd_rn(s, __ldg(p + k * inner));
    }
    out[g] = s;
  }
}

// Rows (inner == 1, len % 4 == 0, 16-byte aligned): one warp per 32 rows,
// lane r adding row r in column order -- the sequential sum, bit for bit --
// from shared memory, where the warp stages 32 x 32 tiles with coalesced
// 16-byte cp.async copies (4 rows x 128 B per instruction) through an
// 8-stage ring, so the loads of later tiles are in flight while the adds of
// the current one run (16 stages, 72 KB: one warp per SM streams a row
// block, so the ring depth sets the bytes in flight).  Rows padded to 36
// floats (16-byte aligned copies).
constexpr int kSeqTile = 32, kSeqStages = 16, kSeqPad = kSeqTile + 4;
constexpr int kSeqSmem = kSeqStages * 32 * kSeqPad * 4;

__global__ void __launch_bounds__(32) sum_rows_seq_kernel(const float *__restrict__ in, float *__restrict__ out,
                                                          uint64_t rows, uint64_t len) {
  extern __shared__ __align__(16) float seq_smem[];
  float(*buf)[32][kSeqPad] = reinterpret_cast<float(*)[32][kSeqPad]>(seq_smem);
  const int lane = threadIdx.x;
  const uint64_t r0 = uint64_t(blockIdx.x) * 32;
  const uint64_t ntiles = (len + kSeqTile - 1) / kSeqTile;
  auto issue = [&](uint64_t t) {
    if (t < ntiles) {
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const int row = i * 4 + (lane >> 3), chunk = lane & 7;
        const uint64_t col = t * kSeqTile + uint64_t(chunk) * 4;
        if (r0 + row < rows && col < len) {
          const float *src = in + (r0 + row) * len + col;
          const uint32_t dst = uint32_t(__cvta_generic_to_shared(&buf[t % kSeqStages][row][chunk * 4]));
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
        }
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
#pragma unroll 1
  for (int t = 0; t < kSeqStages - 1; t++) issue(uint64_t(t));
  float s = 0.0f;
#pragma unroll 1
  for (uint64_t t = 0; t < ntiles; t++) {
    asm volatile("cp.async.wait_group %0;" ::"n"(kSeqStages - 2) : "memory");
    __syncwarp();
    const float *row = buf[t % kSeqStages][lane];
    const uint64_t n = len - t * kSeqTile < uint64_t(kSeqTile) ? len - t * kSeqTile : uint64_t(kSeqTile);
    if (n == kSeqTile) {
#pragma unroll
      for (int c = 0; c < kSeqTile; c++) s = __fadd_rn(s, row[c]);
    } else {
      for (uint64_t c = 0; c < n; c++) s = __fadd_rn(s, row[c]);
    }
    __syncwarp();  // every lane is done with this stage before it is refilled
    issue(t + kSeqStages - 1);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  if (r0 + lane < rows) out[r0 + lane] = s;
}

silcu_status silcu_sum_axis_seq_f32(const float *in, float *out, size_t outer, size_t len, size_t inner,
                                    silcu_stream stream) {
  const size_t total = outer * inner;
  if (total == 0) return SILCU_OK;
  if (!in || !out) return fail(SILCU_INVALID_ARGUMENT, "sum_axis_seq: null pointer");
  const int vec = inner == 1 && len % 4 == 0 && aligned16(in) ? 1 : 0;
  if (vec && len > 0 && (outer + 31) / 32 <= 0x7FFFFFFFull) {
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
      cudaError_t e = cudaFuncSetAttribute(sum_rows_seq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSeqSmem);
      if (e != cudaSuccess) return fail(SILCU_CUDA_ERROR, "sum_axis_seq: smem attribute: %s", cudaGetErrorString(e));
      configured[dev] = true;
    }
    sum_rows_seq_kernel<<<unsigned((outer + 31) / 32), 32, kSeqSmem, as_stream(stream)>>>(in, out, outer, len);
    return check_launch("sum_axis_seq");
  }
  uint64_t grid = (total + 127) / 128;
  const uint64_t cap = uint64_t(sm_count()) * 16;
  if (grid > cap) grid = cap;
  sum_axis_seq_kernel<<<unsigned(grid), 128, 0, as_stream(stream)>>>(in, out, outer, len, inner, vec);
  return check_launch("sum_axis_seq");
}

silcu_status silcu_sum_axis_f32(const float *in, float *out, size_t outer, size_t len, size_t inner, void *ws,
                                size_t wsb, silcu_stream stream) {
  const size_t total = outer * inner;
  if (total == 0) return SILCU_OK;
  if (!in || !out) return fail(SILCU_INVALID_ARGUMENT, "sum_axis: null pointer");
  cudaStream_t s = as_stream(stream);
  if (len == 0) {
    cudaError_t e = cudaMemsetAsync(out, 0, total * sizeof(float), s);
    return e == cudaSuccess ? SILCU_OK : fail(SILCU_CUDA_ERROR, "sum_axis: %s", cudaGetErrorString(e));
  }
  if (inner == 1 && len % 4 == 0 && len <= 32768 && outer <= 0xFFFFFFFFull && aligned16(in)) {
    RowArgs a{in, out, nullptr, nullptr, nullptr, nullptr, uint32_t(outer), uint32_t(len), 0.f};
    return run_rows<kRowSum>("sum_axis(rows)", a, stream);
  }
  if (inner == 1) {
    if (len <= 256) {
      const uint64_t blocks = (outer * 32 + 255) / 256;
      sum_rows_warp_kernel<<<uint32_t(blocks), 256, 0, s>>>(in, out, outer, len);
    } else {
      const bool vec = (len % 4 == 0) && aligned16(in);
      const uint64_t g = outer < 65535ull * 32 ? outer : 65535ull * 32;
      sum_rows_kernel<<<uint32_t(g), 256, 0, s>>>(in, out, outer, len, vec);
    }
    return check_launch("sum_axis(rows)");
  }
  if (outer > 65535) return fail(SILCU_UNSUPPORTED, "sum_axis: outer extent > 65535");
  const uint32_t sp = col_splits(outer, len, inner);
  dim3 grid(uint32_t((inner + 255) / 256), uint32_t(outer), sp);
  if (sp == 1) {
    sum_cols_kernel<<<grid, 256, 0, s>>>(in, out, outer, len, inner, 1);
  } else {
    const size_t need = size_t(sp) * total * sizeof(float);
    if (!ws || wsb < need) return fail(SILCU_WORKSPACE_TOO_SMALL, "sum_axis: workspace %zu < %zu", wsb, need);
    float *part = static_cast<float *>(ws);
    sum_cols_kernel<<<grid, 256, 0, s>>>(in, part, outer, len, inner, sp);
    sum_cols_finish<<<uint32_t((total + 255) / 256), 256, 0, s>>>(part, out, total, sp);
    return check_launch("sum_axis(cols)", 2);
  }
  return check_launch("sum_axis(cols)");
}

}  // extern "C"

// ------------------------------------------------ allocation-free whole sum
// For callers that may not allocate device memory themselves: code running
// inside a host application's custom allocator or memory-pool callback, or a
// plugin whose host forbids cudaMalloc after start-up.  The scratch for the
// first pass lives in a fixed array compiled into this library instead of a
// caller-provided workspace.
namespace silcu {
namespace {

// One fp64 partial per CTA of the first pass: 4096 x 8 B = 32 KiB, held on
// every GPU that loads this library until the process exits.
constexpr int kNoAllocPartials = 4096;
static __device__ __align__(256) double g_noalloc_partials[kNoAllocPartials];
static_assert(kNoAllocPartials >= kMaxPartials, "the first pass never needs more partials than the scratch holds");

// Host code must not pass the symbol itself to a kernel (on the host it is a
// stand-in, not a device address); look the address up once per device.
// The cached address belongs to the device's current context: it does not
// survive a cudaDeviceReset.  Two host threads making their first call at
// once both look it up and store the same value (atomic stores).
double *noalloc_partials(silcu_status *st) {
  static std::atomic<double *> cached[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    *st = fail(SILCU_CUDA_ERROR, "sum_f32_noalloc: no current device");
    return nullptr;
  }
  double *have = cached[dev].load(std::memory_order_acquire);
  if (!have) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_partials);
    if (e != cudaSuccess) {
      *st = fail(SILCU_CUDA_ERROR, "sum_f32_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return nullptr;
    }
    have = static_cast<double *>(p);
    cached[dev].store(have, std::memory_order_release);
  }
  *st = SILCU_OK;
  return have;
}

}  // namespace
}  // namespace silcu

extern "C" silcu_status silcu_sum_f32_noalloc(const float *in, size_t n, float *out, silcu_stream stream) {
  if (!in || !out) return fail(SILCU_INVALID_ARGUMENT, "sum_f32_noalloc: null pointer");
  if (n == 0) return fail(SILCU_INVALID_ARGUMENT, "sum_f32_noalloc: empty input");
  if (n <= size_t(kSeqSumMax)) {  // same small-sum rule as silcu_sum_f32; no scratch needed
    sum_seq_small<<<1, 256, 0, as_stream(stream)>>>(in, int(n), out);
    return check_launch("sum_f32_noalloc");
  }
  const int g = red_grid(n);  // at most kMaxPartials <= kNoAllocPartials (static_assert above)
  silcu_status st;
  double *part = noalloc_partials(&st);
  if (!part) return st;
  // Every CTA of the first pass overwrites its own partial before the finish
  // kernel reads it, so nothing left over from an earlier call is read.
  cudaStream_t s = as_stream(stream);
  reduce_partials<kSum, float><<<g, kRedThreads, 0, s>>>(in, n, part);
  reduce_finish<kSum, float><<<1, 1024, 0, s>>>(part, g, out, nullptr, in);
  return check_launch("sum_f32_noalloc", 2);
}

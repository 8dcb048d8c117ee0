// fp32-faithful SGEMM on the 5th-generation tensor cores (sm_100a).
//
// Split precision (3xTF32, Ootomo & Yokota 2022, "Recovering single precision
// accuracy from Tensor Cores while surpassing the FP32 theoretical peak
// performance"): x = hi + lo with hi = tf32_rna(x), lo = x - hi (exact in
// fp32), and  A.B ~= Ah.Bh + Ah.Bl + Al.Bh  accumulated in fp32 in TMEM.
//
// Pipeline (persistent: one CTA per SM walks 128x128 output tiles):
//   pack_split  (pre-pass) writes hi/lo copies of A and B, K-major, K padded
//               to a multiple of 32, one pass over each operand;
//   warp 0      TMA producer: 4 boxes of 128 rows x 32 fp32 (128 B, 128-byte
//               swizzle) per K block into a 3-stage shared-memory ring;
//   warp 1      allocates all 512 TMEM columns (4 accumulator buffers of 128),
//               one thread issues tcgen05.mma.kind::tf32 (M=128, N=128, K=8)
//               x 3 per K step and tcgen05.commit to release ring slots and to
//               hand each finished chunk of CHUNK_KB K blocks to the epilogue;
//   warps 2-5   drain each chunk with tcgen05.ld into fp32 registers (round to
//               nearest), and at the end of a tile stage 32x32 blocks through
//               shared memory so that the alpha / bias / activation / residual
//               epilogue and the stores are coalesced 128-byte row segments.
// No TMA multicast and no clusters: each CTA loads its own tiles.
// Every mbarrier wait is bounded (wall-clock limit via %globaltimer); on
// expiry it records an error in the device error word and the CTA unwinds,
// frees its TMEM and exits.
#include <cuda.h>
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "gemm_internal.cuh"

namespace silcu {
namespace {

constexpr int BM = 128, BK = 32;
constexpr int STAGE_PITCH = 33;  // floats per staged output row (bank-conflict free)

// Per-variant constants: BN = 128 (3-stage ring, 4 TMEM chunk buffers, 4
// epilogue warps) or BN = 256 (2-stage ring, 2 chunk buffers, 8 epilogue
// warps, each owning 128 columns).  The wider tile halves the shared-memory
// operand traffic per FLOP of A, which bounds the 128-wide variant.
template <int BN_>
struct Cfg {
  static constexpr int BN = BN_;
  static constexpr int TILE_A = BM * BK * 4;
  static constexpr int TILE_B = BN * BK * 4;
  static constexpr int STAGE_BYTES = 2 * TILE_A + 2 * TILE_B;  // Ahi, Alo, Bhi, Blo
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int EPI_WARPS = BN / 32;
  static constexpr int OUT_STAGE_BYTES = EPI_WARPS * 32 * STAGE_PITCH * 4;
  static constexpr int SMEM_BYTES = RING_BYTES + OUT_STAGE_BYTES + 1024 + 256;
  static constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int NBUF = 512 / BN;  // TMEM accumulator buffers (chunks in flight)
  static constexpr uint32_t TMEM_COLS = 512;
  // Instruction descriptor: D fp32, A/B tf32, both K-major, N = BN, M = BM.
  static constexpr uint32_t IDESC =
      (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};
constexpr int CHUNK_KB_DEFAULT = 4;      // K blocks per TMEM accumulation chunk
constexpr int GROUP_M = 8;
constexpr unsigned long long WAIT_NS = 2000000000ull;  // 2 s per wait

struct TcEpi {
  float alpha;
  const float *bias;
  int64_t bias_len;
  int act;
  const float *residual;
  int64_t ldr;
};

struct __align__(64) TcParams {
  CUtensorMap a_hi, a_lo, b_hi, b_lo;  // 3-D {Kp, rows, batch}
  float *C;
  int64_t ldc, stride_c, bin, stride_c_in;
  int M, N, Kp, tiles_m, tiles_n, nbatch, chunk_kb;
  TcEpi epi;
  int *err;
};

// ----------------------------------------------------------------- PTX glue
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait.  Returns false (and records `code`) when the phase does not
// complete within WAIT_NS, or when another CTA already recorded an error.
__device__ __noinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int *err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 1;; i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*reinterpret_cast<volatile int *>(err) != 0) return false;
      if (globaltimer() - t0 > WAIT_NS) {
        atomicCAS(err, 0, code);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor, K-major operand with 128-byte swizzle:
// 8-row x 128-byte swizzle atoms stacked along M/N every 1024 bytes (SBO);
// LBO is unused for this layout (encoded as 1); version 1 (sm_100).
__device__ __forceinline__ uint64_t make_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= uint64_t((addr & 0x3FFFFu) >> 4);
  d |= uint64_t(1) << 16;
  d |= uint64_t(1024 >> 4) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float epi_apply(const TcEpi &e, float acc, int64_t row, int64_t col,
                                           const float *res) {
  float v = acc;
  if (e.alpha != 1.0f) v = __fmul_rn(v, e.alpha);
  if (e.bias) v = __fadd_rn(v, __ldg(e.bias + (col % e.bias_len)));
  if (e.act == SILCU_ACT_RELU) v = v >= 0.0f ? v : 0.0f;
  else if (e.act == SILCU_ACT_SIGMOID) v = sigmoid_ref(v);
  if (res) v = __fadd_rn(v, __ldg(res + row * e.ldr + col));
  return v;
}

// ------------------------------------------------------------------- kernel
// Accumulation is split in two levels (the remedy of Ootomo & Yokota for the
// tensor core's truncating fp32 accumulation): the MMAs of CHUNK_KB K blocks
// accumulate into one of two TMEM buffers; the epilogue warps drain each
// finished chunk into fp32 registers with round-to-nearest adds while the
// MMAs continue in the other buffer.
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

struct Tile {
  int bz, m0, n0;
};

// Grouped raster inside one batch: GROUP_M tile-rows sweep the N tiles
// together so the A and B strips they share stay in L2.
template <int BN>
__device__ __forceinline__ Tile decode_tile(const TcParams &p, int idx) {
  const int tiles_per_batch = p.tiles_m * p.tiles_n;
  Tile r;
  r.bz = idx / tiles_per_batch;
  const int t = idx % tiles_per_batch;
  const int group = t / (GROUP_M * p.tiles_n);
  const int first_m = group * GROUP_M;
  const int gm = min(p.tiles_m - first_m, GROUP_M);
  const int tm = first_m + (t % (GROUP_M * p.tiles_n)) % gm;
  const int tn = (t % (GROUP_M * p.tiles_n)) / gm;
  r.m0 = tm * BM;
  r.n0 = tn * BN;
  return r;
}

// Persistent: CTA i takes tiles i, i + gridDim.x, ...  The TMA ring, the MMA
// chunk buffers and the epilogue run as one continuous stream across tiles,
// so a tile's pipeline fill and its output store overlap its neighbours'.
template <int BN_>
__global__ void __launch_bounds__(Cfg<BN_>::NUM_THREADS, 1) tc_gemm_kernel(const __grid_constant__ TcParams p) {
  using C = Cfg<BN_>;
  constexpr int BN = C::BN, STAGES = C::STAGES, NBUF = C::NBUF, RING_BYTES = C::RING_BYTES;
  constexpr int STAGE_BYTES = C::STAGE_BYTES, TILE_A = C::TILE_A, TILE_B = C::TILE_B;
  constexpr uint32_t TMEM_COLS = C::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float *ostage = reinterpret_cast<float *>(smem + RING_BYTES);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + RING_BYTES + C::OUT_STAGE_BYTES);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 2 * NBUF);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
  const uint32_t tfull0 = smem_u32(bars + 2 * STAGES), tempty0 = smem_u32(bars + 2 * STAGES + NBUF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_tiles = p.tiles_m * p.tiles_n * p.nbatch;
  const int nk = p.Kp / BK;
  const int CHUNK_KB = p.chunk_kb;
  const int nchunks = (nk + CHUNK_KB - 1) / CHUNK_KB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int j = 0; j < NBUF; j++) {
      mbar_init(tfull0 + 8 * j, 1);
      mbar_init(tempty0 + 8 * j, C::EPI_WARPS);  // one arrive per epilogue warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t kbg = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        const Tile tl = decode_tile<BN>(p, tile);
        for (int kb = 0; kb < nk; kb++, kbg++) {
          const uint32_t s = kbg % STAGES;
          const uint32_t ph = (kbg / STAGES) & 1;
          if (kbg >= STAGES && !mbar_wait(empty0 + 8 * s, ph ^ 1, p.err, 1)) { ok = false; break; }
          const uint32_t full = full0 + 8 * s;
          mbar_expect_tx(full, STAGE_BYTES);
          const uint32_t dst = smem_u32(smem + s * STAGE_BYTES);
          const int kc = kb * BK;
          tma_load_3d(dst, &p.a_hi, full, kc, tl.m0, tl.bz);
          tma_load_3d(dst + TILE_A, &p.a_lo, full, kc, tl.m0, tl.bz);
          tma_load_3d(dst + 2 * TILE_A, &p.b_hi, full, kc, tl.n0, tl.bz);
          tma_load_3d(dst + 2 * TILE_A + TILE_B, &p.b_lo, full, kc, tl.n0, tl.bz);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t kbg = 0, cg = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        for (int c = 0; c < nchunks && ok; c++, cg++) {
          const uint32_t j = cg % NBUF, use = cg / NBUF;
          if (cg >= NBUF && !mbar_wait(tempty0 + 8 * j, (use & 1) ^ 1, p.err, 4)) { ok = false; break; }
          tc_fence_after();
          const uint32_t dacc = tmem + j * BN;
          const int kb1 = min(nk, (c + 1) * CHUNK_KB);
          for (int kb = c * CHUNK_KB; kb < kb1; kb++, kbg++) {
            const uint32_t s = kbg % STAGES;
            const uint32_t ph = (kbg / STAGES) & 1;
            if (!mbar_wait(full0 + 8 * s, ph, p.err, 2)) { ok = false; break; }
            tc_fence_after();
            const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
#pragma unroll
            for (int kk = 0; kk < BK / 8; kk++) {
              const uint32_t off = kk * 32;  // 8 tf32 = 32 bytes along K inside the swizzle atom
              const uint64_t ah = make_desc(base + off), al = make_desc(base + TILE_A + off);
              const uint64_t bh = make_desc(base + 2 * TILE_A + off), bl = make_desc(base + 2 * TILE_A + TILE_B + off);
              const uint32_t first = (kb == c * CHUNK_KB && kk == 0) ? 0u : 1u;
              mma_tf32(dacc, al, bh, C::IDESC, first);  // small terms first
              mma_tf32(dacc, ah, bl, C::IDESC, 1u);
              mma_tf32(dacc, ah, bh, C::IDESC, 1u);
            }
            mma_commit(empty0 + 8 * s);
          }
          mma_commit(tfull0 + 8 * j);  // fires when this chunk's MMAs have completed
        }
      }
    }
  } else {
    // Epilogue warps 2..: TMEM lane quarter q = warp % 4 holds tile rows
    // 32q..32q+31; warp group h = (warp - 2) / 4 owns columns 128h..128h+127.
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;
    uint32_t cg = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
      const Tile tl = decode_tile<BN>(p, tile);
      constexpr int EC = 128;  // columns per epilogue warp
      float acc[EC];
#pragma unroll
      for (int i = 0; i < EC; i++) acc[i] = 0.0f;
      for (int c = 0; c < nchunks; c++, cg++) {
        const uint32_t j = cg % NBUF, use = cg / NBUF;
        bool w = mbar_wait(tfull0 + 8 * j, use & 1, p.err, 3);
        w = __all_sync(0xffffffffu, w);  // tcgen05.ld below is warp-collective
        if (!w) { ok = false; break; }
        tc_fence_after();
        const uint32_t src = tmem + (uint32_t(32 * q) << 16) + j * BN + h * EC;
#pragma unroll
        for (int cc = 0; cc < BN / 32; cc += 2) {
          uint32_t r0[32], r1[32];
          tmem_ld32_nowait(src + uint32_t(32 * cc), r0);
          tmem_ld32_nowait(src + uint32_t(32 * cc + 32), r1);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; i++) {
            acc[32 * cc + i] = __fadd_rn(acc[32 * cc + i], __uint_as_float(r0[i]));
            acc[32 * cc + 32 + i] = __fadd_rn(acc[32 * cc + 32 + i], __uint_as_float(r1[i]));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty0 + 8 * j);
      }
      const bool good = __all_sync(0xffffffffu, ok && *reinterpret_cast<volatile int *>(p.err) == 0);
      if (!good) break;
      // Store: each warp owns rows 32q..32q+31 of the tile.  Per 32-column
      // block, lanes write their row into a padded shared-memory block, then
      // read it back by column so that every global access (store, bias,
      // residual) is one coalesced 128-byte row segment.
      float *st = ostage + (warp - 2) * 32 * STAGE_PITCH;
      const int64_t coff = (tl.bz / p.bin) * p.stride_c + (tl.bz % p.bin) * p.stride_c_in;
      float *cbase = p.C + coff;
      const float *res = p.epi.residual ? p.epi.residual + coff : nullptr;
      const int64_t col = int64_t(tl.n0) + h * EC + lane;
#pragma unroll
      for (int cb = 0; cb < EC / 32; cb++) {
#pragma unroll
        for (int i = 0; i < 32; i++) st[lane * STAGE_PITCH + i] = acc[32 * cb + i];
        __syncwarp();
        const int64_t c = col + 32 * cb;
        if (c < p.N) {
#pragma unroll 4
          for (int r = 0; r < 32; r++) {
            const int64_t row = int64_t(tl.m0) + 32 * q + r;
            if (row < p.M) cbase[row * p.ldc + c] = epi_apply(p.epi, st[r * STAGE_PITCH + lane], row, c, res);
          }
        }
        __syncwarp();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// ----------------------------------------------------------- split pre-pass
// src element (b, r, k) at src + (b / bin)*sbatch + (b % bin)*sbatch_in + r*rs + k*ks
// (one of rs/ks is 1).  Writes hi/lo[(b*rows + r)*Kp + k]; k in [K, Kp) is zero-filled.
__global__ void __launch_bounds__(256) pack_split(const float *__restrict__ src, int64_t rs, int64_t ks,
                                                  int64_t sbatch, int64_t bin, int64_t sbatch_in,
                                                  int64_t rows, int64_t K, int64_t Kp,
                                                  float *__restrict__ hi, float *__restrict__ lo) {
  __shared__ float tile[32][33];
  const int64_t b = blockIdx.z;
  const int64_t r0 = int64_t(blockIdx.y) * 32, k0 = int64_t(blockIdx.x) * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  const float *s = src + (b / bin) * sbatch + (b % bin) * sbatch_in;
  if (ks == 1) {  // k contiguous: read along k
    for (int i = ty; i < 32; i += 8) {
      const int64_t r = r0 + i, k = k0 + tx;
      tile[i][tx] = (r < rows && k < K) ? __ldg(s + r * rs + k) : 0.0f;
    }
  } else {  // r contiguous: read along r, transpose through shared memory
    for (int i = ty; i < 32; i += 8) {
      const int64_t k = k0 + i, r = r0 + tx;
      tile[tx][i] = (r < rows && k < K) ? __ldg(s + r * rs + k * ks) : 0.0f;
    }
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int64_t r = r0 + i, k = k0 + tx;
    if (r < rows && k < Kp) {
      const float x = tile[i][tx];
      uint32_t h;
      asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
      const float xh = __uint_as_float(h);
      const size_t o = size_t(b * rows + r) * size_t(Kp) + size_t(k);
      hi[o] = xh;
      lo[o] = __fsub_rn(x, xh);
    }
  }
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

bool make_map(CUtensorMap *m, const float *base, int64_t Kp, int64_t rows, int64_t batch, int box_rows = BM) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {cuuint64_t(Kp), cuuint64_t(rows), cuuint64_t(batch)};
  cuuint64_t strides[2] = {cuuint64_t(Kp) * 4, cuuint64_t(Kp) * 4 * cuuint64_t(rows)};
  cuuint32_t box[3] = {BK, cuuint32_t(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int64_t padded_k(int64_t K) { return ((K + BK - 1) / BK) * BK; }

}  // namespace

template <int BN>
silcu_status launch_tc(const TcParams &p, uint32_t grid, cudaStream_t s) {
  using C = Cfg<BN>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(tc_gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return fail(SILCU_CUDA_ERROR, "sgemm(tc): smem attribute: %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  tc_gemm_kernel<BN><<<grid, C::NUM_THREADS, C::SMEM_BYTES, s>>>(p);
  return check_launch("sgemm(tc)");
}

int64_t total_batch(const silcu_gemm_args &a) { return a.batch * (a.batch_inner > 1 ? a.batch_inner : 1); }

size_t tc_workspace_bytes(const silcu_gemm_args &a) {
  const int64_t Kp = padded_k(a.K > 0 ? a.K : 1);
  return size_t(2) * size_t(Kp) * size_t(total_batch(a)) * size_t(a.M + a.N) * sizeof(float) + 256;
}

silcu_status tc_run(const silcu_gemm_args &a, void *ws, size_t wsb, cudaStream_t s) {
  const int64_t Kp = padded_k(a.K > 0 ? a.K : 1);
  const size_t need = tc_workspace_bytes(a);
  if (!ws || wsb < need) return fail(SILCU_WORKSPACE_TOO_SMALL, "sgemm(tc): workspace %zu < %zu", wsb, need);
  if (a.M > (1 << 30) || a.N > (1 << 30) || Kp > (1 << 30))
    return fail(SILCU_UNSUPPORTED, "sgemm(tc): extent >= 2^30");
  const int BN = a.N > 128 ? 256 : 128;  // wide tiles unless N is small
  const int64_t tiles_m = (a.M + BM - 1) / BM, tiles_n = (a.N + BN - 1) / BN;
  const int64_t nb = total_batch(a), bin = a.batch_inner > 1 ? a.batch_inner : 1;
  if (tiles_m * tiles_n * nb > 0x7FFFFFFF) return fail(SILCU_UNSUPPORTED, "sgemm(tc): too many tiles");
  if (nb > 65535) return fail(SILCU_UNSUPPORTED, "sgemm(tc): batch > 65535");
  float *base = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
  const size_t a_elems = size_t(nb) * a.M * Kp, b_elems = size_t(nb) * a.N * Kp;
  float *a_hi = base, *a_lo = a_hi + a_elems, *b_hi = a_lo + a_elems, *b_lo = b_hi + b_elems;

  // A: rows m, k.  Non-transposed: (m, k) at m*lda + k.  Transposed: k*lda + m.
  {
    const int64_t rs = a.trans_a ? 1 : a.lda, ks = a.trans_a ? a.lda : 1;
    dim3 g(uint32_t(Kp / 32), uint32_t((a.M + 31) / 32), uint32_t(nb));
    pack_split<<<g, 256, 0, s>>>(a.A, rs, ks, a.stride_a, bin, a.stride_a_inner, a.M, a.K, Kp, a_hi, a_lo);
  }
  // B as rows n, k.  Non-transposed B [K,N]: (n, k) at k*ldb + n.  Transposed [N,K]: n*ldb + k.
  {
    const int64_t rs = a.trans_b ? a.ldb : 1, ks = a.trans_b ? 1 : a.ldb;
    dim3 g(uint32_t(Kp / 32), uint32_t((a.N + 31) / 32), uint32_t(nb));
    pack_split<<<g, 256, 0, s>>>(a.B, rs, ks, a.stride_b, bin, a.stride_b_inner, a.N, a.K, Kp, b_hi, b_lo);
  }
  silcu_status st = check_launch("sgemm(tc) pack", 2);
  if (st != SILCU_OK) return st;

  TcParams p;
  memset(&p, 0, sizeof(p));
  if (!make_map(&p.a_hi, a_hi, Kp, a.M, nb) || !make_map(&p.a_lo, a_lo, Kp, a.M, nb) ||
      !make_map(&p.b_hi, b_hi, Kp, a.N, nb, BN) || !make_map(&p.b_lo, b_lo, Kp, a.N, nb, BN))
    return fail(SILCU_CUDA_ERROR, "sgemm(tc): cuTensorMapEncodeTiled failed");
  p.C = a.C;
  p.ldc = a.ldc;
  p.stride_c = a.stride_c;
  p.bin = bin;
  p.stride_c_in = a.stride_c_inner;
  p.M = int(a.M);
  p.N = int(a.N);
  p.Kp = int(Kp);
  p.tiles_m = int(tiles_m);
  p.tiles_n = int(tiles_n);
  p.nbatch = int(nb);
  p.chunk_kb = CHUNK_KB_DEFAULT;
  if (const char *env = getenv("SILCU_TC_CHUNK_KB")) {  // tuning knob: K blocks per accumulation chunk
    const int v = atoi(env);
    if (v >= 1) p.chunk_kb = v;
  }
  p.epi.alpha = a.alpha;
  p.epi.bias = a.bias;
  p.epi.bias_len = a.bias_len > 0 ? a.bias_len : 1;
  p.epi.act = a.act;
  p.epi.residual = a.residual;
  p.epi.ldr = a.ldr;
  p.err = device_error_ptr();
  if (!p.err) return fail(SILCU_CUDA_ERROR, "sgemm(tc): no device error word");

  const int64_t total = tiles_m * tiles_n * nb;
  const uint32_t grid = uint32_t(total < sm_count() ? total : sm_count());
  return BN == 256 ? launch_tc<256>(p, grid, s) : launch_tc<128>(p, grid, s);
}

}  // namespace silcu

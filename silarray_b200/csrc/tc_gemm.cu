// fp32-faithful SGEMM on the 5th-generation tensor cores (sm_100a).
//
// Split precision (3xTF32, Ootomo & Yokota 2022, "Recovering single precision
// accuracy from Tensor Cores while surpassing the FP32 theoretical peak
// performance"): x = hi + lo with hi = tf32_rna(x), lo = x - hi (exact in
// fp32), and  A.B ~= Ah.Bh + Ah.Bl + Al.Bh  accumulated in fp32 in TMEM.
//
// Pipeline (persistent: one CTA per SM walks 128x128 output tiles):
//   split       operands may arrive already split (hi/lo arrays, K-major,
//               e.g. written by the producing kernel); otherwise a pre-pass
//               (pack_split / split_contig) writes hi/lo copies, K-major, K
//               padded to a multiple of 32;
//   warp 0      TMA producer: 4 boxes (A, B x hi, lo) of 16 fp32 per row
//               (64 B, 64-byte swizzle) per K block into a 4- to 8-stage
//               shared-memory ring;
//   warp 1      allocates all 512 TMEM columns (4 accumulator buffers of 128),
//               one thread issues tcgen05.mma.kind::tf32 (M=128, N=128, K=8)
//               x 3 per K step and tcgen05.commit to release ring slots and to
//               hand each finished chunk of CHUNK_KB K blocks to the epilogue;
//   warps 2-5   drain each chunk with tcgen05.ld into fp32 registers (round to
//               nearest), and at the end of a tile stage 32x32 blocks through
//               shared memory so that the alpha / bias / activation / residual
//               epilogue and the stores are coalesced 128-byte row segments.
// Each CTA loads its own tiles (no TMA multicast); large problems run as CTA
// pairs (tcgen05 cta_group::2, 256-row tiles), see tc_gemm_kernel.
// Every mbarrier wait is bounded (wall-clock limit via %globaltimer); on
// expiry it records an error in the device error word and the CTA unwinds,
// frees its TMEM and exits.
#include <cuda.h>
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "gemm_internal.cuh"
#include "tc_common.cuh"

namespace silcu {
namespace {
using namespace tc;

constexpr int BM = 128;
constexpr int BK = 16;    // K per ring stage: one 64-byte swizzle row of fp32
constexpr int KPAD = 32;  // K padding of the split copies written by the pre-pass

// Per-variant constants: BN = 64 (8-stage ring, 8 TMEM chunk buffers, 4
// epilogue warps of 64 columns), BN = 128 (6 stages, 4 buffers, 4 warps) or
// BN = 256 (4 stages, 2 buffers, 8 epilogue warps of 128 columns).  The wider
// tile halves the shared-memory operand traffic per FLOP of A.  Stages of 16
// k keep several TMA fills in flight while the MMAs consume one: a stage of
// 32 k at BN = 256 (96 KB) left room for only two, and the fill latency
// showed up as idle tensor cycles.
template <int BN_, bool PAIR_ = false>
struct Cfg {
  static constexpr int BN = BN_;
  static constexpr bool PAIR = PAIR_;
  static constexpr int TM = PAIR ? 2 * BM : BM;       // output rows per tile (a CTA pair: 256)
  static constexpr int ROWS_B = PAIR ? BN / 2 : BN;   // B rows (K-major copy) held per CTA
  static constexpr int TILE_A = BM * BK * 4;
  static constexpr int TILE_B = ROWS_B * BK * 4;
  static constexpr int STAGE_BYTES = 2 * TILE_A + 2 * TILE_B;  // Ahi, Alo, Bhi, Blo
  static constexpr int EC = BN >= 128 ? 128 : BN;  // columns per epilogue warp
  static constexpr int EPI_WARPS = 4 * (BN / EC);
  // 32x32 fp32 staging blocks per epilogue warp: pairs (smaller stages) can
  // afford two, so consecutive TMA stores overlap.
  static constexpr int OUT_BUFS = PAIR ? 2 : 1;
  static constexpr int OUT_STAGE_BYTES = EPI_WARPS * 4096 * OUT_BUFS;
  static constexpr int STAGES_FIT = (232448 - OUT_STAGE_BYTES - 1024 - 512) / STAGE_BYTES;
  static constexpr int STAGES = PAIR ? (STAGES_FIT < 8 ? STAGES_FIT : 8) : (192 * 1024) / STAGE_BYTES;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int SMEM_BYTES = RING_BYTES + OUT_STAGE_BYTES + 1024 + 512;
  static constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int NBUF = 512 / BN;  // TMEM accumulator buffers (chunks in flight)
  static constexpr uint32_t TMEM_COLS = 512;
  // Instruction descriptor: D fp32, A/B tf32, both K-major, N = BN, M = BM.
  static constexpr uint32_t IDESC =
      (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(TM >> 4) << 24);
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};
constexpr int CHUNK_KB_DEFAULT = 8;      // K blocks per TMEM accumulation chunk (128 k)
constexpr int GROUP_M = 8;

struct TcEpi {
  float alpha;
  const float *bias;
  int bias_len;
  int act;
  const float *residual;
  int64_t ldr;
};

struct __align__(64) TcParams {
  CUtensorMap a_hi, a_lo, b_hi, b_lo;  // 4-D {K, rows, batch_inner, batch}, box {32, 128|BN, 1, 1}
  CUtensorMap c_map, chi_map, clo_map; // 4-D {N, M, batch_inner, batch}, box {32, 32, 1, 1}
  CUtensorMap r_map;                   // the residual, same layout as C (used when tma_r)
  CUtensorMap p_map;                   // split-K partials: 4-D {BN, TM, ksplit, split tiles}, box {32, 32, 1, 1}
  float *C;                            // direct-store fallback when C cannot take TMA stores
  int64_t ldc, stride_c, stride_c_in;
  int M, N, K, tiles_m, tiles_n, nbatch, bin, chunk_kb;
  // Work items: tiles [0, full_items) whole; each later tile's K range in
  // ksplit parts whose plain partials leave through p_map (the epilogue then
  // runs in tile_finish).  full_items = all tiles when nothing is split.
  int full_items, ksplit;
  int tma_c, split_out, tma_r;
  // Implicit-GEMM convolution (conv != 0): A's rows are the output pixels of
  // an NHWC image batch [images, cv_H, cv_W, cv_C] and its K index runs over
  // (kh, kw, channel); a_hi / a_lo are im2col maps of the split input, and
  // each K block (16 channels of one filter tap) loads as one im2col box.
  int conv, cv_H, cv_W, cv_C, cv_K, cv_pad;
  TcEpi epi;
  int *err;
};

struct Tile {
  int bz, m0, n0;
};

// Grouped raster inside one batch: GROUP_M tile-rows sweep the N tiles
// together so the A and B strips they share stay in L2.
__host__ __device__ __forceinline__ Tile tile_at(int tiles_m, int tiles_n, int TM, int BN, int idx) {
  const int tiles_per_batch = tiles_m * tiles_n;
  Tile r;
  r.bz = idx / tiles_per_batch;
  const int t = idx % tiles_per_batch;
  const int group = t / (GROUP_M * tiles_n);
  const int first_m = group * GROUP_M;
  const int gm = tiles_m - first_m < GROUP_M ? tiles_m - first_m : GROUP_M;
  const int tm = first_m + (t % (GROUP_M * tiles_n)) % gm;
  const int tn = (t % (GROUP_M * tiles_n)) / gm;
  r.m0 = tm * TM;
  r.n0 = tn * BN;
  return r;
}

template <int TM, int BN>
__device__ __forceinline__ Tile decode_tile(const TcParams &p, int idx) {
  return tile_at(p.tiles_m, p.tiles_n, TM, BN, idx);
}


// Writes a lane's 32 values (its row of a 32x32 block) into the warp's 4 KB
// staging block in the TMA 128-byte-swizzle layout: 16-byte chunk j of row r
// sits at chunk j ^ (r & 7).  Conflict-free: 8 consecutive lanes cover all banks.
// mode 0 stores the values, 1 their tf32 hi part, 2 the lo remainder.
__device__ __forceinline__ float split_part(float x, int mode) {
  if (mode == 0) return x;
  const float hi = tf32_rna(x);
  return mode == 1 ? hi : __fsub_rn(x, hi);
}

template <int N>
__device__ __forceinline__ void stage_row_swz(float *st, int lane, const float (&v)[N], int base, int mode) {
#pragma unroll
  for (int j = 0; j < 8; j++) {
    float4 f = make_float4(split_part(v[base + 4 * j], mode), split_part(v[base + 4 * j + 1], mode),
                           split_part(v[base + 4 * j + 2], mode), split_part(v[base + 4 * j + 3], mode));
    *reinterpret_cast<float4 *>(st + lane * 32 + 4 * (j ^ (lane & 7))) = f;
  }
}

// Persistent: CTA i takes tiles i, i + gridDim.x, ...  The TMA ring, the MMA
// chunk buffers and the epilogue run as one continuous stream across tiles,
// so a tile's pipeline fill and its output store overlap its neighbours'.
//
// Accumulation is split in two levels (the remedy of Ootomo & Yokota for the
// tensor core's truncating fp32 accumulation): the MMAs of chunk_kb K blocks
// accumulate into one of NBUF TMEM buffers; the epilogue warps drain each
// finished chunk into fp32 registers with round-to-nearest adds while the
// MMAs continue in the other buffers.
//
// PAIR (a cluster of two CTAs on one TPC, tcgen05 cta_group::2): the pair
// computes 256 x BN tiles.  Each CTA loads its own 128 rows of A and half of
// the BN columns of B; the even CTA issues M = 256 MMAs that read both CTAs'
// shared memory and write each CTA's TMEM, waits on its own ring barriers
// (which also count the peer's TMA bytes) and commits to the barriers of both
// CTAs; both CTAs' epilogue warps release the accumulator buffers to it.
// SPLIT: the launch has split-K tiles (full_items < all tiles).  Launches
// without them use the SPLIT = false instance, which has none of the part
// logic and so the register allocation of the plain epilogue.
template <int BN_, bool PAIR, bool SPLIT>
__global__ void __launch_bounds__(Cfg<BN_>::NUM_THREADS, 1) tc_gemm_kernel(const __grid_constant__ TcParams p) {
  using C = Cfg<BN_, PAIR>;
  constexpr int BN = C::BN, STAGES = C::STAGES, NBUF = C::NBUF, RING_BYTES = C::RING_BYTES;
  constexpr int STAGE_BYTES = C::STAGE_BYTES, TILE_A = C::TILE_A, TILE_B = C::TILE_B;
  constexpr uint32_t TMEM_COLS = C::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float *ostage = reinterpret_cast<float *>(smem + RING_BYTES);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + RING_BYTES + C::OUT_STAGE_BYTES);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 2 * NBUF + C::EPI_WARPS);
  const uint32_t rbar0 = smem_u32(bars + 2 * STAGES + 2 * NBUF);  // per epilogue warp: residual block loaded
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
  const uint32_t tfull0 = smem_u32(bars + 2 * STAGES), tempty0 = smem_u32(bars + 2 * STAGES + NBUF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Work items: whole tiles, then (tile, K part) for the split tiles.
  const int total_tiles = p.full_items + (p.tiles_m * p.tiles_n * p.nbatch - p.full_items) * p.ksplit;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int first_tile = PAIR ? int(blockIdx.x >> 1) : int(blockIdx.x);
  const int tile_step = PAIR ? int(gridDim.x >> 1) : int(gridDim.x);
  const int nk = (p.K + BK - 1) / BK;
  const int CHUNK_KB = p.chunk_kb;
  // K blocks [kb0, kb1) of a work item, and its number of accumulation chunks.
  auto item_tile = [&](int item) {
    return (!SPLIT || item < p.full_items) ? item : p.full_items + (item - p.full_items) / p.ksplit;
  };
  auto item_part = [&](int item) { return (!SPLIT || item < p.full_items) ? -1 : (item - p.full_items) % p.ksplit; };
  auto k_range = [&](int item, int &kb0, int &kb1) {
    const int ks = item_part(item);
    kb0 = ks < 0 ? 0 : ks * nk / p.ksplit;
    kb1 = ks < 0 ? nk : (ks + 1) * nk / p.ksplit;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int j = 0; j < NBUF; j++) {
      mbar_init(tfull0 + 8 * j, 1);
      mbar_init(tempty0 + 8 * j, C::EPI_WARPS * (PAIR ? 2 : 1));  // one arrive per epilogue warp (of both CTAs)
    }
    for (int w = 0; w < C::EPI_WARPS; w++) mbar_init(rbar0 + 8 * w, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    if (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t kbg = 0;
      bool ok = true;
      for (int tile = first_tile; tile < total_tiles && ok; tile += tile_step) {
        const Tile tl = decode_tile<C::TM, BN>(p, item_tile(tile));
        const int bo = tl.bz / p.bin, bi = tl.bz % p.bin;
        const int am = tl.m0 + BM * int(rank), bn = tl.n0 + C::ROWS_B * int(rank);
        int kbs, kbe;
        k_range(tile, kbs, kbe);
        for (int kb = kbs; kb < kbe; kb++, kbg++) {
          const uint32_t s = kbg % STAGES;
          const uint32_t ph = (kbg / STAGES) & 1;
          if (kbg >= STAGES && !mbar_wait(empty0 + 8 * s, ph ^ 1, p.err, 1)) { ok = false; break; }
          const uint32_t full = full0 + 8 * s;
          const uint32_t dst = smem_u32(smem + s * STAGE_BYTES);
          const int kc = kb * BK;
          // im2col coordinates of this K block (convolution): filter tap and
          // channel offset, and the base input pixel of the tile's first row
          int cx = 0, cw = 0, ch = 0, cn = 0;
          uint16_t okw = 0, okh = 0;
          if (p.conv) {
            const int tap = kc / p.cv_C;
            cx = kc - tap * p.cv_C;
            okh = uint16_t(tap / p.cv_K);
            okw = uint16_t(tap - int(okh) * p.cv_K);
            cn = am / (p.cv_H * p.cv_W);
            const int r = am - cn * (p.cv_H * p.cv_W);
            ch = r / p.cv_W - p.cv_pad;
            cw = r % p.cv_W - p.cv_pad;
          }
          if (PAIR) {
            // Both CTAs' bytes complete on the even CTA's barrier, which expects them all.
            const uint32_t full_c = mapa_shared(full, 0);
            if (rank == 0) mbar_expect_tx(full, 2 * STAGE_BYTES);
            if (p.conv) {
              tma_load_im2col_pair(dst, &p.a_hi, full_c, cx, cw, ch, cn, okw, okh);
              tma_load_im2col_pair(dst + TILE_A, &p.a_lo, full_c, cx, cw, ch, cn, okw, okh);
            } else {
              tma_load_4d_pair(dst, &p.a_hi, full_c, kc, am, bi, bo);
              tma_load_4d_pair(dst + TILE_A, &p.a_lo, full_c, kc, am, bi, bo);
            }
            tma_load_4d_pair(dst + 2 * TILE_A, &p.b_hi, full_c, kc, bn, bi, bo);
            tma_load_4d_pair(dst + 2 * TILE_A + TILE_B, &p.b_lo, full_c, kc, bn, bi, bo);
          } else {
            mbar_expect_tx(full, STAGE_BYTES);
            if (p.conv) {
              tma_load_im2col(dst, &p.a_hi, full, cx, cw, ch, cn, okw, okh);
              tma_load_im2col(dst + TILE_A, &p.a_lo, full, cx, cw, ch, cn, okw, okh);
            } else {
              tma_load_4d(dst, &p.a_hi, full, kc, am, bi, bo);
              tma_load_4d(dst + TILE_A, &p.a_lo, full, kc, am, bi, bo);
            }
            tma_load_4d(dst + 2 * TILE_A, &p.b_hi, full, kc, bn, bi, bo);
            tma_load_4d(dst + 2 * TILE_A + TILE_B, &p.b_lo, full, kc, bn, bi, bo);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {  // the pair's MMAs are issued by the even CTA
      uint32_t kbg = 0, cg = 0;
      bool ok = true;
      for (int tile = first_tile; tile < total_tiles && ok; tile += tile_step) {
        int kbs, kbe;
        k_range(tile, kbs, kbe);
        const int nchunks = (kbe - kbs + CHUNK_KB - 1) / CHUNK_KB;
        for (int c = 0; c < nchunks && ok; c++, cg++) {
          const uint32_t j = cg % NBUF, use = cg / NBUF;
          if (cg >= NBUF && !mbar_wait(tempty0 + 8 * j, (use & 1) ^ 1, p.err, 4)) { ok = false; break; }
          tc_fence_after();
          const uint32_t dacc = tmem + j * BN;
          const int kc0 = kbs + c * CHUNK_KB, kb1 = min(kbe, kc0 + CHUNK_KB);
          for (int kb = kc0; kb < kb1; kb++, kbg++) {
            const uint32_t s = kbg % STAGES;
            const uint32_t ph = (kbg / STAGES) & 1;
            if (!mbar_wait(full0 + 8 * s, ph, p.err, 2)) { ok = false; break; }
            tc_fence_after();
            const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
#pragma unroll
            for (int kk = 0; kk < BK / 8; kk++) {
              const uint32_t off = kk * 32;  // 8 tf32 = 32 bytes along K inside the 64-byte row
              const uint64_t ah = make_desc_sw64(base + off), al = make_desc_sw64(base + TILE_A + off);
              const uint64_t bh = make_desc_sw64(base + 2 * TILE_A + off),
                             bl = make_desc_sw64(base + 2 * TILE_A + TILE_B + off);
              const uint32_t first = (kb == kc0 && kk == 0) ? 0u : 1u;
              if (PAIR) {
                mma_tf32_pair(dacc, al, bh, C::IDESC, first);  // small terms first
                mma_tf32_pair(dacc, ah, bl, C::IDESC, 1u);
                mma_tf32_pair(dacc, ah, bh, C::IDESC, 1u);
              } else {
                mma_tf32(dacc, al, bh, C::IDESC, first);  // small terms first
                mma_tf32(dacc, ah, bl, C::IDESC, 1u);
                mma_tf32(dacc, ah, bh, C::IDESC, 1u);
              }
            }
            if (PAIR) {  // the stage is free in both CTAs
              mma_commit_pair(empty0 + 8 * s);
              mma_commit_pair(mapa_shared(empty0 + 8 * s, 1));
            } else {
              mma_commit(empty0 + 8 * s);
            }
          }
          if (PAIR) {  // fires when this chunk's MMAs have completed, in both CTAs
            mma_commit_pair(tfull0 + 8 * j);
            mma_commit_pair(mapa_shared(tfull0 + 8 * j, 1));
          } else {
            mma_commit(tfull0 + 8 * j);
          }
        }
      }
    }
  } else {
    // Epilogue warps 2..: TMEM lane quarter q = warp % 4 holds tile rows
    // 32q..32q+31; warp group h = (warp - 2) / 4 owns columns 128h..128h+127.
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;
    float *st = ostage + (warp - 2) * 1024 * C::OUT_BUFS;
    uint32_t nstore = 0;
    const uint32_t rbar = rbar0 + 8 * (warp - 2);
    const uint64_t out_policy = l2_policy_evict_first();  // outputs are not re-read by this kernel
    uint32_t rphase = 0;
    uint32_t cg = 0;
    bool ok = true;
    for (int tile = first_tile; tile < total_tiles && ok; tile += tile_step) {
      const Tile tl = decode_tile<C::TM, BN>(p, item_tile(tile));
      const int m0 = tl.m0 + BM * int(rank);  // this CTA's 128 rows of the tile
      int kbs, kbe;
      k_range(tile, kbs, kbe);
      const int nchunks = (kbe - kbs + CHUNK_KB - 1) / CHUNK_KB;
      constexpr int EC = C::EC;
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
        if constexpr (EC >= 128) {
          // 128 accumulators per thread: one 32-column load at a time keeps
          // the drain within the register budget (no spills).
#pragma unroll
          for (int cc = 0; cc < EC / 32; cc++) {
            uint32_t r0[32];
            tmem_ld32_nowait(src + uint32_t(32 * cc), r0);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; i++) acc[32 * cc + i] = __fadd_rn(acc[32 * cc + i], __uint_as_float(r0[i]));
          }
        } else {
#pragma unroll
          for (int cc = 0; cc < EC / 32; cc += 2) {
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
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (PAIR) mbar_arrive_cluster(mapa_shared(tempty0 + 8 * j, 0));  // the MMA issuer's barrier
          else mbar_arrive(tempty0 + 8 * j);
        }
      }
      const bool good = __all_sync(0xffffffffu, ok && *reinterpret_cast<volatile int *>(p.err) == 0);
      if (!good) break;
      const int part = item_part(tile);
      if (SPLIT && part >= 0) {
        // A K part of a split tile: its plain partial, no epilogue.
        if (m0 + 32 * q >= p.M) continue;
#pragma unroll
        for (int cb = 0; cb < EC / 32; cb++) {
          const int col0 = tl.n0 + h * EC + 32 * cb;
          if (col0 >= p.N) break;  // warp-uniform
          float *sb = st + (C::OUT_BUFS == 2 ? (nstore & 1) * 1024 : 0);
          if (lane == 0) {
            if (C::OUT_BUFS == 2) bulk_wait_read1();
            else bulk_wait_read0();
          }
          __syncwarp();
          stage_row_swz(sb, lane, acc, 32 * cb, 0);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_4d(&p.p_map, smem_u32(sb), h * EC + 32 * cb, BM * int(rank) + 32 * q, part,
                         item_tile(tile) - p.full_items);
            bulk_commit();
          }
          nstore++;
        }
        continue;
      }
      // Epilogue math in registers (lane = row): alpha, bias, activation,
      // residual, in the reference's order; then 32x32 blocks leave through
      // shared memory (TMA stores, or a transposed coalesced store fallback).
      const int bo = tl.bz / p.bin, bi = tl.bz % p.bin;
      const int row = m0 + 32 * q + lane;
      const int64_t coff = int64_t(bo) * p.stride_c + int64_t(bi) * p.stride_c_in;
#pragma unroll
      for (int cb = 0; cb < EC / 32; cb++) {
        const int col0 = tl.n0 + h * EC + 32 * cb;
        if (col0 >= p.N) break;  // warp-uniform
        if (p.epi.alpha != 1.0f) {
#pragma unroll
          for (int i = 0; i < 32; i++) acc[32 * cb + i] = __fmul_rn(acc[32 * cb + i], p.epi.alpha);
        }
        if (p.epi.bias) {
          int bix = col0 % p.epi.bias_len;
#pragma unroll
          for (int i = 0; i < 32; i++) {
            acc[32 * cb + i] = __fadd_rn(acc[32 * cb + i], __ldg(p.epi.bias + bix));
            if (++bix == p.epi.bias_len) bix = 0;
          }
        }
        if (p.epi.act == SILCU_ACT_RELU) {
#pragma unroll
          for (int i = 0; i < 32; i++) acc[32 * cb + i] = acc[32 * cb + i] >= 0.0f ? acc[32 * cb + i] : 0.0f;
        } else if (p.epi.act == SILCU_ACT_SIGMOID) {
#pragma unroll
          for (int i = 0; i < 32; i++) acc[32 * cb + i] = sigmoid_ref(acc[32 * cb + i]);
        }
        if (p.epi.residual && p.tma_r && (p.tma_c || p.split_out)) {
          // The warp's 32 x 32 residual block arrives by one TMA load into the
          // staging block the output will leave through (128-byte swizzle:
          // 16-byte chunk j of row r at j ^ (r & 7)); each lane reads its row.
          if (m0 + 32 * q < p.M) {
            float *sb = st + (C::OUT_BUFS == 2 ? (nstore & 1) * 1024 : 0);
            if (lane == 0) {
              if (C::OUT_BUFS == 2) bulk_wait_read1();
              else bulk_wait_read0();
              mbar_expect_tx(rbar, 4096);
              tma_load_4d(smem_u32(sb), &p.r_map, rbar, col0, m0 + 32 * q, bi, bo);
            }
            const bool w = mbar_wait(rbar, rphase, p.err, 5);
            rphase ^= 1u;
            if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
#pragma unroll
            for (int j = 0; j < 8; j++) {
              const float4 r4 = *reinterpret_cast<const float4 *>(sb + lane * 32 + 4 * (j ^ (lane & 7)));
              acc[32 * cb + 4 * j] = __fadd_rn(acc[32 * cb + 4 * j], r4.x);
              acc[32 * cb + 4 * j + 1] = __fadd_rn(acc[32 * cb + 4 * j + 1], r4.y);
              acc[32 * cb + 4 * j + 2] = __fadd_rn(acc[32 * cb + 4 * j + 2], r4.z);
              acc[32 * cb + 4 * j + 3] = __fadd_rn(acc[32 * cb + 4 * j + 3], r4.w);
            }
            __syncwarp();
          }
        } else if (p.epi.residual && row < p.M) {
          const float *rp = p.epi.residual + coff + int64_t(row) * p.epi.ldr + col0;
          if (col0 + 32 <= p.N && ((reinterpret_cast<uintptr_t>(rp) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              const float4 r4 = __ldg(reinterpret_cast<const float4 *>(rp + i));
              acc[32 * cb + i] = __fadd_rn(acc[32 * cb + i], r4.x);
              acc[32 * cb + i + 1] = __fadd_rn(acc[32 * cb + i + 1], r4.y);
              acc[32 * cb + i + 2] = __fadd_rn(acc[32 * cb + i + 2], r4.z);
              acc[32 * cb + i + 3] = __fadd_rn(acc[32 * cb + i + 3], r4.w);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; i++)
              if (col0 + i < p.N) acc[32 * cb + i] = __fadd_rn(acc[32 * cb + i], __ldg(rp + i));
          }
        }
        if (m0 + 32 * q >= p.M) continue;  // a pair's second half past M: nothing to store
        if (p.tma_c || p.split_out) {
          // up to three outputs leave through the one staging block
#pragma unroll 1
          for (int o = 0; o < 3; o++) {
            if (o == 0 && !p.tma_c) continue;
            if (o > 0 && !p.split_out) break;
            float *sb = st + (C::OUT_BUFS == 2 ? (nstore & 1) * 1024 : 0);
            if (lane == 0) {  // the store that last used this block has read it
              if (C::OUT_BUFS == 2) bulk_wait_read1();
              else bulk_wait_read0();
            }
            __syncwarp();
            stage_row_swz(sb, lane, acc, 32 * cb, o);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              const CUtensorMap *m = o == 0 ? &p.c_map : (o == 1 ? &p.chi_map : &p.clo_map);
              tma_store_4d_hint(m, smem_u32(sb), col0, m0 + 32 * q, bi, bo, out_policy);
              bulk_commit();
            }
            nstore++;
          }
        } else {
          // Fallback (C not TMA-compatible): transpose through the staging
          // block (XOR-swizzled columns, conflict-free) and store 128-byte
          // row segments.
#pragma unroll
          for (int i = 0; i < 32; i++) st[lane * 32 + (i ^ lane)] = acc[32 * cb + i];
          __syncwarp();
          const int c = col0 + lane;
          if (c < p.N) {
            float *cp = p.C + coff + c;
#pragma unroll 4
            for (int r = 0; r < 32; r++) {
              const int rr = m0 + 32 * q + r;
              if (rr < p.M) cp[int64_t(rr) * p.ldc] = st[r * 32 + (lane ^ r)];
            }
          }
          __syncwarp();
        }
      }
    }
    if (lane == 0) bulk_wait_all0();  // every TMA store has completed before exit
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();  // no CTA frees TMEM or leaves while its peer may still use the pair
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// ----------------------------------------------------------- split pre-pass
// src element (b, r, k) at src + (b / bin)*sbatch + (b % bin)*sbatch_in + r*rs + k*ks
// (one of rs/ks is 1); when src_lo is given the value is src + src_lo (an
// operand already held as an exact hi/lo pair).  Writes hi/lo[(b*rows + r)*Kp + k];
// k in [K, Kp) is zero-filled.
__global__ void __launch_bounds__(256) pack_split(const float *__restrict__ src, const float *__restrict__ src_lo,
                                                  int64_t rs, int64_t ks, int64_t sbatch, int64_t bin,
                                                  int64_t sbatch_in, int64_t rows, int64_t K, int64_t Kp,
                                                  float *__restrict__ hi, float *__restrict__ lo) {
  __shared__ float tile[32][33];
  const int64_t b = blockIdx.z;
  const int64_t r0 = int64_t(blockIdx.y) * 32, k0 = int64_t(blockIdx.x) * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  const int64_t boff = (b / bin) * sbatch + (b % bin) * sbatch_in;
  const float *s = src + boff;
  const float *sl = src_lo ? src_lo + boff : nullptr;
  if (ks == 1) {  // k contiguous: read along k
    for (int i = ty; i < 32; i += 8) {
      const int64_t r = r0 + i, k = k0 + tx;
      float x = 0.0f;
      if (r < rows && k < K) {
        x = __ldg(s + r * rs + k);
        if (sl) x = __fadd_rn(x, __ldg(sl + r * rs + k));
      }
      tile[i][tx] = x;
    }
  } else {  // r contiguous: read along r, transpose through shared memory
    for (int i = ty; i < 32; i += 8) {
      const int64_t k = k0 + i, r = r0 + tx;
      float x = 0.0f;
      if (r < rows && k < K) {
        x = __ldg(s + r * rs + k * ks);
        if (sl) x = __fadd_rn(x, __ldg(sl + r * rs + k * ks));
      }
      tile[tx][i] = x;
    }
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int64_t r = r0 + i, k = k0 + tx;
    if (r < rows && k < Kp) {
      const float x = tile[i][tx];
      const float xh = tf32_rna(x);
      const size_t o = size_t(b * rows + r) * size_t(Kp) + size_t(k);
      hi[o] = xh;
      lo[o] = __fsub_rn(x, xh);
    }
  }
}

// Elementwise split of a contiguous K-major operand (no transposition):
// 4 elements per thread, 128-bit loads and stores.
// Transposing split of a pair (value = src + src_lo) for the aligned case:
// a CTA takes 128 rows (tokens) x 32 columns (dims) of one (batch, head)
// block, reads both arrays with 16-byte loads, transposes through padded
// shared memory and writes hi / lo rows of 128 with 16-byte stores.  Output
// as pack_split: element (c, r) of block z at ((z * cols + c) * rows + r).
__global__ void __launch_bounds__(256) transpose_split_pair(const float *__restrict__ src,
                                                            const float *__restrict__ src_lo, int64_t ld,
                                                            int64_t s_b, int64_t s_h, int64_t heads, int64_t rows,
                                                            int64_t cols, float *__restrict__ hi,
                                                            float *__restrict__ lo) {
  __shared__ float th[32][129], tl[32][129];
  const int tid = threadIdx.x;
  const int64_t z = blockIdx.z;
  const int64_t r0 = int64_t(blockIdx.x) * 128, c0 = int64_t(blockIdx.y) * 32;
  const int64_t boff = (z / heads) * s_b + (z % heads) * s_h;
  const float *sh = src + boff, *sl = src_lo + boff;
  const int f = tid & 7;
  float4 vh[4], vl[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int64_t r = r0 + (tid >> 3) + 32 * i;
    if (r < rows) {
      vh[i] = __ldg(reinterpret_cast<const float4 *>(sh + r * ld + c0) + f);
      vl[i] = __ldg(reinterpret_cast<const float4 *>(sl + r * ld + c0) + f);
    } else {
      vh[i] = vl[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int rl = (tid >> 3) + 32 * i;
    th[4 * f + 0][rl] = vh[i].x; th[4 * f + 1][rl] = vh[i].y; th[4 * f + 2][rl] = vh[i].z; th[4 * f + 3][rl] = vh[i].w;
    tl[4 * f + 0][rl] = vl[i].x; tl[4 * f + 1][rl] = vl[i].y; tl[4 * f + 2][rl] = vl[i].z; tl[4 * f + 3][rl] = vl[i].w;
  }
  __syncthreads();
  const int q = tid & 31;
  const int64_t r = r0 + 4 * q;
  if (r >= rows) return;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int d = (tid >> 5) + 8 * i;
    float x[4], h4[4], l4[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      x[e] = __fadd_rn(th[d][4 * q + e], tl[d][4 * q + e]);
      h4[e] = tf32_rna(x[e]);
      l4[e] = __fsub_rn(x[e], h4[e]);
    }
    const size_t o = size_t(z * cols + c0 + d) * size_t(rows) + size_t(r);
    *reinterpret_cast<float4 *>(hi + o) = make_float4(h4[0], h4[1], h4[2], h4[3]);
    *reinterpret_cast<float4 *>(lo + o) = make_float4(l4[0], l4[1], l4[2], l4[3]);
  }
}

__global__ void __launch_bounds__(256) split_contig(const float *__restrict__ src, uint64_t n,
                                                    float *__restrict__ hi, float *__restrict__ lo) {
  const uint64_t stride = uint64_t(gridDim.x) * 256 * 4;
  for (uint64_t i = (uint64_t(blockIdx.x) * 256 + threadIdx.x) * 4; i < n; i += stride) {
    if (i + 4 <= n) {
      const float4 x = __ldcs(reinterpret_cast<const float4 *>(src + i));
      float4 a, b;
      a.x = tf32_rna(x.x); b.x = __fsub_rn(x.x, a.x);
      a.y = tf32_rna(x.y); b.y = __fsub_rn(x.y, a.y);
      a.z = tf32_rna(x.z); b.z = __fsub_rn(x.z, a.z);
      a.w = tf32_rna(x.w); b.w = __fsub_rn(x.w, a.w);
      *reinterpret_cast<float4 *>(hi + i) = a;
      *reinterpret_cast<float4 *>(lo + i) = b;
    } else {
      for (uint64_t k = i; k < n; k++) {
        const float x = src[k], xh = tf32_rna(x);
        hi[k] = xh;
        lo[k] = __fsub_rn(x, xh);
      }
    }
  }
}

// ---------------------------------------------------------------- host side
int64_t padded_k(int64_t K) { return ((K + KPAD - 1) / KPAD) * KPAD; }

template <int BN, bool PAIR, bool SPLIT>
silcu_status launch_tc(const TcParams &p, uint32_t grid, cudaStream_t s) {
  using C = Cfg<BN, PAIR>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<BN, PAIR, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::SMEM_BYTES);
    if (e != cudaSuccess) return fail(SILCU_CUDA_ERROR, "sgemm(tc): smem attribute: %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(C::NUM_THREADS);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = PAIR ? 2 : 1;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, tc_gemm_kernel<BN, PAIR, SPLIT>, p);
  if (e != cudaSuccess) return fail(SILCU_CUDA_ERROR, "sgemm(tc): launch: %s", cudaGetErrorString(e));
  return check_launch("sgemm(tc)");
}

// CTA pairs (256-row tiles) when they occupy nearly every SM pair (90 %), or
// when K is long (>= 2048), where the halved B traffic per CTA pays even with
// split-K filling the grid: measured at M = 2048 / 4096, N = 768, K = 3072
// 59.2 -> 54.8 / 103.3 -> 94.7 us, and QKV (M = 2048, N = 2304, K = 768, 72
// pair tiles) 47.2 -> 45.8 us; at K = 768 with few tiles (N = 768, M = 4096)
// single CTAs stay ahead (38.2 vs 40.0 us).  SILCU_TC_PAIR = 0 / 1 forces the
// choice (tuning).
bool use_pair(int64_t M, int64_t tiles_n, int64_t nb, int64_t K) {
  static const int forced = [] {
    const char *e = getenv("SILCU_TC_PAIR");
    return e ? atoi(e) : -1;
  }();
  if (forced == 0 || forced == 1) return forced == 1 && M >= 2 * BM;
  const int64_t pair_tiles = (M + 2 * BM - 1) / (2 * BM) * tiles_n * nb;
  return M >= 2 * BM && (10 * pair_tiles >= 9 * (sm_count() / 2) || K >= 2048);
}

// Tile width: the widest that N needs.  Narrower tiles never pay for a
// better-filled last wave: measured per FLOP, BN = 128 costs ~1.7x and
// BN = 64 ~3x the time of BN = 256 (the single MMA-issuing thread, not the
// tensor core, bounds small-N MMAs).  SILCU_TC_BN = 64 / 128 / 256 forces
// the width (tuning).
int pick_bn(int64_t N) {
  static const int forced = [] {
    const char *e = getenv("SILCU_TC_BN");
    const int v = e ? atoi(e) : 0;
    return (v == 64 || v == 128 || v == 256) ? v : 0;
  }();
  if (forced) return forced;
  return N > 128 ? 256 : (N > 64 ? 128 : 64);
}

bool a_given_split(const silcu_gemm_args &a) { return a.A_hi && a.A_lo; }
bool b_given_split_kmajor(const silcu_gemm_args &a) { return a.B_hi && a.B_lo && a.trans_b; }

}  // namespace

int64_t total_batch(const silcu_gemm_args &a) { return a.batch * (a.batch_inner > 1 ? a.batch_inner : 1); }

namespace {

struct TcPlan {
  bool pair;
  int BN, TM, ksplit;
  int64_t tiles_m, tiles_n;
  int64_t full_items;  // tiles run whole; the rest run in ksplit K parts
};

// CTA pairs and tile width as above; then split K (batch 1 only) where the
// tiles fill the grid's last wave poorly.  Estimated time with T tiles on U
// persistent CTAs (pairs), a tile taking tau = 2 * 128 * BN * K FLOPs at one
// SM's share of the 3xTF32 ceiling (276 TFLOP/s over 148 SMs):
//   whole tiles                 ceil(T / U) tau
//   every tile in ks parts      ceil(T ks / U) / ks tau            + finish
//   the last wave's r tiles     (floor(T / U) + ceil(r ks / U) / ks) tau + finish
// where finish = 3 us + (1.5 x partial bytes + the split tiles' epilogue
// bytes) / 6.5 TB/s: the partials are written by the kernel and read back by
// the finishing pass, which also reads the residual and writes the outputs.
// The cheapest wins if it beats whole tiles by 5 % (the estimate's margin);
// e.g. at M = 2048 the N = 768 GEMMs split every tile in
// 3 parts and N = 3072 runs 74 whole pair tiles plus 22 in 3 parts.  Every
// part keeps at least two accumulation chunks (256 k).  SILCU_TC_KSPLIT = 1
// disables splitting, 2..8 splits every tile in that many parts (tuning).
TcPlan tc_plan(const silcu_gemm_args &a) {
  TcPlan pl;
  const int64_t Kp = padded_k(a.K > 0 ? a.K : 1);
  const int64_t nb = total_batch(a);
  pl.pair = use_pair(a.M, (a.N + 255) / 256, nb, a.K);
  pl.BN = pick_bn(a.N);
  pl.TM = pl.pair ? 2 * BM : BM;
  pl.tiles_n = (a.N + pl.BN - 1) / pl.BN;
  pl.tiles_m = (a.M + pl.TM - 1) / pl.TM;
  pl.ksplit = 1;
  static const int forced = [] {
    const char *e = getenv("SILCU_TC_KSPLIT");
    return e ? atoi(e) : 0;
  }();
  const int64_t U = pl.pair ? sm_count() / 2 : sm_count();
  const int64_t T = pl.tiles_m * pl.tiles_n * nb;
  pl.full_items = T;
  const int64_t nkb = (Kp + BK - 1) / BK;
  if (nb != 1 || forced == 1 || T > 65535) return pl;  // the finishing pass's grid.y counts split tiles
  if (forced >= 2 && forced <= 8) {
    pl.ksplit = int(forced < nkb ? forced : nkb);
    pl.full_items = 0;
    return pl;
  }
  const double tau = 2.0 * BM * pl.BN * double(Kp) / (276e12 / 148) * 1e6;  // us
  const double tile_elems = double(pl.TM) * pl.BN;
  const double epi_bytes = tile_elems * ((a.C ? 4 : 0) + (a.C_hi && a.C_lo ? 8 : 0) + (a.residual ? 4 : 0));
  auto cdiv = [](int64_t x, int64_t y) { return (x + y - 1) / y; };
  auto finish = [&](int64_t tiles, int ks) {
    return 3.0 + (1.5 * 4.0 * tile_elems * double(tiles) * ks + epi_bytes * double(tiles)) / 6.5e12 * 1e6;
  };
  const double whole = double(cdiv(T, U)) * tau;
  double best = 0.95 * whole;
  const int64_t r = T % U;
  for (int ks = 2; ks <= 8 && nkb / ks >= 2 * CHUNK_KB_DEFAULT; ks++) {
    const double all = double(cdiv(T * ks, U)) / ks * tau + finish(T, ks);
    if (all < best) best = all, pl.ksplit = ks, pl.full_items = 0;
    if (r != 0 && T > U) {
      const double tail = (double(T / U) + double(cdiv(r * ks, U)) / ks) * tau + finish(r, ks);
      if (tail < best) best = tail, pl.ksplit = ks, pl.full_items = T - r;
    }
  }
  return pl;
}

size_t partial_bytes(const silcu_gemm_args &a, const TcPlan &pl) {
  const int64_t tiles = pl.tiles_m * pl.tiles_n * total_batch(a);
  return pl.ksplit > 1 ? size_t(tiles - pl.full_items) * pl.ksplit * pl.TM * pl.BN * sizeof(float) + 256 : 0;
}

// Finishes the split tiles: sums each element's K-part partials in part
// order (round to nearest), then the epilogue in the tensor-core kernel's
// order: alpha, bias, activation, residual; plain and / or split (hi, lo)
// output.  blockIdx.y = split tile, a thread = 4 columns of one row; vec
// (N, ldc, ldr multiples of 4 and 16-byte aligned outputs / residual) selects
// 16-byte accesses.
__device__ __forceinline__ float finish_one(float v, int64_t col, const TcEpi &epi) {
  if (epi.alpha != 1.0f) v = __fmul_rn(v, epi.alpha);
  if (epi.bias) v = __fadd_rn(v, epi.bias[col % epi.bias_len]);
  if (epi.act == SILCU_ACT_RELU) v = v >= 0.0f ? v : 0.0f;
  else if (epi.act == SILCU_ACT_SIGMOID) v = sigmoid_ref(v);
  return v;
}

__global__ void __launch_bounds__(256) tile_finish(const float *__restrict__ part, int ksplit, int full_items,
                                                   int tiles_m, int tiles_n, int TM, int BN, int M, int N,
                                                   TcEpi epi, float *C, int64_t ldc, float *C_hi, float *C_lo,
                                                   int vec) {
  const int bn4 = BN >> 2;
  const int g = blockIdx.x * 256 + threadIdx.x;
  if (g >= TM * bn4) return;
  const int rin = g / bn4, cin = (g - rin * bn4) << 2;
  const Tile tl = tile_at(tiles_m, tiles_n, TM, BN, full_items + int(blockIdx.y));
  const int row = tl.m0 + rin, col = tl.n0 + cin;
  if (row >= M || col >= N) return;
  const int64_t plane = int64_t(TM) * BN;
  const float *src = part + int64_t(blockIdx.y) * ksplit * plane + int64_t(rin) * BN + cin;
  float4 q[8];
#pragma unroll
  for (int k = 0; k < 8; k++)
    if (k < ksplit) q[k] = __ldcs(reinterpret_cast<const float4 *>(src + k * plane));
  float v[4] = {q[0].x, q[0].y, q[0].z, q[0].w};
#pragma unroll
  for (int k = 1; k < 8; k++)
    if (k < ksplit) {
      v[0] = __fadd_rn(v[0], q[k].x);
      v[1] = __fadd_rn(v[1], q[k].y);
      v[2] = __fadd_rn(v[2], q[k].z);
      v[3] = __fadd_rn(v[3], q[k].w);
    }
  const int nv = N - col < 4 ? N - col : 4;
  float rr[4] = {0.f, 0.f, 0.f, 0.f};
  if (epi.residual) {
    const float *rp = epi.residual + int64_t(row) * epi.ldr + col;
    if (vec) {
      const float4 r = __ldg(reinterpret_cast<const float4 *>(rp));
      rr[0] = r.x, rr[1] = r.y, rr[2] = r.z, rr[3] = r.w;
    } else {
      for (int i = 0; i < nv; i++) rr[i] = __ldg(rp + i);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    v[i] = finish_one(v[i], int64_t(col) + i, epi);
    if (epi.residual) v[i] = __fadd_rn(v[i], rr[i]);
  }
  const int64_t o = int64_t(row) * ldc + col;
  float h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    h[i] = tf32_rna(v[i]);
    l[i] = __fsub_rn(v[i], h[i]);
  }
  if (vec) {
    if (C) *reinterpret_cast<float4 *>(C + o) = make_float4(v[0], v[1], v[2], v[3]);
    if (C_hi) {
      *reinterpret_cast<float4 *>(C_hi + o) = make_float4(h[0], h[1], h[2], h[3]);
      *reinterpret_cast<float4 *>(C_lo + o) = make_float4(l[0], l[1], l[2], l[3]);
    }
  } else {
    for (int i = 0; i < nv; i++) {
      if (C) C[o + i] = v[i];
      if (C_hi) {
        C_hi[o + i] = h[i];
        C_lo[o + i] = l[i];
      }
    }
  }
}

}  // namespace

void tc_describe(const silcu_gemm_args &a, silcu_gemm_plan *out) {
  const TcPlan pl = tc_plan(a);
  out->pair = pl.pair ? 1 : 0;
  out->tile_n = pl.BN;
  out->ksplit = pl.ksplit;
  out->tiles = pl.tiles_m * pl.tiles_n * total_batch(a);
  out->whole_tiles = pl.full_items;
}

size_t tc_workspace_bytes(const silcu_gemm_args &a) {
  const int64_t Kp = padded_k(a.K > 0 ? a.K : 1);
  size_t bytes = 256;
  if (!a_given_split(a)) bytes += size_t(2) * Kp * size_t(total_batch(a)) * size_t(a.M) * sizeof(float);
  if (!b_given_split_kmajor(a)) bytes += size_t(2) * Kp * size_t(total_batch(a)) * size_t(a.N) * sizeof(float);
  return bytes + partial_bytes(a, tc_plan(a));
}

silcu_status split_contiguous(const float *src, uint64_t n, float *hi, float *lo, cudaStream_t s) {
  if (n == 0) return SILCU_OK;
  const uint64_t g = (n / 4 + 255) / 256;
  const uint64_t cap = uint64_t(sm_count()) * 8;
  split_contig<<<uint32_t(g < cap ? (g ? g : 1) : cap), 256, 0, s>>>(src, n, hi, lo);
  return check_launch("split");
}

silcu_status tc_run(const silcu_gemm_args &a, void *ws, size_t wsb, cudaStream_t s, const TcConv *conv) {
  const int64_t Kp = padded_k(a.K > 0 ? a.K : 1);
  const size_t need = tc_workspace_bytes(a);
  if (need > 256 && (!ws || wsb < need))
    return fail(SILCU_WORKSPACE_TOO_SMALL, "sgemm(tc): workspace %zu < %zu", wsb, need);
  if (a.M > (1 << 30) || a.N > (1 << 30) || Kp > (1 << 30))
    return fail(SILCU_UNSUPPORTED, "sgemm(tc): extent >= 2^30");
  const int64_t nb = total_batch(a), bin = a.batch_inner > 1 ? a.batch_inner : 1, bout = a.batch;
  const TcPlan plan = tc_plan(a);
  const bool pair = plan.pair;
  const int BN = plan.BN;
  const int64_t tiles_n = plan.tiles_n, tiles_m = plan.tiles_m;
  const int ROWS_B = pair ? BN / 2 : BN;
  if (tiles_m * tiles_n * nb > 0x7FFFFFFF) return fail(SILCU_UNSUPPORTED, "sgemm(tc): too many tiles");
  if (nb > 65535) return fail(SILCU_UNSUPPORTED, "sgemm(tc): batch > 65535");
  const bool asplit = a_given_split(a), bsplit = b_given_split_kmajor(a);
  if (a.A_hi && a.trans_a) return fail(SILCU_UNSUPPORTED, "sgemm(tc): split A must be K-major (trans_a = 0)");
  if (asplit && !(aligned_view(a.A_hi, a.lda, a.stride_a_inner, a.stride_a) &&
                  aligned_view(a.A_lo, a.lda, a.stride_a_inner, a.stride_a)))
    return fail(SILCU_INVALID_ARGUMENT, "sgemm(tc): split A needs 16-byte aligned rows and batch strides");
  if (bsplit && !(aligned_view(a.B_hi, a.ldb, a.stride_b_inner, a.stride_b) &&
                  aligned_view(a.B_lo, a.ldb, a.stride_b_inner, a.stride_b)))
    return fail(SILCU_INVALID_ARGUMENT, "sgemm(tc): split B needs 16-byte aligned rows and batch strides");
  const bool split_out = a.C_hi && a.C_lo;
  const bool tma_c = a.C && aligned_view(a.C, a.ldc, a.stride_c_inner, a.stride_c);
  if (split_out && !(aligned_view(a.C_hi, a.ldc, a.stride_c_inner, a.stride_c) &&
                     aligned_view(a.C_lo, a.ldc, a.stride_c_inner, a.stride_c)))
    return fail(SILCU_INVALID_ARGUMENT, "sgemm(tc): split output needs 16-byte aligned rows and batch strides");
  if (!a.C && !split_out) return fail(SILCU_INVALID_ARGUMENT, "sgemm(tc): no output");

  float *cur = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
  TcParams p;
  memset(&p, 0, sizeof(p));
  int launches = 0;
  // A as rows m, K-major.
  if (conv) {
    if (!asplit || a.batch != 1 || bin != 1 || conv->C % BK != 0 || a.M != conv->N * conv->H * conv->W ||
        a.K != conv->Kf * conv->Kf * conv->C)
      return fail(SILCU_INVALID_ARGUMENT, "sgemm(tc): convolution operand does not match the GEMM");
    if (!make_im2col_map(&p.a_hi, conv->in_hi, conv->N, conv->H, conv->W, conv->C, int(conv->pad), BK, BM,
                         CU_TENSOR_MAP_SWIZZLE_64B) ||
        !make_im2col_map(&p.a_lo, conv->in_lo, conv->N, conv->H, conv->W, conv->C, int(conv->pad), BK, BM,
                         CU_TENSOR_MAP_SWIZZLE_64B))
      return fail(SILCU_CUDA_ERROR, "sgemm(tc): cuTensorMapEncodeIm2col failed (A)");
    p.conv = 1;
    p.cv_H = int(conv->H);
    p.cv_W = int(conv->W);
    p.cv_C = int(conv->C);
    p.cv_K = int(conv->Kf);
    p.cv_pad = int(conv->pad);
  } else if (asplit) {
    if (!make_map4(&p.a_hi, a.A_hi, a.K, a.M, a.lda, bin, a.stride_a_inner, bout, a.stride_a, BK, BM, CU_TENSOR_MAP_SWIZZLE_64B) ||
        !make_map4(&p.a_lo, a.A_lo, a.K, a.M, a.lda, bin, a.stride_a_inner, bout, a.stride_a, BK, BM, CU_TENSOR_MAP_SWIZZLE_64B))
      return fail(SILCU_CUDA_ERROR, "sgemm(tc): cuTensorMapEncodeTiled failed (A)");
  } else {
    const size_t el = size_t(nb) * a.M * Kp;
    float *hi = cur, *lo = cur + el;
    cur += 2 * el;
    const float *src = a.A ? a.A : a.A_hi;
    const float *src_lo = a.A ? nullptr : a.A_lo;
    const int64_t rs = a.trans_a ? 1 : a.lda, ks = a.trans_a ? a.lda : 1;
    if (!a.trans_a && !src_lo && Kp == a.K && a.lda == a.K && bin == 1 && a.stride_a == a.M * a.K) {
      const uint64_t n = uint64_t(el);
      uint64_t g = (n / 4 + 255) / 256;
      const uint64_t cap = uint64_t(sm_count()) * 8;
      split_contig<<<uint32_t(g < cap ? (g ? g : 1) : cap), 256, 0, s>>>(src, n, hi, lo);
    } else {
      dim3 g(uint32_t(Kp / 32), uint32_t((a.M + 31) / 32), uint32_t(nb));
      pack_split<<<g, 256, 0, s>>>(src, src_lo, rs, ks, a.stride_a, bin, a.stride_a_inner, a.M, a.K, Kp, hi, lo);
    }
    launches++;
    if (!make_map4(&p.a_hi, hi, Kp, a.M, Kp, bin, a.M * Kp, bout, bin * a.M * Kp, BK, BM, CU_TENSOR_MAP_SWIZZLE_64B) ||
        !make_map4(&p.a_lo, lo, Kp, a.M, Kp, bin, a.M * Kp, bout, bin * a.M * Kp, BK, BM, CU_TENSOR_MAP_SWIZZLE_64B))
      return fail(SILCU_CUDA_ERROR, "sgemm(tc): cuTensorMapEncodeTiled failed (A pack)");
  }
  // B as rows n, K-major.  Non-transposed B [K,N]: (n, k) at k*ldb + n.  Transposed [N,K]: n*ldb + k.
  if (bsplit) {
    if (!make_map4(&p.b_hi, a.B_hi, a.K, a.N, a.ldb, bin, a.stride_b_inner, bout, a.stride_b, BK, ROWS_B, CU_TENSOR_MAP_SWIZZLE_64B) ||
        !make_map4(&p.b_lo, a.B_lo, a.K, a.N, a.ldb, bin, a.stride_b_inner, bout, a.stride_b, BK, ROWS_B, CU_TENSOR_MAP_SWIZZLE_64B))
      return fail(SILCU_CUDA_ERROR, "sgemm(tc): cuTensorMapEncodeTiled failed (B)");
  } else {
    const size_t el = size_t(nb) * a.N * Kp;
    float *hi = cur, *lo = cur + el;
    cur += 2 * el;
    const float *src = a.B ? a.B : a.B_hi;
    const float *src_lo = a.B ? nullptr : a.B_lo;
    const int64_t rs = a.trans_b ? a.ldb : 1, ks = a.trans_b ? 1 : a.ldb;
    dim3 g(uint32_t(Kp / 32), uint32_t((a.N + 31) / 32), uint32_t(nb));
    pack_split<<<g, 256, 0, s>>>(src, src_lo, rs, ks, a.stride_b, bin, a.stride_b_inner, a.N, a.K, Kp, hi, lo);
    launches++;
    if (!make_map4(&p.b_hi, hi, Kp, a.N, Kp, bin, a.N * Kp, bout, bin * a.N * Kp, BK, ROWS_B, CU_TENSOR_MAP_SWIZZLE_64B) ||
        !make_map4(&p.b_lo, lo, Kp, a.N, Kp, bin, a.N * Kp, bout, bin * a.N * Kp, BK, ROWS_B, CU_TENSOR_MAP_SWIZZLE_64B))
      return fail(SILCU_CUDA_ERROR, "sgemm(tc): cuTensorMapEncodeTiled failed (B pack)");
  }
  if (launches) {
    silcu_status st = check_launch("sgemm(tc) pack", launches);
    if (st != SILCU_OK) return st;
  }
  if (tma_c && !make_map4(&p.c_map, a.C, a.N, a.M, a.ldc, bin, a.stride_c_inner, bout, a.stride_c, 32, 32))
    return fail(SILCU_CUDA_ERROR, "sgemm(tc): cuTensorMapEncodeTiled failed (C)");
  if (split_out &&
      (!make_map4(&p.chi_map, a.C_hi, a.N, a.M, a.ldc, bin, a.stride_c_inner, bout, a.stride_c, 32, 32) ||
       !make_map4(&p.clo_map, a.C_lo, a.N, a.M, a.ldc, bin, a.stride_c_inner, bout, a.stride_c, 32, 32)))
    return fail(SILCU_CUDA_ERROR, "sgemm(tc): cuTensorMapEncodeTiled failed (split C)");
  if (a.residual && aligned_view(a.residual, a.ldr, a.stride_c_inner, a.stride_c)) {
    if (!make_map4(&p.r_map, a.residual, a.N, a.M, a.ldr, bin, a.stride_c_inner, bout, a.stride_c, 32, 32))
      return fail(SILCU_CUDA_ERROR, "sgemm(tc): cuTensorMapEncodeTiled failed (residual)");
    p.tma_r = 1;
  }
  p.C = a.C;
  p.ldc = a.ldc;
  p.stride_c = a.stride_c;
  p.stride_c_in = a.stride_c_inner;
  p.bin = int(bin);
  p.M = int(a.M);
  p.N = int(a.N);
  p.K = int(Kp);  // K blocks past K read zeros (TMA fill or packed padding)
  p.tiles_m = int(tiles_m);
  p.tiles_n = int(tiles_n);
  p.nbatch = int(nb);
  p.tma_c = tma_c ? 1 : 0;
  p.split_out = split_out ? 1 : 0;
  p.chunk_kb = a.acc_chunk_k >= BK ? int(a.acc_chunk_k / BK) : CHUNK_KB_DEFAULT;
  if (const char *env = getenv("SILCU_TC_CHUNK_KB")) {  // tuning knob: K blocks per accumulation chunk
    const int v = atoi(env);
    if (v >= 1) p.chunk_kb = v;
  }
  p.epi.alpha = a.alpha;
  p.epi.bias = a.bias;
  p.epi.bias_len = int(a.bias_len > 0 ? a.bias_len : 1);
  p.epi.act = a.act;
  p.epi.residual = a.residual;
  p.epi.ldr = a.ldr;
  p.err = device_error_ptr();
  if (!p.err) return fail(SILCU_CUDA_ERROR, "sgemm(tc): no device error word");
  p.ksplit = plan.ksplit;
  p.full_items = int(plan.full_items);
  const int64_t split_tiles = tiles_m * tiles_n * nb - plan.full_items;
  float *part = nullptr;
  if (plan.ksplit > 1) {
    // Split tiles store plain partials (tile t, part k at z = k, w = t); their epilogue runs in tile_finish.
    part = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(cur) + 255) & ~uintptr_t(255));
    const int64_t plane = int64_t(plan.TM) * BN;
    if (!make_map4(&p.p_map, part, BN, plan.TM, BN, plan.ksplit, plane, split_tiles, plan.ksplit * plane, 32, 32))
      return fail(SILCU_CUDA_ERROR, "sgemm(tc): cuTensorMapEncodeTiled failed (split-K partials)");
  }
  const int64_t total = plan.full_items + split_tiles * plan.ksplit;
  silcu_status st;
  const bool split = plan.ksplit > 1;
  if (pair) {
    const int64_t pairs = sm_count() / 2;
    const uint32_t grid = uint32_t(2 * (total < pairs ? total : pairs));
    if (BN == 256) st = split ? launch_tc<256, true, true>(p, grid, s) : launch_tc<256, true, false>(p, grid, s);
    else if (BN == 128) st = split ? launch_tc<128, true, true>(p, grid, s) : launch_tc<128, true, false>(p, grid, s);
    else st = split ? launch_tc<64, true, true>(p, grid, s) : launch_tc<64, true, false>(p, grid, s);
  } else {
    const uint32_t grid = uint32_t(total < sm_count() ? total : sm_count());
    if (BN == 256) st = split ? launch_tc<256, false, true>(p, grid, s) : launch_tc<256, false, false>(p, grid, s);
    else if (BN == 128) st = split ? launch_tc<128, false, true>(p, grid, s) : launch_tc<128, false, false>(p, grid, s);
    else st = split ? launch_tc<64, false, true>(p, grid, s) : launch_tc<64, false, false>(p, grid, s);
  }
  if (st != SILCU_OK || plan.ksplit == 1) return st;
  TcEpi epi;
  epi.alpha = a.alpha;
  epi.bias = a.bias;
  epi.bias_len = int(a.bias_len > 0 ? a.bias_len : 1);
  epi.act = a.act;
  epi.residual = a.residual;
  epi.ldr = a.ldr;
  float *c_hi = split_out ? a.C_hi : nullptr, *c_lo = split_out ? a.C_lo : nullptr;
  auto al16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  const int vec = a.N % 4 == 0 && (!a.C || (a.ldc % 4 == 0 && al16(a.C))) &&
                  (!c_hi || (a.ldc % 4 == 0 && al16(c_hi) && al16(c_lo))) &&
                  (!a.residual || (a.ldr % 4 == 0 && al16(a.residual)));
  const dim3 grid(uint32_t((plan.TM * BN / 4 + 255) / 256), uint32_t(split_tiles));
  tile_finish<<<grid, 256, 0, s>>>(part, plan.ksplit, p.full_items, p.tiles_m, p.tiles_n, plan.TM, BN, p.M, p.N, epi,
                                   a.C, a.ldc, c_hi, c_lo, vec);
  return check_launch("sgemm(tc) split-K finish");
}

}  // namespace silcu

extern "C" silcu_status silcu_split_f32(const float *src, size_t rows, size_t cols, size_t ld, int transpose,
                                        float *hi, float *lo, silcu_stream stream) {
  using namespace silcu;
  if (rows == 0 || cols == 0) return SILCU_OK;
  if (!src || !hi || !lo || ld < cols) return fail(SILCU_INVALID_ARGUMENT, "split: bad argument");
  if (rows > 65535ull * 32 || cols > 65535ull * 32) return fail(SILCU_UNSUPPORTED, "split: extent too large");
  const int64_t R = transpose ? cols : rows, K = transpose ? rows : cols;
  const int64_t rs = transpose ? 1 : int64_t(ld), ks = transpose ? int64_t(ld) : 1;
  dim3 g(uint32_t((K + 31) / 32), uint32_t((R + 31) / 32), 1);
  pack_split<<<g, 256, 0, as_stream(stream)>>>(src, nullptr, rs, ks, 0, 1, 0, R, K, K, hi, lo);
  return check_launch("split");
}

extern "C" silcu_status silcu_transpose_split_f32(const float *src, const float *src_lo, size_t rows, size_t cols,
                                                  size_t ld, size_t batch, size_t heads, size_t s_b, size_t s_h,
                                                  float *hi, float *lo, silcu_stream stream) {
  using namespace silcu;
  if (rows == 0 || cols == 0 || batch == 0 || heads == 0) return SILCU_OK;
  if (!src || !hi || !lo || ld < cols) return fail(SILCU_INVALID_ARGUMENT, "transpose_split: bad argument");
  if (rows > 65535ull * 32 || cols > 65535ull * 32 || batch * heads > 65535)
    return fail(SILCU_UNSUPPORTED, "transpose_split: extent too large");
  // output block (b, h) is [cols, rows]: element (c, r) = src[b*s_b + h*s_h + r*ld + c]
  if (src_lo && cols % 32 == 0 && rows % 4 == 0 && ld % 4 == 0 && s_b % 4 == 0 && s_h % 4 == 0 && aligned16(src) &&
      aligned16(src_lo) && aligned16(hi) && aligned16(lo)) {
    dim3 g(uint32_t((rows + 127) / 128), uint32_t(cols / 32), uint32_t(batch * heads));
    transpose_split_pair<<<g, 256, 0, as_stream(stream)>>>(src, src_lo, int64_t(ld), int64_t(s_b), int64_t(s_h),
                                                          int64_t(heads), int64_t(rows), int64_t(cols), hi, lo);
    return check_launch("transpose_split");
  }
  const int64_t R = int64_t(cols), K = int64_t(rows);
  dim3 g(uint32_t((K + 31) / 32), uint32_t((R + 31) / 32), uint32_t(batch * heads));
  pack_split<<<g, 256, 0, as_stream(stream)>>>(src, src_lo, 1, int64_t(ld), int64_t(s_b), int64_t(heads),
                                               int64_t(s_h), R, K, K, hi, lo);
  return check_launch("transpose_split");
}

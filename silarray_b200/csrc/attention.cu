// Fused attention on the 5th-generation tensor cores: O = softmax(Q.K^T * scale) . V
// per (batch, head), without writing the score matrix to HBM.
//
// This fuses the reference's attention chain (bench/composite/bench_transformer.cpp:
// Q.dot(K.transpose()) * scale -> softmax -> .dot(V), i.e. gpu::dot_f32_ex,
// gpu::affine, gpu::softmax and gpu::sgemm_steel of include/gpu.h) into one
// kernel.  Both products are 3xTF32 (x = hi + lo, hi*hi + hi*lo + lo*hi) on
// tcgen05.mma; each score is rounded once as fl(dot * scale) as the reference's
// affine node does; the softmax is the streaming (online) form over key blocks
// of 128, so the result equals the reference's up to fp32 rounding.
//
// Persistent: one CTA per SM takes work items (128 query rows of one
// (batch, head), against all key blocks of 128 or, with a split key axis,
// a range of them) round-robin, and streams the key blocks of all its items
// through one pipeline, so an item's first loads and score products overlap
// the previous item's last blocks.  D = 64.
//   warp 0     TMA: per item Q (hi/lo), then K and V blocks (one stage each,
//              reloaded as soon as the MMA that read them completes)
//   warp 1     TMEM alloc; one thread issues S_0, S_1, then per block t
//              O_t = P_t V_t and S_{t+2} = Q K_{t+2}^T (S double-buffered, so
//              the softmax of block t + 1 overlaps P.V of block t); the score
//              MMAs have N = 128
//   warps 2-9  thread = query row (two warps per row quarter, each with half
//              of the keys and of the output columns): scores from TMEM, running
//              max / sum (exponentials on the hardware ex2 unit), P_j split into
//              hi/lo into TMEM (hi over the scores it replaces, lo in its own
//              columns: the A operand of the P.V MMA), O accumulated in registers
//              with round-to-nearest adds and rescaled as the max moves.
// Shared memory: Q 64 KB + K 64 KB + V 64 KB = 192 KB.  TMEM (512 columns):
// S / P_hi 2 x 128, P_lo 128, O 2 x 64.
// All waits are bounded (as in tc_gemm.cu); no TMA multicast, no clusters.
#include <cmath>
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace silcu {
namespace {
using namespace tc;

constexpr int QT = 128;  // query rows per CTA
constexpr int KB = 128;  // keys per block
constexpr int HD = 64;   // head dimension
constexpr int Q_ATOM = QT * 128;            // 16 KB: 128 rows x 32 fp32
constexpr int K_ATOM = KB * 128;            // 16 KB: 128 key rows x 32 fp32 (also V rows)
constexpr int VT_ATOM = HD * 128;           // 8 KB: V^T, 64 dim rows x 32 keys
constexpr int Q_BYTES = 2 * 2 * Q_ATOM;     // hi, lo x 2 atoms = 64 KB
constexpr int K_BYTES = 2 * 2 * K_ATOM;     // 64 KB
constexpr int V_BYTES = 2 * HD * KB * 4;    // hi, lo of 64 x 128 = 64 KB
constexpr int OFF_Q = 0, OFF_K = Q_BYTES, OFF_V = OFF_K + K_BYTES;
constexpr int DATA_BYTES = OFF_V + V_BYTES;  // 192 KB of 1024-aligned operand buffers
// Ahead of them: the mbarriers + the TMEM slot (256 B) and the row max / sum
// exchange between the softmax warps of a lane quarter (2 x ESPLIT x 128 floats).
// Softmax warps per TMEM lane quarter; each takes 1/ESPLIT of a block's keys
// and of the output columns.
constexpr int ESPLIT = 2;
constexpr int HEAD_BYTES = 256 + 2 * ESPLIT * QT * 4;
constexpr int SMEM_BYTES = 232448;  // the per-CTA maximum; the data start is aligned up past HEAD_BYTES
constexpr int EPI_WARPS = 4 * ESPLIT;
constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
// TMEM columns: S_j (then P_hi_j) in [128*(j&1), +128), P_lo in [256, 384),
// O_j in [384 + 64*(j&1), +64).
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_PLO = 256, COL_O = 384;
constexpr uint32_t IDESC_BASE = (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(QT >> 4) << 24);  // M = 128
constexpr uint32_t IDESC_QK = IDESC_BASE | (uint32_t(KB >> 3) << 17);  // N = 128 keys
constexpr uint32_t IDESC_PV = IDESC_BASE | (uint32_t(HD >> 3) << 17);  // N = 64 dims

struct __align__(64) AttnParams {
  CUtensorMap q_hi, q_lo, k_hi, k_lo, v_hi, v_lo;  // 4-D {inner, rows, heads, batch}
  float *O, *O_hi, *O_lo;
  int64_t ldo, so_b, so_h;
  int Sq, Sk, heads, tiles_q;
  int v_rows;  // V given as [Sk, D] rows (B operand of P.V read MN-major), else V^T [D, Sk]
  float scale;
  // scale_pow2: scale is a positive power of two, so fl(s * scale) is exact
  // and folds into the exponent (scale_log2e = scale * log2 e, also exact)
  // and into the block max (max fl(s * scale) = fl(max s * scale)).
  int scale_pow2;
  float scale_log2e;
  int *err;
  // Split KV: the key blocks of each (batch, head, query tile) in kv_splits
  // contiguous ranges, one CTA each; with kv_splits > 1 a CTA writes its
  // unnormalised O rows, row max m and row sum l to part_o / part_ml and
  // attn_combine forms the output.
  int kv_splits, units, items;  // items = units x kv_splits
  float *part_o, *part_ml;
};

// A work item: the query tile q0 of head h of batch b against the key
// blocks [kb0, kb0 + nb) (range sp of the unit's kv_splits).
struct Item {
  int q0, h, b, kb0, nb, unit, sp;
};

__device__ __forceinline__ Item item_of(const AttnParams &p, int w) {
  Item it;
  it.unit = w / p.kv_splits;
  it.sp = w - it.unit * p.kv_splits;
  const int qt = it.unit % p.tiles_q, bh = it.unit / p.tiles_q;
  it.h = bh % p.heads;
  it.b = bh / p.heads;
  it.q0 = qt * QT;
  const int nbt = (p.Sk + KB - 1) / KB;
  it.kb0 = it.sp * nbt / p.kv_splits;
  it.nb = (it.sp + 1) * nbt / p.kv_splits - it.kb0;
  return it;
}

// Position in this CTA's stream of key blocks: item i (= w), block j of it.
struct Cursor {
  const AttnParams &p;
  int i, w, j;
  Item it;
  __device__ explicit Cursor(const AttnParams &pp) : p(pp), i(0), w(blockIdx.x), j(0) {
    if (w < p.items) it = item_of(p, w);
  }
  __device__ void next() {
    if (++j == it.nb) {
      j = 0;
      i++;
      w += gridDim.x;
      if (w < p.items) it = item_of(p, w);
    }
  }
};

// Descriptor of V [keys, dims] rows as the MN-major B operand of P.V (N =
// dims, K = keys).  For a 32-bit type the MN-major operand must use the
// 128-byte swizzle with 32-byte atoms (descriptor layout 1), which the TMA
// writes with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B: rows of 32 dims (128 B),
// groups of 4 key rows 512 B apart (SBO), the second 32-dim box K_ATOM bytes
// on (LBO = 16 KB).  One MMA (8 keys) spans two groups: 1024 B per k-step.
__device__ __forceinline__ uint64_t make_desc_mn(uint32_t addr) {
  uint64_t d = 0;
  d |= uint64_t((addr & 0x3FFFFu) >> 4);
  d |= uint64_t((KB * 128) >> 4) << 16;
  d |= uint64_t(512 >> 4) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(1) << 61;
  return d;
}

enum Bar { kQFull = 0, kKFull = 1, kKEmpty = 2, kVFull = 3, kVEmpty = 4, kSFull = 5, kPFull = 7, kPEmpty = 8,
           kOFull = 9, kOEmpty = 11, kNumBars = 13 };

// D += A(TMEM, 128 x 8, K-major: lane = row, column = k) . B(shared memory).
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accum));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// e^x for x <= 0 as 2^(x log2 e) on the hardware base-2 exponential
// (ex2.approx: relative error about 2^-22; with the rounding of x log2 e the
// result is within ~1.5e-6 relative for x >= -30, and exactly 0 at -inf).
constexpr float kLog2e = 1.44269504088896341f;
__device__ __forceinline__ float exp_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(__fmul_rn(x, kLog2e)));
  return y;
}
// 2^(x c - mlog2): with c = log2 e and mlog2 = max log2 e it is e^(x - max)
// for x <= max (x = -inf gives 0; the fused product-difference differs from
// rounding (x - max) first by at most |max log2 e| 2^-24 in the exponent).
__device__ __forceinline__ float ex2_fma(float x, float c, float mlog2) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(__fmaf_rn(x, c, -mlog2)));
  return y;
}

// TMEM load of N (16 or 32, or 64 as two 32s) consecutive columns of this warp's lanes.
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t *r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[N]) {
  static_assert(N == 16 || N % 32 == 0, "16 or a multiple of 32 columns");
  if constexpr (N == 16) {
    tmem_ld16_nowait(taddr, r);
  } else {
#pragma unroll
    for (int c = 0; c < N; c += 32) tmem_ld32_nowait(taddr + c, *reinterpret_cast<uint32_t(*)[32]>(r + c));
  }
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <bool POW2>
__global__ void __launch_bounds__(NUM_THREADS, 1) attn_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem_raw);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + kNumBars);
  float *xch = reinterpret_cast<float *>(smem_raw + 256);
  uint8_t *smem =
      reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + HEAD_BYTES + 1023) & ~uintptr_t(1023));
  if (smem + DATA_BYTES > smem_raw + SMEM_BYTES) {  // uniform across the CTA: nothing has started yet
    if (threadIdx.x == 0) atomicCAS(p.err, 0, 99);
    return;
  }
  auto bar = [&](int i) { return smem_u32(bars + i); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // This CTA's work items w = blockIdx.x + i * gridDim.x (w < p.items), each
  // a (batch, head, query tile, key range); their key blocks form one stream
  // t = 0 .. T-1 through the pipeline, so the next item's Q, K, V loads and
  // first score products overlap the current item's last blocks.
  int T = 0;
  for (int w = blockIdx.x; w < p.items; w += gridDim.x) T += item_of(p, w).nb;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; i++) {
      const bool epi = (i == kPFull || i == kOEmpty || i == kOEmpty + 1);
      mbar_init(bar(i), epi ? EPI_WARPS : 1);
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
  const uint32_t base = smem_u32(smem);

  if (warp == 0) {
    if (lane == 0 && T > 0) {
      // K_{t+1} is loaded once S_t has completed (KEmpty completion t), V_t
      // once P.V_{t-1} has (VEmpty completion t - 1): the order in which the
      // MMA thread needs them.  An item's Q goes with its first K: S_t, the
      // last score product of the previous item, has then finished reading
      // the old Q.
      Cursor ck(p), cv(p);
      auto load_k = [&](const Cursor &c) {
        if (c.j == 0) {
          mbar_expect_tx(bar(kQFull), Q_BYTES);
          for (int a = 0; a < 2; a++) {
            tma_load_4d(base + OFF_Q + a * Q_ATOM, &p.q_hi, bar(kQFull), 32 * a, c.it.q0, c.it.h, c.it.b);
            tma_load_4d(base + OFF_Q + 2 * Q_ATOM + a * Q_ATOM, &p.q_lo, bar(kQFull), 32 * a, c.it.q0, c.it.h,
                        c.it.b);
          }
        }
        const int key = (c.it.kb0 + c.j) * KB;
        mbar_expect_tx(bar(kKFull), K_BYTES);
        for (int a = 0; a < 2; a++) {
          tma_load_4d(base + OFF_K + a * K_ATOM, &p.k_hi, bar(kKFull), 32 * a, key, c.it.h, c.it.b);
          tma_load_4d(base + OFF_K + 2 * K_ATOM + a * K_ATOM, &p.k_lo, bar(kKFull), 32 * a, key, c.it.h, c.it.b);
        }
      };
      auto load_v = [&](const Cursor &c) {
        const int key = (c.it.kb0 + c.j) * KB;
        mbar_expect_tx(bar(kVFull), V_BYTES);
        if (p.v_rows) {  // V rows: the boxes of K (32 dims x 128 keys), 32-byte-atom swizzle
          for (int a = 0; a < 2; a++) {
            tma_load_4d(base + OFF_V + a * K_ATOM, &p.v_hi, bar(kVFull), 32 * a, key, c.it.h, c.it.b);
            tma_load_4d(base + OFF_V + 2 * K_ATOM + a * K_ATOM, &p.v_lo, bar(kVFull), 32 * a, key, c.it.h, c.it.b);
          }
        } else {  // V^T: 4 boxes of 32 keys x 64 dims
          for (int a = 0; a < KB / 32; a++) {
            tma_load_4d(base + OFF_V + a * VT_ATOM, &p.v_hi, bar(kVFull), key + 32 * a, 0, c.it.h, c.it.b);
            tma_load_4d(base + OFF_V + V_BYTES / 2 + a * VT_ATOM, &p.v_lo, bar(kVFull), key + 32 * a, 0, c.it.h,
                        c.it.b);
          }
        }
      };
      load_k(ck);
      load_v(cv);
      bool ok = true;
      if (T > 1) {
        ok = mbar_wait(bar(kKEmpty), 0, p.err, 12);
        ck.next();
        if (ok) load_k(ck);
      }
      for (int t = 1; t < T && ok; t++) {
        if (t + 1 < T) {
          if (!mbar_wait(bar(kKEmpty), t & 1, p.err, 12)) break;
          ck.next();
          load_k(ck);
        }
        if (!mbar_wait(bar(kVEmpty), (t - 1) & 1, p.err, 11)) break;
        cv.next();
        load_v(cv);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && T > 0) {
      // Descriptors are built once per buffer and offset by constants (the
      // start-address field is the low 14 bits of a descriptor, address / 16,
      // so desc(a + o) = desc(a) + o / 16).
      const uint64_t dq = make_desc(base + OFF_Q);
      const uint64_t dk = make_desc(base + OFF_K), dv0 = make_desc(base + OFF_V);
      const uint64_t dvm = make_desc_mn(base + OFF_V);
      const bool mn = p.v_rows != 0;
      const uint32_t idesc_pv = mn ? (IDESC_PV | (1u << 16)) : IDESC_PV;  // B MN-major for V rows
      Cursor cq(p);
      auto qk = [&](int t) {  // S_t = Q K_t^T into buffer t & 1
        if (cq.j == 0 && !mbar_wait(bar(kQFull), cq.i & 1, p.err, 13)) return false;
        if (!mbar_wait(bar(kKFull), t & 1, p.err, 17)) return false;
        tc_fence_after();
        const uint32_t scol = tmem + 128 * (t & 1);
#pragma unroll
        for (int kk = 0; kk < HD / 8; kk++) {
          const uint32_t off = (kk & 3) * 32;
          const uint64_t qh = dq + uint64_t(((kk >> 2) * Q_ATOM + off) >> 4);
          const uint64_t ql = qh + uint64_t((2 * Q_ATOM) >> 4);
          const uint64_t kh = dk + uint64_t(((kk >> 2) * K_ATOM + off) >> 4);
          const uint64_t kl = kh + uint64_t((2 * K_ATOM) >> 4);
          mma_tf32(scol, ql, kh, IDESC_QK, kk == 0 ? 0u : 1u);
          mma_tf32(scol, qh, kl, IDESC_QK, 1u);
          mma_tf32(scol, qh, kh, IDESC_QK, 1u);
        }
        mma_commit(bar(kKEmpty));
        mma_commit(bar(kSFull + (t & 1)));
        cq.next();
        return true;
      };
      auto pv = [&](int t) {  // O_t = P_t V_t into buffer t & 1
        const int u = t & 1;
        if (!mbar_wait(bar(kPFull), t & 1, p.err, 14)) return false;
        if (!mbar_wait(bar(kVFull), t & 1, p.err, 15)) return false;
        if (t >= 2 && !mbar_wait(bar(kOEmpty + u), ((t >> 1) & 1) ^ 1, p.err, 16)) return false;
        tc_fence_after();
        const uint32_t phi = tmem + 128 * u, plo = tmem + COL_PLO, ocol = tmem + COL_O + 64 * u;
        const uint64_t dv = mn ? dvm : dv0;
#pragma unroll
        for (int kk = 0; kk < KB / 8; kk++) {
          // V^T: K-major, 8 keys = 32 bytes along a row; V rows: 8 keys = one 1024-byte row group.
          const uint64_t vh = dv + uint64_t((mn ? kk * 1024 : (kk >> 2) * VT_ATOM + (kk & 3) * 32) >> 4);
          const uint64_t vl = vh + uint64_t((mn ? 2 * K_ATOM : V_BYTES / 2) >> 4);
          mma_tf32_ts(ocol, plo + 8 * kk, vh, idesc_pv, kk == 0 ? 0u : 1u);
          mma_tf32_ts(ocol, phi + 8 * kk, vl, idesc_pv, 1u);
          mma_tf32_ts(ocol, phi + 8 * kk, vh, idesc_pv, 1u);
        }
        mma_commit(bar(kVEmpty));
        mma_commit(bar(kPEmpty));
        mma_commit(bar(kOFull + u));
        return true;
      };
      bool ok = qk(0);
      if (ok && T > 1) ok = qk(1);
      for (int t = 0; t < T && ok; t++) {
        ok = pv(t);
        // S_{t+2} reuses S_t's columns, which hold P_hi_t: issued after P.V_t,
        // and MMAs of one thread run in issue order.
        if (ok && t + 2 < T) ok = qk(t + 2);
      }
    }
  } else {
    // Softmax warps: thread = query row r of the tile (TMEM lane r); the two
    // warps of a lane quarter take key / output-column halves hh = 0, 1 and
    // meet through shared memory (named barrier 1 over the 256 epilogue threads).
    const int q = warp & 3;
    const int hh = (warp - 2) >> 2;
    const int r = 32 * q + lane;
    float *xmax = xch;                                         // [ESPLIT][QT]
    float *xsum = xmax + ESPLIT * QT;                          // [ESPLIT][QT]
    const uint32_t lane_base = tmem + (uint32_t(32 * q) << 16);
    constexpr int HK = KB / ESPLIT, HO = HD / ESPLIT;
    float o[HO];
#pragma unroll
    for (int i = 0; i < HO; i++) o[i] = 0.0f;
    float m = __int_as_float(0xff800000), l = 0.0f, corr_prev = 1.0f;
    // Where row r of an item's output goes: with a split key axis the row of
    // its (unit, range) slot in part_o / part_ml, else the element offset of
    // the row in O (-1: past Sq).
    auto out_of = [&](const Item &it) -> int64_t {
      if (p.kv_splits > 1) return (int64_t(it.unit) * p.kv_splits + it.sp) * QT + r;
      const int row = it.q0 + r;
      if (row >= p.Sq) return -1;
      return int64_t(it.b) * p.so_b + int64_t(it.h) * p.so_h + int64_t(row) * p.ldo + HO * hh;
    };
    // O = o / l, or with a split key axis this range's o, m, l; written once
    // the item's last O block is folded in.
    auto write_out = [&](int64_t dst, float m_it, float l_it) {
      if (p.kv_splits > 1) {
        float *po = p.part_o + dst * HD + HO * hh;
#pragma unroll
        for (int c = 0; c < HO; c += 4)
          *reinterpret_cast<float4 *>(po + c) = make_float4(o[c], o[c + 1], o[c + 2], o[c + 3]);
        if (hh == 0) *reinterpret_cast<float2 *>(p.part_ml + dst * 2) = make_float2(m_it, l_it);
        return;
      }
      if (dst < 0 || *reinterpret_cast<volatile int *>(p.err) != 0) return;
      const float inv = __frcp_rn(l_it);
#pragma unroll
      for (int c = 0; c < HO; c += 4) {
        float4 v = make_float4(__fmul_rn(o[c], inv), __fmul_rn(o[c + 1], inv), __fmul_rn(o[c + 2], inv),
                               __fmul_rn(o[c + 3], inv));
        if (p.O) *reinterpret_cast<float4 *>(p.O + dst + c) = v;
        if (p.O_hi) {
          float4 hv = make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
          *reinterpret_cast<float4 *>(p.O_hi + dst + c) = hv;
          *reinterpret_cast<float4 *>(p.O_lo + dst + c) =
              make_float4(__fsub_rn(v.x, hv.x), __fsub_rn(v.y, hv.y), __fsub_rn(v.z, hv.z), __fsub_rn(v.w, hv.w));
        }
      }
    };
    // fold O_t (relative to the max before block t + 1) into o
    auto fold = [&](int t) {
      const int u = t & 1;
      bool w = mbar_wait(bar(kOFull + u), (t >> 1) & 1, p.err, 20);
      if (!__all_sync(0xffffffffu, w)) return false;
      tc_fence_after();
      uint32_t r0[HO];
      tmem_ld_cols<HO>(lane_base + COL_O + 64 * u + HO * hh, r0);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kOEmpty + u));
#pragma unroll
      for (int i = 0; i < HO; i++) o[i] = __fadd_rn(__fmul_rn(o[i], corr_prev), __uint_as_float(r0[i]));
      return true;
    };
    // the current item (its block j of nb from key block kb0) and where
    // the previous one's rows go
    int item = blockIdx.x, j = 0, nb = 0, kb0 = 0;
    int64_t dst_prev = 0, dst = 0;
    if (T > 0) {
      const Item it = item_of(p, item);
      nb = it.nb, kb0 = it.kb0, dst = out_of(it);
    }
    float m_prev = m, l_prev = l;
    bool ok = true;
    for (int t = 0; t < T; t++) {
      const int s = t & 1;
      if (j == nb) {  // the next item: its row state starts afresh
        item += gridDim.x;
        const Item it = item_of(p, item);
        nb = it.nb, kb0 = it.kb0, j = 0;
        dst_prev = dst, dst = out_of(it);
        m_prev = m, l_prev = l;
        m = __int_as_float(0xff800000), l = 0.0f;
      }
      bool w = mbar_wait(bar(kSFull + s), (t >> 1) & 1, p.err, 19);
      if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
      tc_fence_after();
      float sc[HK];
      {
        uint32_t r0[HK];
        tmem_ld_cols<HK>(lane_base + 128 * s + HK * hh, r0);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < HK; i++) sc[i] = __uint_as_float(r0[i]);
      }
      float mj = __int_as_float(0xff800000);
      const int key0 = (kb0 + j) * KB;
      const bool tail = key0 + KB > p.Sk;
#pragma unroll
      for (int i = 0; i < HK; i++) {
        // the reference's `* scale` node (exact, and applied below, for a power-of-two scale)
        float x = POW2 ? sc[i] : __fmul_rn(sc[i], p.scale);
        if (tail && key0 + HK * hh + i >= p.Sk) x = __int_as_float(0xff800000);
        sc[i] = x;
        mj = fmaxf(mj, x);
      }
      if (POW2) mj = __fmul_rn(mj, p.scale);
      xmax[hh * QT + r] = mj;
      asm volatile("bar.sync 1, %0;" ::"n"(32 * EPI_WARPS) : "memory");
      float m_new = m;
#pragma unroll
      for (int e = 0; e < ESPLIT; e++) m_new = fmaxf(m_new, xmax[e * QT + r]);
      const float corr = (m == m_new) ? 1.0f : exp_ex2(__fsub_rn(m, m_new));
      // e^(x - m) = 2^(x log2 e - m log2 e): one fused multiply-add per score
      // (the max's product rounded once per block, -inf for an empty row)
      const float mlog2 = __fmul_rn(m_new, kLog2e);
      float ps = 0.0f;
#pragma unroll
      for (int i = 0; i < HK; i++) {
        const float e = ex2_fma(sc[i], POW2 ? p.scale_log2e : kLog2e, mlog2);
        sc[i] = e;
        ps += e;
      }
      xsum[hh * QT + r] = ps;
      m = m_new;
      // P_t: hi over this half's scores (already read), lo into the P_lo
      // columns once P.V_{t-1} has finished reading them.
      if (t >= 1) {
        bool w3 = mbar_wait(bar(kPEmpty), (t - 1) & 1, p.err, 22);
        if (!__all_sync(0xffffffffu, w3)) { ok = false; break; }
        tc_fence_after();
      }
#pragma unroll
      for (int c = 0; c < HK; c += 32) {
        uint32_t hv[32], lv[32];
        // P >= 0: round-to-nearest-away to tf32 is "add half a tf32 ulp,
        // clear the 13 low bits" (integer pipe, not the conversion unit).
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const uint32_t hb = (__float_as_uint(sc[c + i]) + 0x1000u) & 0xFFFFE000u;
          hv[i] = hb;
          lv[i] = __float_as_uint(__fsub_rn(sc[c + i], __uint_as_float(hb)));
        }
        tmem_st32(lane_base + 128 * s + HK * hh + c, hv);
        tmem_st32(lane_base + COL_PLO + HK * hh + c, lv);
      }
      tmem_st_wait();
      tc_fence_before();
      asm volatile("bar.sync 1, %0;" ::"n"(32 * EPI_WARPS) : "memory");
      float ls = xsum[r];
#pragma unroll
      for (int e = 1; e < ESPLIT; e++) ls = __fadd_rn(ls, xsum[e * QT + r]);
      l = __fadd_rn(__fmul_rn(l, corr), ls);
      if (lane == 0) mbar_arrive(bar(kPFull));
      if (t >= 1) {
        // O_{t-1}, folded while P.V_t runs; when it closed the previous item,
        // that item's rows are written and o starts afresh.
        if (!fold(t - 1)) { ok = false; break; }
        if (j == 0) {
          write_out(dst_prev, m_prev, l_prev);
#pragma unroll
          for (int i = 0; i < HO; i++) o[i] = 0.0f;
        }
      }
      corr_prev = corr;
      j++;
    }
    if (ok && T > 0 && fold(T - 1)) write_out(dst, m, l);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// Output of a split-KV launch: per query row, the shares of the S key ranges
// (O_s relative to its max m_s, sum l_s) rescaled to the common max:
// O = sum_s O_s e^(m_s - M) / sum_s l_s e^(m_s - M), ranges added in order.
// A thread = 4 output columns of one row.
__global__ void __launch_bounds__(256) attn_combine(const AttnParams p) {
  const int64_t g = int64_t(blockIdx.x) * 256 + threadIdx.x;
  const int c4 = int(g % (HD / 4)), r = int((g / (HD / 4)) % QT);
  const int unit = int(g / (HD / 4) / QT);
  if (unit >= p.units || *reinterpret_cast<volatile int *>(p.err) != 0) return;
  const int qt = unit % p.tiles_q, bh = unit / p.tiles_q;
  const int h = bh % p.heads, b = bh / p.heads;
  const int row = qt * QT + r;
  if (row >= p.Sq) return;
  const int S = p.kv_splits;
  float M = __int_as_float(0xff800000);
  for (int s = 0; s < S; s++) M = fmaxf(M, p.part_ml[((size_t(unit) * S + s) * QT + r) * 2]);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float L = 0.0f;
  for (int s = 0; s < S; s++) {
    const size_t slot = size_t(unit) * S + s;
    const float2 ml = *reinterpret_cast<const float2 *>(p.part_ml + (slot * QT + r) * 2);
    const float w = (ml.x == M) ? 1.0f : exp_ex2(__fsub_rn(ml.x, M));
    const float4 o = *reinterpret_cast<const float4 *>(p.part_o + (slot * QT + r) * HD + 4 * c4);
    acc.x = __fadd_rn(acc.x, __fmul_rn(o.x, w));
    acc.y = __fadd_rn(acc.y, __fmul_rn(o.y, w));
    acc.z = __fadd_rn(acc.z, __fmul_rn(o.z, w));
    acc.w = __fadd_rn(acc.w, __fmul_rn(o.w, w));
    L = __fadd_rn(L, __fmul_rn(ml.y, w));
  }
  const float inv = __frcp_rn(L);
  const float4 v = make_float4(__fmul_rn(acc.x, inv), __fmul_rn(acc.y, inv), __fmul_rn(acc.z, inv),
                               __fmul_rn(acc.w, inv));
  const int64_t off = int64_t(b) * p.so_b + int64_t(h) * p.so_h + int64_t(row) * p.ldo + 4 * c4;
  if (p.O) *reinterpret_cast<float4 *>(p.O + off) = v;
  if (p.O_hi) {
    const float4 hv = make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
    *reinterpret_cast<float4 *>(p.O_hi + off) = hv;
    *reinterpret_cast<float4 *>(p.O_lo + off) =
        make_float4(__fsub_rn(v.x, hv.x), __fsub_rn(v.y, hv.y), __fsub_rn(v.z, hv.z), __fsub_rn(v.w, hv.w));
  }
}

bool view_ok(const void *p, int64_t ld, int64_t sb, int64_t sh) {
  return p && aligned16(p) && ld % 4 == 0 && sb % 4 == 0 && sh % 4 == 0;
}

}  // namespace
}  // namespace silcu

using namespace silcu;

namespace {

// Key-range split per (batch, head, query tile) for a launch of U such
// units over nbt key blocks on the SMs (one CTA per SM): modelled time
// waves(U*S) * (ceil(nbt/S) + 1 block of fixed cost) plus the combine pass
// (about one block); a split is taken only when the model gains 15 %.
int choose_kv_splits(int64_t U, int64_t nbt) {
  const int64_t sms = sm_count();
  auto cost = [&](int64_t S) {
    const int64_t waves = (U * S + sms - 1) / sms;
    return double(waves * ((nbt + S - 1) / S + 1)) + (S > 1 ? 1.0 : 0.0);
  };
  int best = 1;
  double bc = cost(1);
  for (int64_t S = 2; S <= 4 && S <= nbt; S++) {
    const double c = cost(S);
    if (c < 0.85 * bc && c < cost(best)) best = int(S);
  }
  return best;
}

int64_t splits_for(const silcu_attention_args &a) {
  if (a.Sq <= 0 || a.Sk <= 0 || a.batch <= 0 || a.heads <= 0) return 1;
  const int64_t U = (a.Sq + QT - 1) / QT * a.heads * a.batch;
  const int64_t nbt = (a.Sk + KB - 1) / KB;
  if (const char *e = getenv("SILCU_ATTN_SPLITS")) {  // tuning override, clamped to [1, min(4, nbt)]
    const int64_t S = atoi(e);
    return S < 1 ? 1 : S > 4 ? 4 : S > nbt ? nbt : S;
  }
  return choose_kv_splits(U, nbt);
}

size_t split_ws_bytes(int64_t U, int64_t S) {
  if (S <= 1) return 0;
  return size_t(U) * S * QT * (HD + 2) * sizeof(float) + 256;
}

silcu_status attention_launch(const silcu_attention_args *ap, int64_t S, void *ws, size_t wsb,
                              silcu_stream stream) {
  if (!ap) return fail(SILCU_INVALID_ARGUMENT, "attention: null args");
  const silcu_attention_args &a = *ap;
  if (a.D != HD) return fail(SILCU_UNSUPPORTED, "attention: head dimension %lld (only 64)", (long long)a.D);
  if (a.Sq <= 0 || a.Sk <= 0 || a.batch <= 0 || a.heads <= 0)
    return fail(SILCU_INVALID_ARGUMENT, "attention: empty extent");
  const bool v_rows = a.V_hi || a.V_lo;
  if (v_rows && (a.Vt_hi || a.Vt_lo)) return fail(SILCU_INVALID_ARGUMENT, "attention: give V or V^T, not both");
  const float *v_hi = v_rows ? a.V_hi : a.Vt_hi, *v_lo = v_rows ? a.V_lo : a.Vt_lo;
  if (!(view_ok(a.Q_hi, a.ldq, a.sq_b, a.sq_h) && view_ok(a.Q_lo, a.ldq, a.sq_b, a.sq_h) &&
        view_ok(a.K_hi, a.ldk, a.sk_b, a.sk_h) && view_ok(a.K_lo, a.ldk, a.sk_b, a.sk_h) &&
        view_ok(v_hi, a.ldv, a.sv_b, a.sv_h) && view_ok(v_lo, a.ldv, a.sv_b, a.sv_h)))
    return fail(SILCU_INVALID_ARGUMENT, "attention: operands need 16-byte aligned rows and strides");
  const bool split_out = a.O_hi && a.O_lo;
  if (!a.O && !split_out) return fail(SILCU_INVALID_ARGUMENT, "attention: no output");
  if ((a.O && !view_ok(a.O, a.ldo, a.so_b, a.so_h)) ||
      (split_out && !(view_ok(a.O_hi, a.ldo, a.so_b, a.so_h) && view_ok(a.O_lo, a.ldo, a.so_b, a.so_h))))
    return fail(SILCU_INVALID_ARGUMENT, "attention: output needs 16-byte aligned rows and strides");
  const int64_t tiles_q = (a.Sq + QT - 1) / QT;
  if (tiles_q * a.heads * a.batch > 0x7FFFFFFF || a.Sq > (1 << 30) || a.Sk > (1 << 30))
    return fail(SILCU_UNSUPPORTED, "attention: too large");
  AttnParams p;
  memset(&p, 0, sizeof(p));
  const CUtensorMapSwizzle vsw = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;  // V rows: see make_desc_mn
  if (!make_map4(&p.q_hi, a.Q_hi, HD, a.Sq, a.ldq, a.heads, a.sq_h, a.batch, a.sq_b, 32, QT) ||
      !make_map4(&p.q_lo, a.Q_lo, HD, a.Sq, a.ldq, a.heads, a.sq_h, a.batch, a.sq_b, 32, QT) ||
      !make_map4(&p.k_hi, a.K_hi, HD, a.Sk, a.ldk, a.heads, a.sk_h, a.batch, a.sk_b, 32, KB) ||
      !make_map4(&p.k_lo, a.K_lo, HD, a.Sk, a.ldk, a.heads, a.sk_h, a.batch, a.sk_b, 32, KB) ||
      !(v_rows ? make_map4(&p.v_hi, v_hi, HD, a.Sk, a.ldv, a.heads, a.sv_h, a.batch, a.sv_b, 32, KB, vsw)
              : make_map4(&p.v_hi, v_hi, a.Sk, HD, a.ldv, a.heads, a.sv_h, a.batch, a.sv_b, 32, HD)) ||
      !(v_rows ? make_map4(&p.v_lo, v_lo, HD, a.Sk, a.ldv, a.heads, a.sv_h, a.batch, a.sv_b, 32, KB, vsw)
              : make_map4(&p.v_lo, v_lo, a.Sk, HD, a.ldv, a.heads, a.sv_h, a.batch, a.sv_b, 32, HD)))
    return fail(SILCU_CUDA_ERROR, "attention: cuTensorMapEncodeTiled failed");
  p.v_rows = v_rows ? 1 : 0;
  p.O = a.O;
  p.O_hi = split_out ? a.O_hi : nullptr;
  p.O_lo = split_out ? a.O_lo : nullptr;
  p.ldo = a.ldo;
  p.so_b = a.so_b;
  p.so_h = a.so_h;
  p.Sq = int(a.Sq);
  p.Sk = int(a.Sk);
  p.heads = int(a.heads);
  p.tiles_q = int(tiles_q);
  p.scale = a.scale;
  {
    int ex = 0;
    const bool normal = std::isfinite(a.scale) && a.scale > 0.0f && std::fabs(a.scale) >= 1.17549435e-38f;
    p.scale_pow2 = (normal && std::frexp(a.scale, &ex) == 0.5f && ex > -100 && ex < 100) ? 1 : 0;
    p.scale_log2e = a.scale * kLog2e;
  }
  p.err = device_error_ptr();
  if (!p.err) return fail(SILCU_CUDA_ERROR, "attention: no device error word");
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attn_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return fail(SILCU_CUDA_ERROR, "attention: smem attribute: %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  const int64_t U = tiles_q * a.heads * a.batch;
  const int64_t nbt = (a.Sk + KB - 1) / KB;
  if (S < 1 || S > nbt || U * S > 0x7FFFFFFF) S = 1;
  p.kv_splits = int(S);
  p.units = int(U);
  p.items = int(U * S);
  if (S > 1) {
    const size_t need = split_ws_bytes(U, S);
    if (!ws || wsb < need) return fail(SILCU_WORKSPACE_TOO_SMALL, "attention: workspace %zu < %zu", wsb, need);
    if (!aligned16(ws)) return fail(SILCU_INVALID_ARGUMENT, "attention: workspace not 16-byte aligned");
    p.part_o = static_cast<float *>(ws);
    p.part_ml = p.part_o + size_t(U) * S * QT * HD;
  }
  // persistent: one CTA per SM, items dealt round-robin
  const int64_t grid = U * S < sm_count() ? U * S : sm_count();
  if (p.scale_pow2)
    attn_kernel<true><<<uint32_t(grid), NUM_THREADS, SMEM_BYTES, as_stream(stream)>>>(p);
  else
    attn_kernel<false><<<uint32_t(grid), NUM_THREADS, SMEM_BYTES, as_stream(stream)>>>(p);
  silcu_status r = check_launch("attention");
  if (r != SILCU_OK || S == 1) return r;
  const int64_t threads = U * QT * (HD / 4);
  attn_combine<<<uint32_t((threads + 255) / 256), 256, 0, as_stream(stream)>>>(p);
  return check_launch("attention(combine)");
}

}  // namespace

extern "C" {

silcu_status silcu_attention_f32(const silcu_attention_args *args, silcu_stream stream) {
  return attention_launch(args, 1, nullptr, 0, stream);
}

size_t silcu_attention_workspace_bytes(const silcu_attention_args *args) {
  if (!args) return 0;
  const int64_t S = splits_for(*args);
  const int64_t U = (args->Sq + QT - 1) / QT * args->heads * args->batch;
  return split_ws_bytes(U, S);
}

silcu_status silcu_attention_ex(const silcu_attention_args *args, void *ws, size_t wsb, silcu_stream stream) {
  if (!args) return fail(SILCU_INVALID_ARGUMENT, "attention: null args");
  int64_t S = splits_for(*args);
  if (S > 1 && wsb < split_ws_bytes((args->Sq + QT - 1) / QT * args->heads * args->batch, S)) S = 1;
  return attention_launch(args, S, ws, wsb, stream);
}

}  // extern "C"

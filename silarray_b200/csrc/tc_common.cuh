// PTX building blocks shared by the tcgen05 kernels (tc_gemm.cu,
// attention.cu): mbarriers with bounded waits, TMA loads/stores, tcgen05
// MMA / commit / TMEM loads, shared-memory matrix descriptors, the tf32
// split, and host-side tensor-map encoding.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "common.cuh"

namespace silcu {
namespace tc {

constexpr unsigned long long WAIT_NS = 2000000000ull;  // 2 s per wait

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
// complete within `limit_ns`, or when another CTA already recorded an error.
static __device__ __noinline__ bool mbar_wait_limit(uint32_t bar, uint32_t parity, int *err, int code,
                                                     unsigned long long limit_ns) {
  // try_wait suspends in hardware until the phase completes or a short time
  // limit passes, so the first polls cost nothing; the wall-clock limit (a
  // slow %globaltimer read) only starts after them.
  for (int i = 0; i < 64; i++)
    if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 1;; i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*reinterpret_cast<volatile int *>(err) != 0) return false;
      if (globaltimer() - t0 > limit_ns) {
        atomicCAS(err, 0, code);
        return false;
      }
    }
  }
}

static __device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int *err, int code) {
  return mbar_wait_limit(bar, parity, err, code, WAIT_NS);
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// im2col load of a 4-D NHWC tensor {C, W, H, N}: pixelsPerColumn pixels
// walked in W, H, N order from the base pixel (w, h, n) inside the map's
// bounding box, channelsPerPixel channels from c, each pixel shifted by the
// filter tap (kw, kh); pixels outside the tensor read zeros.
__device__ __forceinline__ void tma_load_im2col(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c, int w,
                                                int h, int n, uint16_t kw, uint16_t kh) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c), "r"(w), "r"(h), "r"(n), "h"(kw), "h"(kh)
      : "memory");
}

// The same for a CTA pair (tcgen05 cta_group::2): completes on `bar`, which
// may be the pair leader's barrier.
__device__ __forceinline__ void tma_load_im2col_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c,
                                                     int w, int h, int n, uint16_t kw, uint16_t kh) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c), "r"(w), "r"(h), "r"(n), "h"(kw), "h"(kh)
      : "memory");
}

// CTA-pair form (tcgen05 cta_group::2): the box lands in this CTA's shared
// memory; the byte count completes on `bar`, a shared::cluster address that
// may be the pair leader's barrier.
__device__ __forceinline__ void tma_load_4d_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1,
                                                 int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Arrive on a barrier anywhere in the cluster (release at cluster scope).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// Every thread of every CTA in the cluster.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// TMA store of one 32x32 fp32 box from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_4d(const CUtensorMap *map, uint32_t src, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
// The same store with an L2 eviction-priority hint (createpolicy): outputs
// that the kernel never reads again are marked evict-first, so they do not
// push operand tiles that later tiles re-read out of the L2.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void tma_store_4d_hint(const CUtensorMap *map, uint32_t src, int c0, int c1, int c2, int c3,
                                                  uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3, %4, %5}], [%1], %6;" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t h;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
  return __uint_as_float(h);
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
// K-major operand, 64-byte swizzle: rows of 16 fp32 (64 B), 8-row groups
// 512 B apart (the layout a SWIZZLE_64B TMA box of 16 fp32 writes).
__device__ __forceinline__ uint64_t make_desc_sw64(uint32_t addr) {
  uint64_t d = 0;
  d |= uint64_t((addr & 0x3FFFFu) >> 4);
  d |= uint64_t(1) << 16;
  d |= uint64_t(512 >> 4) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(4) << 61;
  return d;
}

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

// Pair MMA (issued by the even CTA): A rows 0-127 from this CTA's shared
// memory and 128-255 from the peer's at the same offsets, B columns split in
// halves the same way; D in each CTA's TMEM (its 128 rows).
__device__ __forceinline__ void mma_tf32_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum));
}

// Completion of the pair's MMAs (issued so far by this thread) arrives once
// on `cluster_bar`, a shared::cluster address in either CTA of the pair.
__device__ __forceinline__ void mma_commit_pair(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
               : "memory");
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

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}


// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
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

// A 4-D fp32 view {inner, rows, bin, bout} with element strides {1, ld, s_in,
// s_out}, boxes {box0, box1, 1, 1}, 128-byte swizzle.  Strides of extent-1
// dimensions are replaced by a valid dummy.
inline bool make_map4(CUtensorMap *m, const float *base, int64_t inner, int64_t rows, int64_t ld, int64_t bin,
               int64_t s_in, int64_t bout, int64_t s_out, int box0, int box1,
               CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const int64_t span = ld * rows;
  if (bin <= 1) s_in = span;
  if (bout <= 1) s_out = s_in * (bin > 1 ? bin : 1);
  cuuint64_t dims[4] = {cuuint64_t(inner), cuuint64_t(rows), cuuint64_t(bin), cuuint64_t(bout)};
  cuuint64_t strides[3] = {cuuint64_t(ld) * 4, cuuint64_t(s_in) * 4, cuuint64_t(s_out) * 4};
  cuuint32_t box[4] = {cuuint32_t(box0), cuuint32_t(box1), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

typedef CUresult (*EncodeIm2colFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const int *, const int *, cuuint32_t, cuuint32_t,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// An fp32 NHWC tensor as the im2col source of a stride-1 convolution with
// padding pad on every side: the base pixels of the outputs span
// [-pad, extent - 1 - pad] in W and H (bounding-box corners -pad, -pad);
// boxes of `pixels` pixels x `channels` channels.
inline bool make_im2col_map(CUtensorMap *m, const float *base, int64_t N, int64_t H, int64_t W, int64_t C, int pad,
                            int channels, int pixels, CUtensorMapSwizzle swz) {
  static EncodeIm2colFn fn = nullptr;
  if (!fn) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeIm2colFn>(ptr);
  }
  if (!fn) return false;
  cuuint64_t dims[4] = {cuuint64_t(C), cuuint64_t(W), cuuint64_t(H), cuuint64_t(N)};
  cuuint64_t strides[3] = {cuuint64_t(C) * 4, cuuint64_t(W * C) * 4, cuuint64_t(H * W * C) * 4};
  int lower[2] = {-pad, -pad}, upper[2] = {-pad, -pad};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float *>(base), dims, strides, lower, upper,
            cuuint32_t(channels), cuuint32_t(pixels), es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline bool aligned_view(const void *p, int64_t ld, int64_t s_in, int64_t s_out) {
  return p && aligned16(p) && ld % 4 == 0 && s_in % 4 == 0 && s_out % 4 == 0 && ld > 0;
}

}  // namespace tc
}  // namespace silcu

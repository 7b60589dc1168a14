// Thin inline-PTX wrappers for the sm_100a features the tensor-core kernels
// use: mbarriers, TMA tensor loads (no multicast), and tcgen05 (TMEM
// allocation, MMA, commit, TMEM loads).  Written from the PTX ISA.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace tl {

// cuTensorMapEncodeTiled, fetched from the driver once (nullptr when the
// driver does not offer it).
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);
EncodeTiledFn tensor_map_encoder();

namespace ptx {

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// One bounded test of the phase: the thread may stay suspended in the
// instruction until the phase completes, for up to about 100 us (the
// suspend-time hint), so waiting warps do not spin through issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(100000u)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete, for at most
// `limit_ns`.  Returns false on timeout (the caller aborts its work).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && global_timer_ns() - t0 > limit_ns) return false;
  }
}

// ----------------------------------------------------- CTA pairs (clusters)
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The shared::cluster address of `local`'s counterpart in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(const void *local, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_addr(local)), "r"(rank));
  return a;
}

// Every thread of every CTA of the cluster arrives, then waits for all.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

// Arrive on an mbarrier of another CTA of the cluster (shared::cluster address).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// ----------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_3d(void *smem_dst, const CUtensorMap *map,
                                            uint64_t *bar, int32_t c0, int32_t c1,
                                            int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
      : "memory");
}

// Tiled TMA load of a box of a rank-(2 + nb) map (nb = 0..3 batch
// coordinates in zc), completing on `bar`; no multicast.
__device__ __forceinline__ void tma_load_nd(void *smem_dst, const CUtensorMap *map,
                                            uint64_t *bar, int32_t c0, int32_t c1, int nb,
                                            const int32_t *zc) {
  const uint64_t m = reinterpret_cast<uint64_t>(map);
  const uint32_t d = smem_addr(smem_dst), b = smem_addr(bar);
  switch (nb) {
    case 0:
      asm volatile(
          "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
          " [%0], [%1, {%2, %3}], [%4];" ::"r"(d),
          "l"(m), "r"(c0), "r"(c1), "r"(b)
          : "memory");
      break;
    case 1:
      asm volatile(
          "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
          " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(d),
          "l"(m), "r"(c0), "r"(c1), "r"(zc[0]), "r"(b)
          : "memory");
      break;
    case 2:
      asm volatile(
          "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
          " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(d),
          "l"(m), "r"(c0), "r"(c1), "r"(zc[0]), "r"(zc[1]), "r"(b)
          : "memory");
      break;
    default:
      asm volatile(
          "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
          " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(d),
          "l"(m), "r"(c0), "r"(c1), "r"(zc[0]), "r"(zc[1]), "r"(zc[2]), "r"(b)
          : "memory");
      break;
  }
}

// Tiled TMA load into this CTA's shared memory whose completion is counted
// on an mbarrier of the pair's first CTA (`bar` a shared::cluster address):
// the loads of both CTAs of a cta_group::2 product signal one barrier.  No
// multicast.
__device__ __forceinline__ void tma_load_pair(void *smem_dst, const CUtensorMap *map,
                                              uint32_t bar, int rank, const int32_t *c) {
  const uint64_t m = reinterpret_cast<uint64_t>(map);
  const uint32_t d = smem_addr(smem_dst);
  switch (rank) {
    case 2:
      asm volatile(
          "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
          " [%0], [%1, {%2, %3}], [%4];" ::"r"(d),
          "l"(m), "r"(c[0]), "r"(c[1]), "r"(bar)
          : "memory");
      break;
    case 3:
      asm volatile(
          "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
          " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(d),
          "l"(m), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(bar)
          : "memory");
      break;
    case 4:
      asm volatile(
          "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
          " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(d),
          "l"(m), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]), "r"(bar)
          : "memory");
      break;
    default:
      asm volatile(
          "cp.async.bulk.tensor.5d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
          " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(d),
          "l"(m), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]), "r"(c[4]), "r"(bar)
          : "memory");
      break;
  }
}

// Prefetch of a box of a rank-(2 + nb) map into L2 (no shared memory, no
// barrier): the data a later tiled load of the same box will find in L2.
__device__ __forceinline__ void tma_prefetch_nd(const CUtensorMap *map, int32_t c0, int32_t c1,
                                                int nb, const int32_t *zc) {
  const uint64_t m = reinterpret_cast<uint64_t>(map);
  switch (nb) {
    case 0:
      asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(m),
                   "r"(c0), "r"(c1)
                   : "memory");
      break;
    case 1:
      asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(m),
                   "r"(c0), "r"(c1), "r"(zc[0])
                   : "memory");
      break;
    case 2:
      asm volatile(
          "cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(m),
          "r"(c0), "r"(c1), "r"(zc[0]), "r"(zc[1])
          : "memory");
      break;
    default:
      asm volatile(
          "cp.async.bulk.prefetch.tensor.5d.L2.global.tile [%0, {%1, %2, %3, %4, %5}];" ::"l"(m),
          "r"(c0), "r"(c1), "r"(zc[0]), "r"(zc[1]), "r"(zc[2])
          : "memory");
      break;
  }
}

// Tiled TMA load of a box of a rank-`rank` map (3..5) at coordinates c.
__device__ __forceinline__ void tma_load_rank(void *smem_dst, const CUtensorMap *map,
                                              uint64_t *bar, int rank, const int32_t *c) {
  const uint64_t m = reinterpret_cast<uint64_t>(map);
  const uint32_t d = smem_addr(smem_dst), b = smem_addr(bar);
  switch (rank) {
    case 3:
      asm volatile(
          "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
          " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(d),
          "l"(m), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(b)
          : "memory");
      break;
    case 4:
      asm volatile(
          "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
          " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(d),
          "l"(m), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]), "r"(b)
          : "memory");
      break;
    default:
      asm volatile(
          "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
          " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(d),
          "l"(m), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]), "r"(c[4]), "r"(b)
          : "memory");
      break;
  }
}

// Tiled TMA store of a box to a rank-(2 + nb) map (bulk async-group).
__device__ __forceinline__ void tma_store_nd(const CUtensorMap *map, const void *smem_src,
                                             int32_t c0, int32_t c1, int nb, const int32_t *zc) {
  const uint64_t m = reinterpret_cast<uint64_t>(map);
  const uint32_t s = smem_addr(smem_src);
  switch (nb) {
    case 0:
      asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                   ::"l"(m), "r"(s), "r"(c0), "r"(c1)
                   : "memory");
      break;
    case 1:
      asm volatile(
          "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
              m),
          "r"(s), "r"(c0), "r"(c1), "r"(zc[0])
          : "memory");
      break;
    case 2:
      asm volatile(
          "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::
              "l"(m),
          "r"(s), "r"(c0), "r"(c1), "r"(zc[0]), "r"(zc[1])
          : "memory");
      break;
    default:
      asm volatile(
          "cp.async.bulk.tensor.5d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5, %6}], "
          "[%1];" ::"l"(m),
          "r"(s), "r"(c0), "r"(c1), "r"(zc[0]), "r"(zc[1]), "r"(zc[2])
          : "memory");
      break;
  }
}

// Tiled TMA store of a shared-memory box to global memory (no multicast;
// elements outside the tensor are not written), tracked by bulk async-groups.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *smem_src,
                                             int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_addr(smem_src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Waits until at most N committed bulk groups of this thread still read
// their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Waits until at most N committed bulk groups of this thread are incomplete
// (their global writes done).
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// TMEM of a CTA pair: allocated, released and freed by the same warp of
// both CTAs together.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D (+)= A * B on a CTA pair (cta_group::2): M = 256, rows 0-127 of A and the
// first N/2 columns of B in the issuing (first) CTA's shared memory, the
// rest at the same offsets in its peer's; each CTA's TMEM holds its 128
// rows of D.  Issued by one thread of the first CTA.
__device__ __forceinline__ void mma_tf32_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` (same offset) in every CTA of `mask` once all previously
// issued pair MMAs of this thread complete.
__device__ __forceinline__ void mma_commit_pair(uint64_t *bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_addr(bar)),
      "h"(mask)
      : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::tf32, one CTA.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}

// 16 consecutive 32-bit TMEM columns of this warp's 32 lanes (one per
// thread).  The load and its tcgen05.wait::ld are one asm statement: the
// load writes its destination registers asynchronously, and with the wait
// in a separate statement the compiler may copy those registers (a move, a
// spill) before the data has arrived.
__device__ __forceinline__ void tmem_load_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// x rounded to the nearest tf32 value (ties away from zero), as an fp32
// bit pattern whose low 13 mantissa bits are zero (cvt.rna.tf32.f32).
__device__ __forceinline__ float round_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// 2^x by the ex2.approx instruction (flush-to-zero; relative error about
// 2^-22), for softmax exponentials written as 2^((x - max) * log2(e)).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 32 consecutive 32-bit TMEM columns of this warp's 32 lanes (one per
// thread), load and wait in one statement (see tmem_load_32x32b_x16).
__device__ __forceinline__ void tmem_load_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Named barrier `id` (1..15) over `count` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// (the loads above already wait; kept for call sites that order on it)
__device__ __forceinline__ void tmem_load_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor (tcgen05 "matrix descriptor"):
//   [0,14) start address >> 4, [16,30) leading byte offset >> 4,
//   [32,46) stride byte offset >> 4, [46,48) version = 1,
//   [49,52) base offset = 0, [61,64) layout (swizzle) type.
enum SmemLayout : uint32_t {
  kSwizzleNone = 0,
  kSwizzle128B32BAtom = 1,  // MN-major 32-bit operands (TMA SWIZZLE_128B_ATOM_32B)
  kSwizzle128B = 2,         // K-major (TMA SWIZZLE_128B)
};

__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes,
                                              uint32_t sbo_bytes, SmemLayout layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3fffu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3fffu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3fffu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(layout) << 61;
  return d;
}

// Instruction descriptor for kind::tf32 with fp32 accumulation:
//   [4,6) D format (1 = f32), [7,10) A format (2 = tf32), [10,13) B format,
//   bit 15 A major (1 = MN), bit 16 B major, [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_tf32(uint32_t M, uint32_t N, bool a_mn,
                                                  bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

}  // namespace ptx
}  // namespace tl

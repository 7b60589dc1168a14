// Fused attention on the tensor cores for short sequences (T <= 192) and
// 64-wide heads: the executor's attention composite (include/nn/
// multi_head.h:45-52) without its T x T score tensor in HBM.
//
// Forward, one CTA per (batch, head, 128 query rows), 320 threads:
//   warp 0      TMA: the Q tile, all of K (K-major) and V (MN-major)
//   warp 1      TMEM owner, MMA issuer: S = Q K^T into TMEM (128 x nk fp32),
//               then O = P V block by block as the softmax hands over P
//   warps 2..9  softmax, two warps per TMEM lane quadrant on alternate
//               32-key blocks: pass 1 an online (max, sum) of S / divisor +
//               mask, merged across the pair through shared memory; pass 2
//               writes P = exp(x - max) / sum into shared memory in the
//               MMA's K-major layout (also the TMA box of the P store);
//               finally O from TMEM to global.
// P leaves through TMA stores (the backward reads it); S never leaves TMEM.
//
// Every wait is bounded (2 s): on timeout the CTA raises TL_FLAG_TIMEOUT,
// lets what it issued finish and returns.
#include "attention_tc.h"
#include "tc_ptx.cuh"

#include <cuda.h>

namespace tl {
namespace {

constexpr int kSoftWarps = 8;
constexpr int kThreads = 64 + 32 * kSoftWarps;
constexpr uint32_t BMQ = 128;  // query rows of a CTA
constexpr uint32_t HD = 64;    // head width
constexpr uint64_t kWaitLimitNs = 2000000000ull;

struct FwdMaps {
  CUtensorMap q, k, v, p;
};

struct FwdArgs {
  uint32_t T, H, nk, qtiles;
  const float *divisor, *mask;
  float *o;
  uint64_t sb, sh, ld;  // element strides of q, k, v, o: batch, head, row
  uint32_t *status;
};

// Shared memory (offsets from a 1024-aligned base): Q 2 x [128 x 32],
// K 2 x [nk x 32] (K-major, 128-byte swizzle), V 2 x [nk x 32] (MN-major,
// 32-byte-atom swizzle), P (nk / 32) x [128 x 32] (K-major), barriers.
constexpr uint32_t kQ = 0;
constexpr uint32_t kK = kQ + 2 * BMQ * 128;
constexpr uint32_t kV = kK + 2 * kMaxFusedKeys * 128;
constexpr uint32_t kP = kV + 2 * kMaxFusedKeys * 128;
constexpr uint32_t kBars = kP + (kMaxFusedKeys / 32) * BMQ * 128;
constexpr size_t kFwdSmem = 1024 + kBars + 256;
static_assert(kFwdSmem <= 232448, "forward tile exceeds shared memory");

__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t j) {
  return r * 128u + ((j ^ (r & 7u)) << 4);
}

__device__ __forceinline__ void online_add(float &m, float &s, float x) {
  if (x > m) {
    s = s * expf(m - x) + 1.0f;
    m = x;
  } else if (x != -INFINITY) {
    s += expf(x - m);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
attn_fwd_kernel(const __grid_constant__ FwdMaps maps, const FwdArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kBars);
  uint64_t *bar_qk = bars, *bar_v = bars + 1, *bar_s = bars + 2, *bar_o = bars + 3;
  uint64_t *bar_p = bars + 4;  // one per 32-key block
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar_p + kMaxFusedKeys / 32);
  volatile uint32_t *abort_flag = tmem_slot + 1;
  // (max, sum) of each row half, exchanged after pass 1 (Q is dead by then)
  float2 *red = reinterpret_cast<float2 *>(smem + kQ);

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const uint32_t nkb = a.nk / 32;
  const uint32_t qt = blockIdx.x % a.qtiles;
  const uint32_t bh = blockIdx.x / a.qtiles;
  const int32_t hh = static_cast<int32_t>(bh % a.H), bb = static_cast<int32_t>(bh / a.H);
  const int32_t q0 = static_cast<int32_t>(qt * BMQ);

  if (threadIdx.x == 0) {
    ptx::mbar_init(bar_qk, 1);
    ptx::mbar_init(bar_v, 1);
    ptx::mbar_init(bar_s, 1);
    ptx::mbar_init(bar_o, 1);
    for (uint32_t c = 0; c < nkb; ++c) ptx::mbar_init(&bar_p[c], 4 * 32);
    *abort_flag = 0;
    ptx::fence_barrier_init();
    ptx::prefetch_tensormap(&maps.q);
    ptx::prefetch_tensormap(&maps.k);
    ptx::prefetch_tensormap(&maps.v);
    ptx::prefetch_tensormap(&maps.p);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem, tmem_o = tmem + 256;
  pdl_enter();

  auto timeout = [&]() {
    *abort_flag = 1;
    raise_flag(a.status, TL_FLAG_TIMEOUT);
  };

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t kbytes = a.nk * 128;
      ptx::mbar_arrive_expect_tx(bar_qk, 2 * BMQ * 128 + 2 * kbytes);
      for (int kb = 0; kb < 2; ++kb) {
        const int32_t cq[4] = {32 * kb, q0, hh, bb};
        ptx::tma_load_rank(smem + kQ + kb * BMQ * 128, &maps.q, bar_qk, 4, cq);
        const int32_t ck[4] = {32 * kb, 0, hh, bb};
        ptx::tma_load_rank(smem + kK + kb * kbytes, &maps.k, bar_qk, 4, ck);
      }
      ptx::mbar_arrive_expect_tx(bar_v, 2 * kbytes);
      const int32_t cv[5] = {0, 0, 0, hh, bb};
      ptx::tma_load_rank(smem + kV, &maps.v, bar_v, 5, cv);
      // the loads must land before the CTA may exit
      if (!ptx::mbar_wait_bounded(bar_qk, 0, kWaitLimitNs) ||
          !ptx::mbar_wait_bounded(bar_v, 0, kWaitLimitNs))
        timeout();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool issued = false;
      const uint32_t sq = ptx::smem_addr(smem + kQ), sk = ptx::smem_addr(smem + kK);
      const uint32_t sv = ptx::smem_addr(smem + kV), sp = ptx::smem_addr(smem + kP);
      if (ptx::mbar_wait_bounded(bar_qk, 0, kWaitLimitNs)) {
        ptx::tc_fence_after();
        const uint32_t idesc_s = ptx::idesc_tf32(BMQ, a.nk, false, false);
#pragma unroll
        for (uint32_t kb = 0; kb < 2; ++kb)
#pragma unroll
          for (uint32_t kk = 0; kk < 4; ++kk)
            ptx::mma_tf32(tmem_s,
                          ptx::smem_desc(sq + kb * BMQ * 128 + kk * 32, 16, 1024,
                                         ptx::kSwizzle128B),
                          ptx::smem_desc(sk + kb * a.nk * 128 + kk * 32, 16, 1024,
                                         ptx::kSwizzle128B),
                          idesc_s, (kb | kk) ? 1u : 0u);
        issued = true;
        ptx::mma_commit(bar_s);
        bool ok = ptx::mbar_wait_bounded(bar_v, 0, kWaitLimitNs);
        const uint32_t idesc_o = ptx::idesc_tf32(BMQ, HD, false, true);
        for (uint32_t c = 0; c < nkb && ok; ++c) {
          if (!ptx::mbar_wait_bounded(&bar_p[c], 0, kWaitLimitNs)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
#pragma unroll
          for (uint32_t kk = 0; kk < 4; ++kk)
            ptx::mma_tf32(tmem_o,
                          ptx::smem_desc(sp + c * BMQ * 128 + kk * 32, 16, 1024,
                                         ptx::kSwizzle128B),
                          ptx::smem_desc(sv + (c * 32 + kk * 8) * 128, a.nk * 128, 512,
                                         ptx::kSwizzle128B32BAtom),
                          idesc_o, (c | kk) ? 1u : 0u);
        }
        if (!ok) timeout();
        ptx::mma_commit(bar_o);
      } else {
        timeout();
      }
      // what was issued has finished before TMEM is released
      if (issued) ptx::mbar_wait_bounded(bar_o, 0, kWaitLimitNs);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int e = warp - 2;
    const uint32_t q = warp & 3, half = e >> 2;
    const uint32_t row = q * 32 + lane;
    const uint32_t grow = qt * BMQ + row;
    const bool row_ok = grow < a.T;
    const float dv = *a.divisor;
    const float *mrow = (a.mask && row_ok) ? a.mask + static_cast<size_t>(grow) * a.T : nullptr;
    const uint32_t lane_base = (q * 32u) << 16;
    bool ok = ptx::mbar_wait_bounded(bar_s, 0, kWaitLimitNs);
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0) timeout();
      ok = false;
    }
    float m = -INFINITY, s = 0.0f;
    if (ok) {
      ptx::tc_fence_after();
      for (uint32_t c = half; c < nkb; c += 2) {
        uint32_t r[32];
        ptx::tmem_load_32x32b_x32(tmem_s + lane_base + c * 32, r);
        ptx::tmem_load_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const uint32_t col = c * 32 + j;
          if (col < a.T) {
            float x = __uint_as_float(r[j]) / dv;
            if (mrow) x = x + mrow[col];
            online_add(m, s, x);
          }
        }
      }
      red[half * BMQ + row] = make_float2(m, s);
    }
    ptx::named_bar_sync(1, 32 * kSoftWarps);
    if (ok) {
      const float2 o2 = red[(half ^ 1) * BMQ + row];
      online_merge(m, s, o2.x, o2.y);
      for (uint32_t c = half; c < nkb; c += 2) {
        uint32_t r[32];
        ptx::tmem_load_32x32b_x32(tmem_s + lane_base + c * 32, r);
        ptx::tmem_load_wait();
        uint8_t *blk = smem + kP + c * BMQ * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float p4[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t col = c * 32 + 4 * j + i;
            float x = __uint_as_float(r[4 * j + i]) / dv;
            if (mrow && col < a.T) x = x + mrow[col];
            p4[i] = col < a.T ? expf(x - m) / s : 0.0f;
          }
          *reinterpret_cast<float4 *>(blk + swz(row, j)) = make_float4(p4[0], p4[1], p4[2], p4[3]);
        }
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(&bar_p[c]);
      }
    }
    // P to global: every block is complete once all softmax warps are here
    ptx::named_bar_sync(1, 32 * kSoftWarps);
    if (ok && e == 0 && lane == 0) {
      for (uint32_t c = 0; c < nkb; ++c)
        ptx::tma_store_3d(&maps.p, smem + kP + c * BMQ * 128, static_cast<int32_t>(c * 32), q0,
                          static_cast<int32_t>(bh));
      ptx::bulk_commit_group();
    }
    // O = P V: TMEM -> global, each warp of a pair 32 of the 64 columns
    ok = ok && ptx::mbar_wait_bounded(bar_o, 0, kWaitLimitNs);
    if (__all_sync(0xffffffffu, ok) && !*abort_flag) {
      ptx::tc_fence_after();
      uint32_t r[32];
      ptx::tmem_load_32x32b_x32(tmem_o + lane_base + half * 32, r);
      ptx::tmem_load_wait();
      if (row_ok) {
        float4 *dst = reinterpret_cast<float4 *>(a.o + bb * a.sb + hh * a.sh +
                                                 static_cast<uint64_t>(grow) * a.ld + half * 32);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                               __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
      }
    } else if (lane == 0 && !ok) {
      timeout();
    }
    if (e == 0 && lane == 0) ptx::bulk_wait_group<0>();
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------ backward
// Query side, one CTA per (batch, head, 128 query rows), 320 threads:
//   warp 0      TMA: dO and V (K-major), this tile's rows of P (K-major,
//               as the forward stored them), K (MN-major)
//   warp 1      dP = dO V^T into TMEM, then dQ = dS K block by block
//   warps 2..9  softmax derivative (include/passes/execute.h:291-308):
//               pass 1 rowsum(dP * P), merged across the warp pair; pass 2
//               dS = P * (dP - rowsum) / divisor written over P in shared
//               memory (the dQ MMA's A operand and the TMA box of the dS
//               store); then dQ from TMEM to global.
struct BwdQMaps {
  CUtensorMap d_o, v, k, p, ds;
};

struct BwdQArgs {
  uint32_t T, H, nk, qtiles;
  const float *divisor;
  float *dq;
  uint64_t sb, sh, ld;
  uint32_t *status;
};

__global__ void __launch_bounds__(kThreads, 1)
attn_bwd_q_kernel(const __grid_constant__ BwdQMaps maps, const BwdQArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  // same footprint as the forward: dO in Q's place, V in K's, K in V's,
  // P / dS in P's
  uint8_t *s_do = smem + kQ, *s_v = smem + kK, *s_k = smem + kV, *s_p = smem + kP;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kBars);
  uint64_t *bar_a = bars, *bar_k = bars + 1, *bar_pl = bars + 2, *bar_dp = bars + 3,
           *bar_dq = bars + 4;
  uint64_t *bar_ds = bars + 5;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar_ds + kMaxFusedKeys / 32);
  volatile uint32_t *abort_flag = tmem_slot + 1;
  // row sums of each half, exchanged after pass 1 (dO is dead by then)
  float2 *red_sm = reinterpret_cast<float2 *>(s_do);

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const uint32_t nkb = a.nk / 32;
  const uint32_t qt = blockIdx.x % a.qtiles;
  const uint32_t bh = blockIdx.x / a.qtiles;
  const int32_t hh = static_cast<int32_t>(bh % a.H), bb = static_cast<int32_t>(bh / a.H);
  const int32_t q0 = static_cast<int32_t>(qt * BMQ);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 5; ++i) ptx::mbar_init(&bars[i], 1);
    for (uint32_t c = 0; c < nkb; ++c) ptx::mbar_init(&bar_ds[c], 4 * 32);
    *abort_flag = 0;
    ptx::fence_barrier_init();
    ptx::prefetch_tensormap(&maps.d_o);
    ptx::prefetch_tensormap(&maps.v);
    ptx::prefetch_tensormap(&maps.k);
    ptx::prefetch_tensormap(&maps.p);
    ptx::prefetch_tensormap(&maps.ds);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_dp = tmem, tmem_dq = tmem + 256;
  pdl_enter();

  auto timeout = [&]() {
    *abort_flag = 1;
    raise_flag(a.status, TL_FLAG_TIMEOUT);
  };

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t kbytes = a.nk * 128;
      ptx::mbar_arrive_expect_tx(bar_a, 2 * BMQ * 128 + 2 * kbytes);
      for (int kb = 0; kb < 2; ++kb) {
        const int32_t cd[4] = {32 * kb, q0, hh, bb};
        ptx::tma_load_rank(s_do + kb * BMQ * 128, &maps.d_o, bar_a, 4, cd);
        const int32_t cv[4] = {32 * kb, 0, hh, bb};
        ptx::tma_load_rank(s_v + kb * kbytes, &maps.v, bar_a, 4, cv);
      }
      ptx::mbar_arrive_expect_tx(bar_pl, nkb * BMQ * 128);
      for (uint32_t c = 0; c < nkb; ++c)
        ptx::tma_load_3d(s_p + c * BMQ * 128, &maps.p, bar_pl, static_cast<int32_t>(c * 32), q0,
                         static_cast<int32_t>(bh));
      ptx::mbar_arrive_expect_tx(bar_k, 2 * kbytes);
      const int32_t ck[5] = {0, 0, 0, hh, bb};
      ptx::tma_load_rank(s_k, &maps.k, bar_k, 5, ck);
      if (!ptx::mbar_wait_bounded(bar_a, 0, kWaitLimitNs) ||
          !ptx::mbar_wait_bounded(bar_pl, 0, kWaitLimitNs) ||
          !ptx::mbar_wait_bounded(bar_k, 0, kWaitLimitNs))
        timeout();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool issued = false;
      const uint32_t sdo = ptx::smem_addr(s_do), sv = ptx::smem_addr(s_v);
      const uint32_t sk = ptx::smem_addr(s_k), sp = ptx::smem_addr(s_p);
      if (ptx::mbar_wait_bounded(bar_a, 0, kWaitLimitNs)) {
        ptx::tc_fence_after();
        const uint32_t idesc_p = ptx::idesc_tf32(BMQ, a.nk, false, false);
#pragma unroll
        for (uint32_t kb = 0; kb < 2; ++kb)
#pragma unroll
          for (uint32_t kk = 0; kk < 4; ++kk)
            ptx::mma_tf32(tmem_dp,
                          ptx::smem_desc(sdo + kb * BMQ * 128 + kk * 32, 16, 1024,
                                         ptx::kSwizzle128B),
                          ptx::smem_desc(sv + kb * a.nk * 128 + kk * 32, 16, 1024,
                                         ptx::kSwizzle128B),
                          idesc_p, (kb | kk) ? 1u : 0u);
        issued = true;
        ptx::mma_commit(bar_dp);
        bool ok = ptx::mbar_wait_bounded(bar_k, 0, kWaitLimitNs);
        const uint32_t idesc_q = ptx::idesc_tf32(BMQ, HD, false, true);
        for (uint32_t c = 0; c < nkb && ok; ++c) {
          if (!ptx::mbar_wait_bounded(&bar_ds[c], 0, kWaitLimitNs)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
#pragma unroll
          for (uint32_t kk = 0; kk < 4; ++kk)
            ptx::mma_tf32(tmem_dq,
                          ptx::smem_desc(sp + c * BMQ * 128 + kk * 32, 16, 1024,
                                         ptx::kSwizzle128B),
                          ptx::smem_desc(sk + (c * 32 + kk * 8) * 128, a.nk * 128, 512,
                                         ptx::kSwizzle128B32BAtom),
                          idesc_q, (c | kk) ? 1u : 0u);
        }
        if (!ok) timeout();
        ptx::mma_commit(bar_dq);
      } else {
        timeout();
      }
      if (issued) ptx::mbar_wait_bounded(bar_dq, 0, kWaitLimitNs);
    }
  } else {
    const int e = warp - 2;
    const uint32_t q = warp & 3, half = e >> 2;
    const uint32_t row = q * 32 + lane;
    const uint32_t grow = qt * BMQ + row;
    const float dv = *a.divisor;
    const uint32_t lane_base = (q * 32u) << 16;
    bool ok = ptx::mbar_wait_bounded(bar_dp, 0, kWaitLimitNs) &&
              ptx::mbar_wait_bounded(bar_pl, 0, kWaitLimitNs);
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0) timeout();
      ok = false;
    }
    float sum = 0.0f;
    if (ok) {
      ptx::tc_fence_after();
      for (uint32_t c = half; c < nkb; c += 2) {
        uint32_t r[32];
        ptx::tmem_load_32x32b_x32(tmem_dp + lane_base + c * 32, r);
        ptx::tmem_load_wait();
        const uint8_t *blk = s_p + c * BMQ * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 p4 = *reinterpret_cast<const float4 *>(blk + swz(row, j));
          sum += __uint_as_float(r[4 * j]) * p4.x;
          sum += __uint_as_float(r[4 * j + 1]) * p4.y;
          sum += __uint_as_float(r[4 * j + 2]) * p4.z;
          sum += __uint_as_float(r[4 * j + 3]) * p4.w;
        }
      }
      red_sm[half * BMQ + row] = make_float2(sum, 0.0f);
    }
    ptx::named_bar_sync(1, 32 * kSoftWarps);
    if (ok) {
      // both halves add in the same order: low columns first
      const float lo = red_sm[row].x, hi = red_sm[BMQ + row].x;
      sum = lo + hi;
      for (uint32_t c = half; c < nkb; c += 2) {
        uint32_t r[32];
        ptx::tmem_load_32x32b_x32(tmem_dp + lane_base + c * 32, r);
        ptx::tmem_load_wait();
        uint8_t *blk = s_p + c * BMQ * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float4 *slot = reinterpret_cast<float4 *>(blk + swz(row, j));
          const float4 p4 = *slot;
          *slot = make_float4(p4.x * (__uint_as_float(r[4 * j]) - sum) / dv,
                              p4.y * (__uint_as_float(r[4 * j + 1]) - sum) / dv,
                              p4.z * (__uint_as_float(r[4 * j + 2]) - sum) / dv,
                              p4.w * (__uint_as_float(r[4 * j + 3]) - sum) / dv);
        }
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(&bar_ds[c]);
      }
    }
    ptx::named_bar_sync(1, 32 * kSoftWarps);
    if (ok && e == 0 && lane == 0) {
      for (uint32_t c = 0; c < nkb; ++c)
        ptx::tma_store_3d(&maps.ds, s_p + c * BMQ * 128, static_cast<int32_t>(c * 32), q0,
                          static_cast<int32_t>(bh));
      ptx::bulk_commit_group();
    }
    ok = ok && ptx::mbar_wait_bounded(bar_dq, 0, kWaitLimitNs);
    if (__all_sync(0xffffffffu, ok) && !*abort_flag) {
      ptx::tc_fence_after();
      uint32_t r[32];
      ptx::tmem_load_32x32b_x32(tmem_dq + lane_base + half * 32, r);
      ptx::tmem_load_wait();
      if (grow < a.T) {
        float4 *dst = reinterpret_cast<float4 *>(a.dq + bb * a.sb + hh * a.sh +
                                                 static_cast<uint64_t>(grow) * a.ld + half * 32);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                               __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
      }
    } else if (lane == 0 && !ok) {
      timeout();
    }
    if (e == 0 && lane == 0) ptx::bulk_wait_group<0>();
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem, 512);
}

// Key side, one CTA per (batch, head, 128 keys), 192 threads:
//   warp 0      TMA ring over 32-query blocks: dS^T and P^T (MN-major, from
//               the [T, T] matrices), Q and dO (MN-major)
//   warp 1      dK += dS^T Q and dV += P^T dO into TMEM (64 columns each)
//   warps 2..5  dK, dV from TMEM to global
constexpr int kKvThreads = 64 + 128;
constexpr int kKvStages = 4;
constexpr uint32_t kKvA = 128 * 32 * 4;  // 128 keys x 32 queries
constexpr uint32_t kKvB = 32 * HD * 4;   // 32 queries x 64
constexpr uint32_t kKvStage = 2 * kKvA + 2 * kKvB;
constexpr size_t kKvSmem = 1024 + kKvStages * kKvStage + 256;

struct BwdKvMaps {
  CUtensorMap ds, p, q, d_o;
};

struct BwdKvArgs {
  uint32_t T, H, ktiles, qblocks;
  float *dk, *dv;
  uint64_t sb, sh, ld;
  uint32_t *status;
};

__global__ void __launch_bounds__(kKvThreads, 1)
attn_bwd_kv_kernel(const __grid_constant__ BwdKvMaps maps, const BwdKvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kKvStages * kKvStage);
  uint64_t *empty = full + kKvStages;
  uint64_t *done = empty + kKvStages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  volatile uint32_t *abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const uint32_t kt = blockIdx.x % a.ktiles;
  const uint32_t bh = blockIdx.x / a.ktiles;
  const int32_t hh = static_cast<int32_t>(bh % a.H), bb = static_cast<int32_t>(bh / a.H);
  const int32_t k0 = static_cast<int32_t>(kt * 128);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kKvStages; ++i) {
      ptx::mbar_init(&full[i], 1);
      ptx::mbar_init(&empty[i], 1);
    }
    ptx::mbar_init(done, 1);
    *abort_flag = 0;
    ptx::fence_barrier_init();
    ptx::prefetch_tensormap(&maps.ds);
    ptx::prefetch_tensormap(&maps.p);
    ptx::prefetch_tensormap(&maps.q);
    ptx::prefetch_tensormap(&maps.d_o);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, 128);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_enter();

  auto timeout = [&]() {
    *abort_flag = 1;
    raise_flag(a.status, TL_FLAG_TIMEOUT);
  };

  if (warp == 0) {
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0;
      for (uint32_t qb = 0; qb < a.qblocks; ++qb) {
        if (!ptx::mbar_wait_bounded(&empty[stage], phase ^ 1, kWaitLimitNs)) {
          timeout();
          break;
        }
        uint8_t *st = smem + stage * kKvStage;
        ptx::mbar_arrive_expect_tx(&full[stage], kKvStage);
        const int32_t y = static_cast<int32_t>(qb * 32);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          ptx::tma_load_3d(st + j * 4096, &maps.ds, &full[stage], k0 + 32 * j, y,
                           static_cast<int32_t>(bh));
          ptx::tma_load_3d(st + kKvA + j * 4096, &maps.p, &full[stage], k0 + 32 * j, y,
                           static_cast<int32_t>(bh));
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int32_t c[4] = {32 * j, y, hh, bb};
          ptx::tma_load_rank(st + 2 * kKvA + j * 4096, &maps.q, &full[stage], 4, c);
          ptx::tma_load_rank(st + 2 * kKvA + kKvB + j * 4096, &maps.d_o, &full[stage], 4, c);
        }
        ++issued;
        if (++stage == kKvStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      // every issued stage has landed before the CTA may exit
      uint32_t back = issued < kKvStages ? issued : kKvStages;
      uint32_t s = stage, p = phase;
      for (uint32_t i = 0; i < back; ++i) {
        if (s == 0) {
          s = kKvStages - 1;
          p ^= 1;
        } else {
          --s;
        }
        if (!ptx::mbar_wait_bounded(&full[s], p, kWaitLimitNs)) {
          timeout();
          break;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = ptx::idesc_tf32(128, HD, true, true);
      uint32_t stage = 0, phase = 0;
      bool issued = false;
      for (uint32_t qb = 0; qb < a.qblocks && !*abort_flag; ++qb) {
        if (!ptx::mbar_wait_bounded(&full[stage], phase, kWaitLimitNs)) {
          timeout();
          break;
        }
        ptx::tc_fence_after();
        const uint32_t st = ptx::smem_addr(smem + stage * kKvStage);
#pragma unroll
        for (uint32_t kk = 0; kk < 4; ++kk) {
          const uint32_t acc = (qb | kk) ? 1u : 0u;
          ptx::mma_tf32(tmem,
                        ptx::smem_desc(st + kk * 1024, 4096, 512, ptx::kSwizzle128B32BAtom),
                        ptx::smem_desc(st + 2 * kKvA + kk * 1024, 4096, 512,
                                       ptx::kSwizzle128B32BAtom),
                        idesc, acc);
          ptx::mma_tf32(tmem + HD,
                        ptx::smem_desc(st + kKvA + kk * 1024, 4096, 512,
                                       ptx::kSwizzle128B32BAtom),
                        ptx::smem_desc(st + 2 * kKvA + kKvB + kk * 1024, 4096, 512,
                                       ptx::kSwizzle128B32BAtom),
                        idesc, acc);
        }
        issued = true;
        ptx::mma_commit(&empty[stage]);
        if (++stage == kKvStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (issued) {
        ptx::mma_commit(done);
        if (!ptx::mbar_wait_bounded(done, 0, kWaitLimitNs)) timeout();
      } else {
        ptx::mbar_arrive(done);  // nothing to wait for: release the epilogue
      }
    }
  } else {
    const uint32_t q = warp & 3;
    const uint32_t key = kt * 128 + q * 32 + lane;
    const bool ok = ptx::mbar_wait_bounded(done, 0, kWaitLimitNs);
    if (__all_sync(0xffffffffu, ok) && !*abort_flag) {
      ptx::tc_fence_after();
      const uint32_t lane_base = (q * 32u) << 16;
      const uint64_t off = bb * a.sb + hh * a.sh + static_cast<uint64_t>(key) * a.ld;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        ptx::tmem_load_32x32b_x32(tmem + lane_base + c * 32, r);
        ptx::tmem_load_wait();
        if (key < a.T) {
          float *base = (c < 2 ? a.dk : a.dv) + off + (c & 1) * 32;
          float4 *dst = reinterpret_cast<float4 *>(base);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                 __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
        }
      }
    } else if (lane == 0 && !ok) {
      timeout();
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem, 128);
}

bool encode(CUtensorMap *map, const float *base, int rank, const cuuint64_t *dims,
            const cuuint64_t *strides_bytes, const cuuint32_t *box, CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, static_cast<cuuint32_t>(rank),
             const_cast<float *>(base), dims, strides_bytes, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [D, T, H, B] view of a head-strided operand, box 32 x rows.
bool head_map(CUtensorMap *map, const float *base, const FusedAttnShape &sh, uint32_t rows) {
  const cuuint64_t dims[4] = {HD, sh.T, sh.H, sh.B};
  const cuuint64_t st[3] = {sh.ld * 4, sh.sh * 4, sh.sb * 4};
  const cuuint32_t box[4] = {32, rows, 1, 1};
  return encode(map, base, 4, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// [32, T, D / 32, H, B] view (the MN-major operand layout: 32-wide column
// chunks of rows), box 32 x rows x D / 32.
bool head_map_mn(CUtensorMap *map, const float *base, const FusedAttnShape &sh, uint32_t rows) {
  const cuuint64_t dims[5] = {32, sh.T, HD / 32, sh.H, sh.B};
  const cuuint64_t st[4] = {sh.ld * 4, 128, sh.sh * 4, sh.sb * 4};
  const cuuint32_t box[5] = {32, rows, HD / 32, 1, 1};
  return encode(map, base, 5, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
}

// [T, T, B * H] view of P (or dS), box 32 x rows: K-major rows of 128
// queries, or (32-byte-atom swizzle) MN-major 32 x 32 blocks.
bool scores_map(CUtensorMap *map, const float *base, const FusedAttnShape &sh,
                uint32_t rows = BMQ, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  const cuuint64_t dims[3] = {sh.T, sh.T, static_cast<cuuint64_t>(sh.B) * sh.H};
  const cuuint64_t st[2] = {static_cast<cuuint64_t>(sh.T) * 4,
                            static_cast<cuuint64_t>(sh.T) * sh.T * 4};
  const cuuint32_t box[3] = {32, rows, 1};
  return encode(map, base, 3, dims, st, box, swz);
}

// [D, T, H, B] view with 32 x 32 boxes in the MN-major layout.
bool head_map_mn32(CUtensorMap *map, const float *base, const FusedAttnShape &sh) {
  const cuuint64_t dims[4] = {HD, sh.T, sh.H, sh.B};
  const cuuint64_t st[3] = {sh.ld * 4, sh.sh * 4, sh.sb * 4};
  const cuuint32_t box[4] = {32, 32, 1, 1};
  return encode(map, base, 4, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
}

template <typename K>
int set_smem(K kernel, size_t bytes, bool &done, const char *what) {
  if (done) return TL_OK;
  int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(bytes)),
                      what);
  if (rc == TL_OK) done = true;
  return rc;
}

}  // namespace

bool fused_attention_supported(const FusedAttnShape &sh, const void *const *ptrs, int n) {
  if (sh.D != HD || sh.T == 0 || sh.T > kMaxFusedKeys || sh.T % 4 != 0) return false;
  if (sh.ld % 4 || sh.sh % 4 || sh.sb % 4) return false;
  if (static_cast<uint64_t>(sh.B) * sh.H * ((sh.T + BMQ - 1) / BMQ) > 0x7fffffffu) return false;
  for (int i = 0; i < n; ++i)
    if (ptrs[i] && !aligned16(ptrs[i])) return false;
  return tensor_map_encoder() != nullptr;
}

int launch_attention_fwd_tc(const float *q, const float *k, const float *v, const float *divisor,
                            const float *mask, float *p, float *o, const FusedAttnShape &sh,
                            cudaStream_t s) {
  FwdMaps maps{};
  FwdArgs a{};
  a.T = sh.T;
  a.H = sh.H;
  a.nk = (sh.T + 31) / 32 * 32;
  a.qtiles = (sh.T + BMQ - 1) / BMQ;
  a.divisor = divisor;
  a.mask = mask;
  a.o = o;
  a.sb = sh.sb;
  a.sh = sh.sh;
  a.ld = sh.ld;
  a.status = device_status_ptr();
  if (!a.status) return fail(TL_ERR_CUDA, "tl_attention_fwd: no status word");
  if (!head_map(&maps.q, q, sh, BMQ) || !head_map(&maps.k, k, sh, a.nk) ||
      !head_map_mn(&maps.v, v, sh, a.nk) || !scores_map(&maps.p, p, sh))
    return fail(TL_ERR_UNSUPPORTED, "tl_attention_fwd: tensor maps refused");
  static bool attr = false;
  int rc = set_smem(attn_fwd_kernel, kFwdSmem, attr, "tl_attention_fwd: shared memory");
  if (rc) return rc;
  const unsigned grid = static_cast<unsigned>(static_cast<uint64_t>(sh.B) * sh.H * a.qtiles);
  launch_pdl(attn_fwd_kernel, grid, kThreads, kFwdSmem, s, maps, a);
  return launch_status("tl_attention_fwd");
}

int launch_attention_bwd_tc(const float *q, const float *k, const float *v, const float *p,
                            const float *divisor, const float *d_o, float *dq, float *dk,
                            float *dv, float *ds, const FusedAttnShape &sh, cudaStream_t s) {
  uint32_t *status = device_status_ptr();
  if (!status) return fail(TL_ERR_CUDA, "tl_attention_bwd: no status word");
  const uint32_t nk = (sh.T + 31) / 32 * 32;
  BwdQMaps qm{};
  BwdQArgs qa{};
  qa.T = sh.T;
  qa.H = sh.H;
  qa.nk = nk;
  qa.qtiles = (sh.T + BMQ - 1) / BMQ;
  qa.divisor = divisor;
  qa.dq = dq;
  qa.sb = sh.sb;
  qa.sh = sh.sh;
  qa.ld = sh.ld;
  qa.status = status;
  BwdKvMaps km{};
  BwdKvArgs ka{};
  ka.T = sh.T;
  ka.H = sh.H;
  ka.ktiles = (sh.T + 127) / 128;
  ka.qblocks = (sh.T + 31) / 32;
  ka.dk = dk;
  ka.dv = dv;
  ka.sb = sh.sb;
  ka.sh = sh.sh;
  ka.ld = sh.ld;
  ka.status = status;
  if (!head_map(&qm.d_o, d_o, sh, BMQ) || !head_map(&qm.v, v, sh, nk) ||
      !head_map_mn(&qm.k, k, sh, nk) || !scores_map(&qm.p, p, sh) ||
      !scores_map(&qm.ds, ds, sh) ||
      !scores_map(&km.ds, ds, sh, 32, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B) ||
      !scores_map(&km.p, p, sh, 32, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B) ||
      !head_map_mn32(&km.q, q, sh) || !head_map_mn32(&km.d_o, d_o, sh))
    return fail(TL_ERR_UNSUPPORTED, "tl_attention_bwd: tensor maps refused");
  static bool attr_q = false, attr_kv = false;
  int rc = set_smem(attn_bwd_q_kernel, kFwdSmem, attr_q, "tl_attention_bwd: shared memory");
  if (rc == TL_OK)
    rc = set_smem(attn_bwd_kv_kernel, kKvSmem, attr_kv, "tl_attention_bwd: shared memory");
  if (rc) return rc;
  const uint64_t bhn = static_cast<uint64_t>(sh.B) * sh.H;
  launch_pdl(attn_bwd_q_kernel, static_cast<unsigned>(bhn * qa.qtiles), kThreads, kFwdSmem, s,
             qm, qa);
  rc = launch_status("tl_attention_bwd (dQ)");
  if (rc) return rc;
  launch_pdl(attn_bwd_kv_kernel, static_cast<unsigned>(bhn * ka.ktiles), kKvThreads, kKvSmem, s,
             km, ka);
  return launch_status("tl_attention_bwd (dK, dV)");
}

}  // namespace tl

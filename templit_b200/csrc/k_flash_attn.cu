// Flash attention on the tensor cores for 64-wide heads and any sequence
// length: the executor's attention composite (include/nn/multi_head.h:45-52,
// S = Q K^T / divisor + mask, P = softmax(S), O = P V) and its backward (the
// product rules and SFTMX_DERIVATIVE, include/passes/execute.h:187-232,
// 291-308) without any T x T tensor in HBM.
//
// Forward, one CTA per (batch, head, 128 query rows), 192 threads:
//   warp 0     TMA: the Q tile, then 64-key blocks of K and V (3-stage rings)
//   warp 1     TMEM owner, MMA issuer: S_j = Q K_j^T into one of two TMEM
//              score buffers; once the softmax hands P_j over in shared
//              memory, O_j = P_j V_j into one of two TMEM output buffers
//   warps 2-5  softmax, one query row per thread (TMEM lane quadrant =
//              warp % 4): online max and sum over the key blocks in log2
//              units, P_j = 2^(x - m) into shared memory, and the running
//              output O = O * 2^(m_old - m_new) + O_j in registers (O_j of
//              block j is merged while the MMAs of block j + 1 run)
// and leaves O and the row log-sum-exp L = ln sum_k e^{S_k} ([B, H, T]);
// P is never stored.
//
// Backward, from Q, K, V, dO, L and Delta = rowsum(dO * O) (= rowsum(dP * P)
// of the reference's softmax derivative), P recomputed as e^(S - L):
//   query side, one CTA per (batch, head, 128 queries): S_j = Q K_j^T and
//     dP_j = dO V_j^T into TMEM, dS_j = P_j (dP_j - Delta) / divisor into
//     shared memory, dQ += dS_j K_j in TMEM;
//   key side, one CTA per (batch, head, 128 keys): S^T = K Q_i^T and
//     dP^T = V dO_i^T over 64-query blocks, P^T and dS^T into shared memory,
//     dV += P^T dO_i and dK += dS^T Q_i in TMEM.
// Both are deterministic (no atomics).  A causal mask (nn::causal_mask,
// include/nn/attention.h:10-22) is applied by position and the blocks it
// zeroes are skipped; any other additive [T, T] mask is read per score.
//
// Products are TF32 (tcgen05.mma kind::tf32, fp32 accumulation in TMEM),
// the softmax is fp32.  Every mbarrier wait is bounded (2 s): on timeout
// the CTA raises TL_FLAG_TIMEOUT, lets what it issued finish and returns.
#include "attn_maps.cuh"
#include "attention_tc.h"
#include "tc_ptx.cuh"

#include <cuda.h>

namespace tl {
namespace {

constexpr uint32_t HD = kFusedHeadDim;  // 64
constexpr uint32_t BMQ = 128;           // rows of a CTA tile (queries or keys)
constexpr uint32_t BNK = 64;            // keys (or queries) per inner block
constexpr int kThreads = 192;           // TMA warp, MMA warp, four softmax warps
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

constexpr uint32_t kTile128 = BMQ * HD * 4;  // 32 KB: 128 rows x 64, two 16 KB blocks
constexpr uint32_t kTile64 = BNK * HD * 4;   // 16 KB: 64 rows x 64, two 8 KB blocks
constexpr uint32_t kScore = BMQ * BNK * 4;   // 32 KB: 128 x 64 scores, two 16 KB blocks

__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t j) {
  return r * 128u + ((j ^ (r & 7u)) << 4);
}

__device__ __forceinline__ uint8_t *align1024(uint8_t *p) {
  return reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(p) + 1023) &
                                     ~static_cast<uintptr_t>(1023));
}

// Descriptors of the operand layouts (see the GEMM): K-major blocks
// [K / 32][rows][32] with 128-byte swizzle; MN-major chunks [MN / 32][K
// rows][32] with 32-byte atoms.  k-step kk (8 of K) of block kb.
__device__ __forceinline__ uint64_t kmaj(uint32_t base, uint32_t rows, uint32_t kb, uint32_t kk) {
  return ptx::smem_desc(base + kb * rows * 128 + kk * 32, 16, 1024, ptx::kSwizzle128B);
}
__device__ __forceinline__ uint64_t mnmaj(uint32_t base, uint32_t krows, uint32_t kb,
                                          uint32_t kk) {
  return ptx::smem_desc(base + (kb * 32 + kk * 8) * 128, krows * 128, 512,
                        ptx::kSwizzle128B32BAtom);
}

// 64 columns of this thread's TMEM lane, as floats.
__device__ __forceinline__ void tmem_row64(uint32_t taddr, float (&x)[64]) {
  uint32_t r[32];
  ptx::tmem_load_32x32b_x32(taddr, r);
  ptx::tmem_load_wait();
#pragma unroll
  for (int i = 0; i < 32; ++i) x[i] = __uint_as_float(r[i]);
  ptx::tmem_load_32x32b_x32(taddr + 32, r);
  ptx::tmem_load_wait();
#pragma unroll
  for (int i = 0; i < 32; ++i) x[32 + i] = __uint_as_float(r[i]);
}

// Row `row` (0..127) of a 128 x 64 K-major score block (two 16 KB blocks of
// 32 columns) from 64 values.
__device__ __forceinline__ void put_row64(uint8_t *block, uint32_t row, const float (&v)[64]) {
#pragma unroll
  for (int kb = 0; kb < 2; ++kb)
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<float4 *>(block + kb * 16384 + swz(row, c)) =
          make_float4(v[kb * 32 + 4 * c], v[kb * 32 + 4 * c + 1], v[kb * 32 + 4 * c + 2],
                      v[kb * 32 + 4 * c + 3]);
}

struct View {
  float *p;
  uint64_t sb, sh, ld;
};

__device__ __forceinline__ float *row_ptr(const View &v, uint32_t b, uint32_t h, uint32_t t) {
  return v.p + b * v.sb + h * v.sh + static_cast<uint64_t>(t) * v.ld;
}

__device__ __forceinline__ void store_row64(const View &v, uint32_t b, uint32_t h, uint32_t t,
                                            const float (&x)[64], float scale) {
  float4 *dst = reinterpret_cast<float4 *>(row_ptr(v, b, h, t));
#pragma unroll
  for (int j = 0; j < 16; ++j)
    dst[j] = make_float4(x[4 * j] * scale, x[4 * j + 1] * scale, x[4 * j + 2] * scale,
                         x[4 * j + 3] * scale);
}

struct Maps {
  CUtensorMap a, b, c, d, e, f;
};

struct Args {
  uint32_t T, H, tiles;  // tiles per (batch, head)
  const float *divisor, *mask;
  const uint32_t *mask_flag;  // nonzero: the mask is the causal one
  float *lse, *delta;         // [B, H, T]
  View out0, out1;            // O (forward); dQ (query side); dK, dV (key side)
  uint32_t *status;
};

struct Ctx {
  uint32_t bh, b, h, tile0;
  bool causal, masked;
};

__device__ __forceinline__ Ctx context(const Args &a) {
  Ctx c;
  const uint32_t t = blockIdx.x % a.tiles;
  c.bh = blockIdx.x / a.tiles;
  c.h = c.bh % a.H;
  c.b = c.bh / a.H;
  c.tile0 = t * BMQ;
  c.masked = a.mask != nullptr;
  c.causal = c.masked && a.mask_flag && *a.mask_flag != 0;
  return c;
}

// Score of (query, key) in log2 units: s / divisor * log2(e) + mask *
// log2(e); -inf where the causal mask or the sequence end masks it.
__device__ __forceinline__ float score2(float s, float c, const Args &a, const Ctx &x,
                                        uint32_t query, uint32_t key) {
  if (key >= a.T || query >= a.T || (x.causal && key > query)) return -INFINITY;
  float v = s * c;
  if (x.masked && !x.causal) v += a.mask[static_cast<uint64_t>(query) * a.T + key] * kLog2e;
  return v;
}

// =================================================================== forward
constexpr int kFwdStages = 3;
constexpr uint32_t kFwdQ = 0;
constexpr uint32_t kFwdK = kFwdQ + kTile128;
constexpr uint32_t kFwdV = kFwdK + kFwdStages * kTile64;
constexpr uint32_t kFwdP = kFwdV + kFwdStages * kTile64;
constexpr uint32_t kFwdBars = kFwdP + 2 * kScore;
constexpr size_t kFwdSmem = 1024 + kFwdBars + 256;

template <bool KT>
__global__ void __launch_bounds__(kThreads, 1)
flash_fwd_kernel(const __grid_constant__ Maps maps, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kFwdBars);
  uint64_t *qfull = bars;
  uint64_t *kfull = bars + 1, *kempty = kfull + kFwdStages;
  uint64_t *vfull = kempty + kFwdStages, *vempty = vfull + kFwdStages;
  uint64_t *sfull = vempty + kFwdStages, *sfree = sfull + 2;
  uint64_t *pfull = sfree + 2, *ofull = pfull + 2, *ofree = ofull + 2, *drain = ofree + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile uint32_t *abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    ptx::mbar_init(qfull, 1);
    for (int i = 0; i < kFwdStages; ++i) {
      ptx::mbar_init(&kfull[i], 1);
      ptx::mbar_init(&kempty[i], 1);
      ptx::mbar_init(&vfull[i], 1);
      ptx::mbar_init(&vempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&sfull[i], 1);
      ptx::mbar_init(&sfree[i], 128);
      ptx::mbar_init(&pfull[i], 128);
      ptx::mbar_init(&ofull[i], 1);
      ptx::mbar_init(&ofree[i], 128);
    }
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_barrier_init();
    ptx::prefetch_tensormap(&maps.a);
    ptx::prefetch_tensormap(&maps.b);
    ptx::prefetch_tensormap(&maps.c);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, 256);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem, tmem_o = tmem + 128;  // two 64-column buffers each
  pdl_enter();
  const Ctx x = context(a);
  const uint32_t last_row = min(a.T, x.tile0 + BMQ);
  const uint32_t nkb = ((x.causal ? last_row : a.T) + BNK - 1) / BNK;
  auto timeout = [&]() {
    *abort_flag = 1;
    raise_flag(a.status, TL_FLAG_TIMEOUT);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ loads
    if (lane == 0) {
      const int32_t hh = static_cast<int32_t>(x.h), bb = static_cast<int32_t>(x.b);
      ptx::mbar_arrive_expect_tx(qfull, kTile128);
      for (int kb = 0; kb < 2; ++kb) {
        const int32_t c[4] = {32 * kb, static_cast<int32_t>(x.tile0), hh, bb};
        ptx::tma_load_rank(smem + kFwdQ + kb * 16384, &maps.a, qfull, 4, c);
      }
      uint32_t issued = 0;
      for (uint32_t j = 0; j < nkb && !*abort_flag; ++j) {
        const uint32_t s = j % kFwdStages, ph = (j / kFwdStages) & 1;
        const int32_t key0 = static_cast<int32_t>(j * BNK);
        if (!ptx::mbar_wait_bounded(&kempty[s], ph ^ 1, kWaitLimitNs)) {
          timeout();
          break;
        }
        ptx::mbar_arrive_expect_tx(&kfull[s], kTile64);
        uint8_t *sk = smem + kFwdK + s * kTile64;
        for (int c = 0; c < 2; ++c) {
          const int32_t cc[4] = {KT ? key0 + 32 * c : 32 * c, KT ? 0 : key0, hh, bb};
          ptx::tma_load_rank(sk + c * 8192, &maps.b, &kfull[s], 4, cc);
        }
        if (!ptx::mbar_wait_bounded(&vempty[s], ph ^ 1, kWaitLimitNs)) {
          timeout();
          break;
        }
        ptx::mbar_arrive_expect_tx(&vfull[s], kTile64);
        const int32_t cv[5] = {0, key0, 0, hh, bb};
        ptx::tma_load_rank(smem + kFwdV + s * kTile64, &maps.c, &vfull[s], 5, cv);
        ++issued;
      }
      // every issued load has landed before the CTA may exit
      if (!ptx::mbar_wait_bounded(qfull, 0, kWaitLimitNs)) timeout();
      for (uint32_t j = issued > kFwdStages ? issued - kFwdStages : 0; j < issued; ++j) {
        const uint32_t s = j % kFwdStages, ph = (j / kFwdStages) & 1;
        if (!ptx::mbar_wait_bounded(&kfull[s], ph, kWaitLimitNs) ||
            !ptx::mbar_wait_bounded(&vfull[s], ph, kWaitLimitNs)) {
          timeout();
          break;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMAs
    if (lane == 0) {
      const uint32_t sq = ptx::smem_addr(smem + kFwdQ);
      const uint32_t idesc_s = ptx::idesc_tf32(BMQ, BNK, false, KT);
      const uint32_t idesc_o = ptx::idesc_tf32(BMQ, HD, false, true);
      bool ok = ptx::mbar_wait_bounded(qfull, 0, kWaitLimitNs), issued = false;
      auto pv = [&](uint32_t i) {
        const uint32_t s = i % kFwdStages;
        if (!ptx::mbar_wait_bounded(&pfull[i & 1], (i >> 1) & 1, kWaitLimitNs) ||
            !ptx::mbar_wait_bounded(&vfull[s], (i / kFwdStages) & 1, kWaitLimitNs) ||
            (i >= 2 && !ptx::mbar_wait_bounded(&ofree[i & 1], ((i - 2) >> 1) & 1, kWaitLimitNs)))
          return false;
        ptx::tc_fence_after();
        const uint32_t sp = ptx::smem_addr(smem + kFwdP + (i & 1) * kScore);
        const uint32_t sv = ptx::smem_addr(smem + kFwdV + s * kTile64);
#pragma unroll
        for (uint32_t kb = 0; kb < 2; ++kb)
#pragma unroll
          for (uint32_t kk = 0; kk < 4; ++kk)
            ptx::mma_tf32(tmem_o + (i & 1) * HD, kmaj(sp, BMQ, kb, kk), mnmaj(sv, BNK, kb, kk),
                          idesc_o, (kb | kk) ? 1u : 0u);
        ptx::mma_commit(&ofull[i & 1]);
        ptx::mma_commit(&vempty[s]);
        return true;
      };
      for (uint32_t j = 0; j < nkb && ok; ++j) {
        const uint32_t s = j % kFwdStages;
        if (!ptx::mbar_wait_bounded(&kfull[s], (j / kFwdStages) & 1, kWaitLimitNs) ||
            (j >= 2 && !ptx::mbar_wait_bounded(&sfree[j & 1], ((j - 2) >> 1) & 1, kWaitLimitNs))) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t sk = ptx::smem_addr(smem + kFwdK + s * kTile64);
#pragma unroll
        for (uint32_t kb = 0; kb < 2; ++kb)
#pragma unroll
          for (uint32_t kk = 0; kk < 4; ++kk)
            ptx::mma_tf32(tmem_s + (j & 1) * BNK, kmaj(sq, BMQ, kb, kk),
                          KT ? mnmaj(sk, HD, kb, kk) : kmaj(sk, BNK, kb, kk), idesc_s,
                          (kb | kk) ? 1u : 0u);
        issued = true;
        ptx::mma_commit(&sfull[j & 1]);
        ptx::mma_commit(&kempty[s]);
        if (j >= 1 && !pv(j - 1)) ok = false;
      }
      if (ok && nkb > 0 && !pv(nkb - 1)) ok = false;
      if (!ok) {
        timeout();
        if (issued) {  // in-flight MMAs finish before TMEM is released
          ptx::mma_commit(drain);
          ptx::mbar_wait_bounded(drain, 0, kWaitLimitNs);
        }
      } else if (issued) {
        // the stage releases nobody waits for (the last kFwdStages K and V
        // stages): their arrivals must have landed before the CTA exits, or
        // they would reach the barriers of the next CTA in this shared memory
        ptx::mma_commit(drain);
        ok = ptx::mbar_wait_bounded(drain, 0, kWaitLimitNs);
        for (uint32_t j = nkb > kFwdStages ? nkb - kFwdStages : 0; ok && j < nkb; ++j)
          ok = ptx::mbar_wait_bounded(&kempty[j % kFwdStages], (j / kFwdStages) & 1,
                                      kWaitLimitNs) &&
               ptx::mbar_wait_bounded(&vempty[j % kFwdStages], (j / kFwdStages) & 1,
                                      kWaitLimitNs);
        if (!ok) timeout();
      }
    }
  } else {
    // ---------------------------------------------------------- softmax
    const uint32_t q = warp & 3;
    const uint32_t rloc = q * 32 + lane, row = x.tile0 + rloc;
    const uint32_t lane_base = (q * 32u) << 16;
    const float c = kLog2e / *a.divisor;
    float acc[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) acc[i] = 0.0f;
    float m = -INFINITY, l = 0.0f, alpha_pend = 1.0f;
    bool ok = true;
    auto merge = [&](uint32_t i, float alpha) {
      const bool got = ptx::mbar_wait_bounded(&ofull[i & 1], (i >> 1) & 1, kWaitLimitNs);
      if (!__all_sync(0xffffffffu, got)) return false;
      ptx::tc_fence_after();
      float o[64];
      tmem_row64(tmem_o + (i & 1) * HD + lane_base, o);
      ptx::tc_fence_before();
      ptx::mbar_arrive(&ofree[i & 1]);
#pragma unroll
      for (int k = 0; k < 64; ++k) acc[k] = acc[k] * alpha + o[k];
      return true;
    };
    for (uint32_t j = 0; j < nkb && ok; ++j) {
      const bool got = ptx::mbar_wait_bounded(&sfull[j & 1], (j >> 1) & 1, kWaitLimitNs);
      if (!__all_sync(0xffffffffu, got) || *abort_flag) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      float s[64];
      tmem_row64(tmem_s + (j & 1) * BNK + lane_base, s);
      ptx::tc_fence_before();
      ptx::mbar_arrive(&sfree[j & 1]);
      const uint32_t key0 = j * BNK;
      float mb = -INFINITY;
#pragma unroll
      for (int k = 0; k < 64; ++k) {
        s[k] = score2(s[k], c, a, x, row, key0 + k);
        mb = fmaxf(mb, s[k]);
      }
      const float m_new = fmaxf(m, mb);
      float alpha = 1.0f, sum = 0.0f;
      if (m_new == -INFINITY) {
#pragma unroll
        for (int k = 0; k < 64; ++k) s[k] = 0.0f;
      } else {
        alpha = ptx::ex2_approx(m - m_new);
#pragma unroll
        for (int k = 0; k < 64; ++k) {
          s[k] = ptx::ex2_approx(s[k] - m_new);
          sum += s[k];
        }
      }
      l = l * alpha + sum;
      m = m_new;
      put_row64(smem + kFwdP + (j & 1) * kScore, rloc, s);
      ptx::fence_proxy_async_smem();
      ptx::mbar_arrive(&pfull[j & 1]);
      if (j >= 1 && !merge(j - 1, alpha_pend)) {
        ok = false;
        break;
      }
      alpha_pend = alpha;
    }
    if (ok && nkb > 0) ok = merge(nkb - 1, alpha_pend);
    if (!ok) {
      if (lane == 0) timeout();
    } else if (row < a.T) {
      const float inv = 1.0f / l;  // l == 0 only for a fully masked row (NaN, as the reference)
      store_row64(a.out0, x.b, x.h, row, acc, inv);
      a.lse[static_cast<uint64_t>(x.bh) * a.T + row] = m * kLn2 + logf(l);
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem, 256);
}

// ======================================================== backward: Delta
// delta[b, h, t] = sum_d dO[b, h, t, d] * O[b, h, t, d]: one warp per row.
__global__ void __launch_bounds__(256)
flash_delta_kernel(View d_o, View o, uint32_t T, uint32_t H, uint64_t rows, float *delta) {
  pdl_enter();
  const uint64_t warps = static_cast<uint64_t>(gridDim.x) * (blockDim.x / 32);
  const uint32_t lane = threadIdx.x & 31;
  for (uint64_t r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; r < rows; r += warps) {
    const uint32_t t = static_cast<uint32_t>(r % T);
    const uint32_t bh = static_cast<uint32_t>(r / T);
    const float2 g = reinterpret_cast<const float2 *>(row_ptr(d_o, bh / H, bh % H, t))[lane];
    const float2 v = reinterpret_cast<const float2 *>(row_ptr(o, bh / H, bh % H, t))[lane];
    float acc = g.x * v.x + g.y * v.y;
#pragma unroll
    for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) delta[r] = acc;
  }
}

// ==================================================== backward: query side
constexpr int kBqStages = 2;
constexpr uint32_t kBqQ = 0, kBqDo = kTile128;
constexpr uint32_t kBqStage = 3 * kTile64;  // K (for S), K (for dQ), V
constexpr uint32_t kBqKv = 2 * kTile128;
constexpr uint32_t kBqDs = kBqKv + kBqStages * kBqStage;
constexpr uint32_t kBqBars = kBqDs + 2 * kScore;
constexpr size_t kBqSmem = 1024 + kBqBars + 256;
static_assert(kBqSmem <= 232448, "query-side backward shared memory");

template <bool KT>
__global__ void __launch_bounds__(kThreads, 1)
flash_bwd_q_kernel(const __grid_constant__ Maps maps, const Args a) {
  // maps: a Q (K-major), b dO (K-major), c K for S, d K for dQ, e V (K-major)
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kBqBars);
  uint64_t *qfull = bars;
  uint64_t *kvfull = bars + 1, *kvempty = kvfull + kBqStages;
  uint64_t *sfull = kvempty + kBqStages, *sfree = sfull + 2;
  uint64_t *dsfull = sfree + 2, *dsfree = dsfull + 2, *dqdone = dsfree + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(dqdone + 1);
  volatile uint32_t *abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    ptx::mbar_init(qfull, 1);
    for (int i = 0; i < kBqStages; ++i) {
      ptx::mbar_init(&kvfull[i], 1);
      ptx::mbar_init(&kvempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&sfull[i], 1);
      ptx::mbar_init(&sfree[i], 128);
      ptx::mbar_init(&dsfull[i], 128);
      ptx::mbar_init(&dsfree[i], 1);
    }
    ptx::mbar_init(dqdone, 1);
    *abort_flag = 0;
    ptx::fence_barrier_init();
    ptx::prefetch_tensormap(&maps.a);
    ptx::prefetch_tensormap(&maps.b);
    ptx::prefetch_tensormap(&maps.c);
    ptx::prefetch_tensormap(&maps.d);
    ptx::prefetch_tensormap(&maps.e);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem, tmem_dp = tmem + 128, tmem_dq = tmem + 256;
  pdl_enter();
  const Ctx x = context(a);
  const uint32_t last_row = min(a.T, x.tile0 + BMQ);
  const uint32_t nkb = ((x.causal ? last_row : a.T) + BNK - 1) / BNK;
  auto timeout = [&]() {
    *abort_flag = 1;
    raise_flag(a.status, TL_FLAG_TIMEOUT);
  };

  if (warp == 0) {
    if (lane == 0) {
      const int32_t hh = static_cast<int32_t>(x.h), bb = static_cast<int32_t>(x.b);
      ptx::mbar_arrive_expect_tx(qfull, 2 * kTile128);
      for (int kb = 0; kb < 2; ++kb) {
        const int32_t c[4] = {32 * kb, static_cast<int32_t>(x.tile0), hh, bb};
        ptx::tma_load_rank(smem + kBqQ + kb * 16384, &maps.a, qfull, 4, c);
        ptx::tma_load_rank(smem + kBqDo + kb * 16384, &maps.b, qfull, 4, c);
      }
      uint32_t issued = 0;
      for (uint32_t j = 0; j < nkb && !*abort_flag; ++j) {
        const uint32_t s = j % kBqStages, ph = (j / kBqStages) & 1;
        const int32_t key0 = static_cast<int32_t>(j * BNK);
        if (!ptx::mbar_wait_bounded(&kvempty[s], ph ^ 1, kWaitLimitNs)) {
          timeout();
          break;
        }
        uint8_t *st = smem + kBqKv + s * kBqStage;
        ptx::mbar_arrive_expect_tx(&kvfull[s], kBqStage);
        for (int c = 0; c < 2; ++c) {
          // K for S = Q K^T: K-major rows, or MN-major from K^T
          const int32_t ck[4] = {KT ? key0 + 32 * c : 32 * c, KT ? 0 : key0, hh, bb};
          ptx::tma_load_rank(st + c * 8192, &maps.c, &kvfull[s], 4, ck);
          // V for dP = dO V^T: K-major rows
          const int32_t cv[4] = {32 * c, key0, hh, bb};
          ptx::tma_load_rank(st + 2 * kTile64 + c * 8192, &maps.e, &kvfull[s], 4, cv);
          // K for dQ = dS K: K-major over keys from K^T
          if (KT) ptx::tma_load_rank(st + kTile64 + c * 8192, &maps.d, &kvfull[s], 4, ck);
        }
        if (!KT) {  // MN-major K chunks for dQ = dS K
          const int32_t cm[5] = {0, key0, 0, hh, bb};
          ptx::tma_load_rank(st + kTile64, &maps.d, &kvfull[s], 5, cm);
        }
        ++issued;
      }
      if (!ptx::mbar_wait_bounded(qfull, 0, kWaitLimitNs)) timeout();
      for (uint32_t j = issued > kBqStages ? issued - kBqStages : 0; j < issued; ++j)
        if (!ptx::mbar_wait_bounded(&kvfull[j % kBqStages], (j / kBqStages) & 1, kWaitLimitNs)) {
          timeout();
          break;
        }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t sq = ptx::smem_addr(smem + kBqQ), sdo = ptx::smem_addr(smem + kBqDo);
      const uint32_t idesc_s = ptx::idesc_tf32(BMQ, BNK, false, KT);
      const uint32_t idesc_dp = ptx::idesc_tf32(BMQ, BNK, false, false);
      const uint32_t idesc_dq = ptx::idesc_tf32(BMQ, HD, false, !KT);
      bool ok = ptx::mbar_wait_bounded(qfull, 0, kWaitLimitNs), issued = false;
      auto dq = [&](uint32_t i) {
        if (!ptx::mbar_wait_bounded(&dsfull[i & 1], (i >> 1) & 1, kWaitLimitNs)) return false;
        ptx::tc_fence_after();
        const uint32_t sds = ptx::smem_addr(smem + kBqDs + (i & 1) * kScore);
        const uint32_t skq = ptx::smem_addr(smem + kBqKv + (i % kBqStages) * kBqStage + kTile64);
#pragma unroll
        for (uint32_t kb = 0; kb < 2; ++kb)
#pragma unroll
          for (uint32_t kk = 0; kk < 4; ++kk)
            ptx::mma_tf32(tmem_dq, kmaj(sds, BMQ, kb, kk),
                          KT ? kmaj(skq, HD, kb, kk) : mnmaj(skq, BNK, kb, kk), idesc_dq,
                          (i | kb | kk) ? 1u : 0u);
        ptx::mma_commit(&dsfree[i & 1]);
        ptx::mma_commit(&kvempty[i % kBqStages]);
        return true;
      };
      for (uint32_t j = 0; j < nkb && ok; ++j) {
        const uint32_t s = j % kBqStages;
        if (!ptx::mbar_wait_bounded(&kvfull[s], (j / kBqStages) & 1, kWaitLimitNs) ||
            (j >= 2 && !ptx::mbar_wait_bounded(&sfree[j & 1], ((j - 2) >> 1) & 1, kWaitLimitNs))) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t st = ptx::smem_addr(smem + kBqKv + s * kBqStage);
#pragma unroll
        for (uint32_t kb = 0; kb < 2; ++kb)
#pragma unroll
          for (uint32_t kk = 0; kk < 4; ++kk) {
            ptx::mma_tf32(tmem_s + (j & 1) * BNK, kmaj(sq, BMQ, kb, kk),
                          KT ? mnmaj(st, HD, kb, kk) : kmaj(st, BNK, kb, kk), idesc_s,
                          (kb | kk) ? 1u : 0u);
            ptx::mma_tf32(tmem_dp + (j & 1) * BNK, kmaj(sdo, BMQ, kb, kk),
                          kmaj(st + 2 * kTile64, BNK, kb, kk), idesc_dp, (kb | kk) ? 1u : 0u);
          }
        issued = true;
        ptx::mma_commit(&sfull[j & 1]);
        if (j >= 1 && !dq(j - 1)) ok = false;
      }
      if (ok && nkb > 0 && !dq(nkb - 1)) ok = false;
      if (issued) ptx::mma_commit(dqdone);
      else ptx::mbar_arrive(dqdone);
      if (!ok) {
        timeout();
        ptx::mbar_wait_bounded(dqdone, 0, kWaitLimitNs);  // in-flight MMAs finish first
      } else if (issued) {
        // releases nobody waits for (the last dS buffers and K/V stages):
        // landed before the CTA exits, not on the next CTA's barriers
        ok = ptx::mbar_wait_bounded(dqdone, 0, kWaitLimitNs);
        for (uint32_t i = nkb > 2 ? nkb - 2 : 0; ok && i < nkb; ++i)
          ok = ptx::mbar_wait_bounded(&dsfree[i & 1], (i >> 1) & 1, kWaitLimitNs);
        for (uint32_t i = nkb > kBqStages ? nkb - kBqStages : 0; ok && i < nkb; ++i)
          ok = ptx::mbar_wait_bounded(&kvempty[i % kBqStages], (i / kBqStages) & 1,
                                      kWaitLimitNs);
        if (!ok) timeout();
      }
    }
  } else {
    const uint32_t q = warp & 3;
    const uint32_t rloc = q * 32 + lane, row = x.tile0 + rloc;
    const uint32_t lane_base = (q * 32u) << 16;
    const float inv = 1.0f / *a.divisor, c = kLog2e * inv;
    const bool live = row < a.T;
    const float lse2 = live ? a.lse[static_cast<uint64_t>(x.bh) * a.T + row] * kLog2e : 0.0f;
    const float dl = live ? a.delta[static_cast<uint64_t>(x.bh) * a.T + row] : 0.0f;
    bool ok = true;
    for (uint32_t j = 0; j < nkb && ok; ++j) {
      const bool got = ptx::mbar_wait_bounded(&sfull[j & 1], (j >> 1) & 1, kWaitLimitNs);
      if (!__all_sync(0xffffffffu, got) || *abort_flag) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      float s[64], dp[64];
      tmem_row64(tmem_s + (j & 1) * BNK + lane_base, s);
      tmem_row64(tmem_dp + (j & 1) * BNK + lane_base, dp);
      ptx::tc_fence_before();
      ptx::mbar_arrive(&sfree[j & 1]);
      const uint32_t key0 = j * BNK;
#pragma unroll
      for (int k = 0; k < 64; ++k) {
        const float v = score2(s[k], c, a, x, row, key0 + k);
        const float p = v == -INFINITY ? 0.0f : ptx::ex2_approx(v - lse2);
        s[k] = p * (dp[k] - dl) * inv;
      }
      if (j >= 2) {
        const bool fr = ptx::mbar_wait_bounded(&dsfree[j & 1], ((j - 2) >> 1) & 1, kWaitLimitNs);
        if (!__all_sync(0xffffffffu, fr)) {
          ok = false;
          break;
        }
      }
      put_row64(smem + kBqDs + (j & 1) * kScore, rloc, s);
      ptx::fence_proxy_async_smem();
      ptx::mbar_arrive(&dsfull[j & 1]);
    }
    const bool got = ok && ptx::mbar_wait_bounded(dqdone, 0, kWaitLimitNs);
    if (!__all_sync(0xffffffffu, got) || *abort_flag) {
      if (lane == 0) timeout();
    } else {
      ptx::tc_fence_after();
      float g[64];
      tmem_row64(tmem_dq + lane_base, g);
      if (live) store_row64(a.out0, x.b, x.h, row, g, 1.0f);
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem, 512);
}

// ====================================================== backward: key side
constexpr int kBkStages = 2;  // Q and dO blocks for S^T and dP^T
constexpr uint32_t kBkK = 0, kBkV = kTile128;
constexpr uint32_t kBkA = 2 * kTile128;                       // stages of (Q, dO) K-major
constexpr uint32_t kBkMn = kBkA + kBkStages * 2 * kTile64;    // Q, dO MN-major (one set)
constexpr uint32_t kBkPt = kBkMn + 2 * kTile64;               // P^T (128 keys x 64 queries)
constexpr uint32_t kBkDst = kBkPt + kScore;                   // dS^T
constexpr uint32_t kBkBars = kBkDst + kScore;
constexpr size_t kBkSmem = 1024 + kBkBars + 256;
static_assert(kBkSmem <= 232448, "key-side backward shared memory");

template <bool KT>
__global__ void __launch_bounds__(kThreads, 1)
flash_bwd_kv_kernel(const __grid_constant__ Maps maps, const Args a) {
  // maps: a K (A operand: K-major rows, or MN-major from K^T), b V (K-major),
  // c Q K-major, d dO K-major, e Q MN-major, f dO MN-major
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kBkBars);
  uint64_t *kvfull = bars;
  uint64_t *afull = bars + 1, *aempty = afull + kBkStages;
  uint64_t *mnfull = aempty + kBkStages, *mnempty = mnfull + 1;
  uint64_t *sfull = mnempty + 1, *sfree = sfull + 2;
  uint64_t *pdfull = sfree + 2, *pdfree = pdfull + 1, *done = pdfree + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  volatile uint32_t *abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    ptx::mbar_init(kvfull, 1);
    for (int i = 0; i < kBkStages; ++i) {
      ptx::mbar_init(&afull[i], 1);
      ptx::mbar_init(&aempty[i], 1);
    }
    ptx::mbar_init(mnfull, 1);
    ptx::mbar_init(mnempty, 1);
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&sfull[i], 1);
      ptx::mbar_init(&sfree[i], 128);
    }
    ptx::mbar_init(pdfull, 128);
    ptx::mbar_init(pdfree, 1);
    ptx::mbar_init(done, 1);
    *abort_flag = 0;
    ptx::fence_barrier_init();
    ptx::prefetch_tensormap(&maps.a);
    ptx::prefetch_tensormap(&maps.b);
    ptx::prefetch_tensormap(&maps.c);
    ptx::prefetch_tensormap(&maps.d);
    ptx::prefetch_tensormap(&maps.e);
    ptx::prefetch_tensormap(&maps.f);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem, tmem_dp = tmem + 128, tmem_dk = tmem + 256,
                 tmem_dv = tmem + 320;
  pdl_enter();
  const Ctx x = context(a);
  // queries that can see this tile's keys: all, or from its first key on
  const uint32_t qb0 = x.causal ? x.tile0 / BNK : 0;
  const uint32_t nqb = (a.T + BNK - 1) / BNK;
  const uint32_t nblk = nqb > qb0 ? nqb - qb0 : 0;
  auto timeout = [&]() {
    *abort_flag = 1;
    raise_flag(a.status, TL_FLAG_TIMEOUT);
  };

  if (warp == 0) {
    if (lane == 0) {
      const int32_t hh = static_cast<int32_t>(x.h), bb = static_cast<int32_t>(x.b);
      const int32_t k0 = static_cast<int32_t>(x.tile0);
      ptx::mbar_arrive_expect_tx(kvfull, 2 * kTile128);
      if (KT) {
        for (int c = 0; c < 4; ++c) {
          const int32_t ck[4] = {k0 + 32 * c, 0, hh, bb};
          ptx::tma_load_rank(smem + kBkK + c * 8192, &maps.a, kvfull, 4, ck);
        }
      } else {
        for (int kb = 0; kb < 2; ++kb) {
          const int32_t ck[4] = {32 * kb, k0, hh, bb};
          ptx::tma_load_rank(smem + kBkK + kb * 16384, &maps.a, kvfull, 4, ck);
        }
      }
      for (int kb = 0; kb < 2; ++kb) {
        const int32_t cv[4] = {32 * kb, k0, hh, bb};
        ptx::tma_load_rank(smem + kBkV + kb * 16384, &maps.b, kvfull, 4, cv);
      }
      // K-major (Q, dO) of block t run up to two blocks ahead; the MN-major
      // set of block t follows once block t - 1's dK / dV products are done
      uint32_t issued_a = 0, issued_mn = 0;
      bool ok = true;
      auto load_a = [&](uint32_t t) {
        const uint32_t s = t % kBkStages, ph = (t / kBkStages) & 1;
        if (!ptx::mbar_wait_bounded(&aempty[s], ph ^ 1, kWaitLimitNs)) return false;
        const int32_t y = static_cast<int32_t>((qb0 + t) * BNK);
        uint8_t *st = smem + kBkA + s * 2 * kTile64;
        ptx::mbar_arrive_expect_tx(&afull[s], 2 * kTile64);
        for (int kb = 0; kb < 2; ++kb) {
          const int32_t c[4] = {32 * kb, y, hh, bb};
          ptx::tma_load_rank(st + kb * 8192, &maps.c, &afull[s], 4, c);
          ptx::tma_load_rank(st + kTile64 + kb * 8192, &maps.d, &afull[s], 4, c);
        }
        ++issued_a;
        return true;
      };
      auto load_mn = [&](uint32_t t) {
        if (!ptx::mbar_wait_bounded(mnempty, (t & 1) ^ 1, kWaitLimitNs)) return false;
        const int32_t y = static_cast<int32_t>((qb0 + t) * BNK);
        ptx::mbar_arrive_expect_tx(mnfull, 2 * kTile64);
        const int32_t c[5] = {0, y, 0, hh, bb};
        ptx::tma_load_rank(smem + kBkMn, &maps.e, mnfull, 5, c);
        ptx::tma_load_rank(smem + kBkMn + kTile64, &maps.f, mnfull, 5, c);
        ++issued_mn;
        return true;
      };
      for (uint32_t t = 0; t < nblk && t < kBkStages && ok; ++t) ok = load_a(t);
      for (uint32_t t = 0; t < nblk && ok && !*abort_flag; ++t) {
        ok = load_mn(t);
        if (ok && t + kBkStages < nblk) ok = load_a(t + kBkStages);
      }
      if (!ok) timeout();
      if (!ptx::mbar_wait_bounded(kvfull, 0, kWaitLimitNs)) timeout();
      for (uint32_t t = issued_a > kBkStages ? issued_a - kBkStages : 0; t < issued_a; ++t)
        if (!ptx::mbar_wait_bounded(&afull[t % kBkStages], (t / kBkStages) & 1, kWaitLimitNs)) {
          timeout();
          break;
        }
      if (issued_mn && !ptx::mbar_wait_bounded(mnfull, (issued_mn - 1) & 1, kWaitLimitNs))
        timeout();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t sk = ptx::smem_addr(smem + kBkK), sv = ptx::smem_addr(smem + kBkV);
      const uint32_t idesc_s = ptx::idesc_tf32(BMQ, BNK, KT, false);
      const uint32_t idesc_dp = ptx::idesc_tf32(BMQ, BNK, false, false);
      const uint32_t idesc_g = ptx::idesc_tf32(BMQ, HD, false, true);
      bool ok = ptx::mbar_wait_bounded(kvfull, 0, kWaitLimitNs), issued = false;
      auto grads = [&](uint32_t t) {
        if (!ptx::mbar_wait_bounded(pdfull, t & 1, kWaitLimitNs) ||
            !ptx::mbar_wait_bounded(mnfull, t & 1, kWaitLimitNs))
          return false;
        ptx::tc_fence_after();
        const uint32_t spt = ptx::smem_addr(smem + kBkPt), sds = ptx::smem_addr(smem + kBkDst);
        const uint32_t sqm = ptx::smem_addr(smem + kBkMn), sdom = sqm + kTile64;
#pragma unroll
        for (uint32_t kb = 0; kb < 2; ++kb)
#pragma unroll
          for (uint32_t kk = 0; kk < 4; ++kk) {
            const uint32_t acc = (t | kb | kk) ? 1u : 0u;
            ptx::mma_tf32(tmem_dv, kmaj(spt, BMQ, kb, kk), mnmaj(sdom, BNK, kb, kk), idesc_g, acc);
            ptx::mma_tf32(tmem_dk, kmaj(sds, BMQ, kb, kk), mnmaj(sqm, BNK, kb, kk), idesc_g, acc);
          }
        ptx::mma_commit(pdfree);
        ptx::mma_commit(mnempty);
        return true;
      };
      for (uint32_t t = 0; t < nblk && ok; ++t) {
        const uint32_t s = t % kBkStages;
        if (!ptx::mbar_wait_bounded(&afull[s], (t / kBkStages) & 1, kWaitLimitNs) ||
            (t >= 2 && !ptx::mbar_wait_bounded(&sfree[t & 1], ((t - 2) >> 1) & 1, kWaitLimitNs))) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t sa = ptx::smem_addr(smem + kBkA + s * 2 * kTile64);
#pragma unroll
        for (uint32_t kb = 0; kb < 2; ++kb)
#pragma unroll
          for (uint32_t kk = 0; kk < 4; ++kk) {
            ptx::mma_tf32(tmem_s + (t & 1) * BNK, KT ? mnmaj(sk, HD, kb, kk) : kmaj(sk, BMQ, kb, kk),
                          kmaj(sa, BNK, kb, kk), idesc_s, (kb | kk) ? 1u : 0u);
            ptx::mma_tf32(tmem_dp + (t & 1) * BNK, kmaj(sv, BMQ, kb, kk),
                          kmaj(sa + kTile64, BNK, kb, kk), idesc_dp, (kb | kk) ? 1u : 0u);
          }
        issued = true;
        ptx::mma_commit(&sfull[t & 1]);
        ptx::mma_commit(&aempty[s]);
        if (t >= 1 && !grads(t - 1)) ok = false;
      }
      if (ok && nblk > 0 && !grads(nblk - 1)) ok = false;
      if (issued) ptx::mma_commit(done);
      else ptx::mbar_arrive(done);
      if (!ok) {
        timeout();
        ptx::mbar_wait_bounded(done, 0, kWaitLimitNs);
      } else if (issued && nblk > 0) {
        // releases nobody waits for (the last Q / dO stages, P^T / dS^T
        // buffer and MN-major set): landed before the CTA exits, not on the
        // next CTA's barriers
        ok = ptx::mbar_wait_bounded(done, 0, kWaitLimitNs) &&
             ptx::mbar_wait_bounded(pdfree, (nblk - 1) & 1, kWaitLimitNs) &&
             ptx::mbar_wait_bounded(mnempty, (nblk - 1) & 1, kWaitLimitNs);
        for (uint32_t t = nblk > kBkStages ? nblk - kBkStages : 0; ok && t < nblk; ++t)
          ok = ptx::mbar_wait_bounded(&aempty[t % kBkStages], (t / kBkStages) & 1, kWaitLimitNs);
        if (!ok) timeout();
      }
    }
  } else {
    const uint32_t q = warp & 3;
    const uint32_t rloc = q * 32 + lane, key = x.tile0 + rloc;
    const uint32_t lane_base = (q * 32u) << 16;
    const float inv = 1.0f / *a.divisor, c = kLog2e * inv;
    const float *lse = a.lse + static_cast<uint64_t>(x.bh) * a.T;
    const float *dlt = a.delta + static_cast<uint64_t>(x.bh) * a.T;
    bool ok = true;
    for (uint32_t t = 0; t < nblk && ok; ++t) {
      const bool got = ptx::mbar_wait_bounded(&sfull[t & 1], (t >> 1) & 1, kWaitLimitNs);
      if (!__all_sync(0xffffffffu, got) || *abort_flag) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      float s[64], dp[64];
      tmem_row64(tmem_s + (t & 1) * BNK + lane_base, s);
      tmem_row64(tmem_dp + (t & 1) * BNK + lane_base, dp);
      ptx::tc_fence_before();
      ptx::mbar_arrive(&sfree[t & 1]);
      const uint32_t y0 = (qb0 + t) * BNK;
#pragma unroll
      for (int k = 0; k < 64; ++k) {
        const uint32_t query = y0 + k;
        const float v = score2(s[k], c, a, x, query, key);
        const bool live = v != -INFINITY;
        const float p = live ? ptx::ex2_approx(v - lse[query] * kLog2e) : 0.0f;
        s[k] = p;
        dp[k] = live ? p * (dp[k] - dlt[query]) * inv : 0.0f;
      }
      if (t >= 1) {
        const bool fr = ptx::mbar_wait_bounded(pdfree, (t - 1) & 1, kWaitLimitNs);
        if (!__all_sync(0xffffffffu, fr)) {
          ok = false;
          break;
        }
      }
      put_row64(smem + kBkPt, rloc, s);
      put_row64(smem + kBkDst, rloc, dp);
      ptx::fence_proxy_async_smem();
      ptx::mbar_arrive(pdfull);
    }
    const bool got = ok && ptx::mbar_wait_bounded(done, 0, kWaitLimitNs);
    if (!__all_sync(0xffffffffu, got) || *abort_flag) {
      if (lane == 0) timeout();
    } else {
      ptx::tc_fence_after();
      float g[64];
      tmem_row64(tmem_dk + lane_base, g);
      if (key < a.T) store_row64(a.out0, x.b, x.h, key, g, 1.0f);
      tmem_row64(tmem_dv + lane_base, g);
      if (key < a.T) store_row64(a.out1, x.b, x.h, key, g, 1.0f);
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem, 512);
}

// ============================================== probabilities (fallback)
// P[b, h, t, :] = exp(S[b, h, t, :] / divisor + mask - L[b, h, t]) in place
// over the scores S = Q K^T that a tensor-core product wrote into p: one
// warp per row, the softmax output a reader other than the fused backward
// asks for.
__global__ void __launch_bounds__(256)
flash_probs_rows_kernel(float *p, const float *divisor, const float *mask,
                        const uint32_t *mask_flag, const float *lse, uint32_t T, uint64_t rows) {
  pdl_enter();
  const float inv = 1.0f / *divisor;
  const bool causal = mask && mask_flag && *mask_flag != 0;
  const uint64_t warps = static_cast<uint64_t>(gridDim.x) * (blockDim.x / 32);
  const uint32_t lane = threadIdx.x & 31;
  for (uint64_t r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; r < rows; r += warps) {
    const uint32_t t = static_cast<uint32_t>(r % T);
    const float L = lse[r];
    float *row = p + r * T;
    for (uint32_t key = lane; key < T; key += 32) {
      float v = row[key] * inv;
      if (causal) {
        if (key > t) v = -INFINITY;
      } else if (mask) {
        v = v + mask[static_cast<uint64_t>(t) * T + key];
      }
      row[key] = expf(v - L);
    }
  }
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

View view_of(const HeadView &v) { return View{const_cast<float *>(v.p), v.sb, v.sh, v.ld}; }

Args base_args(const AttnDims &d, const float *divisor, const float *mask,
               const uint32_t *mask_flag, float *lse, float *delta) {
  Args a{};
  a.T = d.T;
  a.H = d.H;
  a.tiles = (d.T + BMQ - 1) / BMQ;
  a.divisor = divisor;
  a.mask = mask;
  a.mask_flag = mask ? mask_flag : nullptr;
  a.lse = lse;
  a.delta = delta;
  a.status = device_status_ptr();
  return a;
}

unsigned grid_of(const AttnDims &d) {
  return static_cast<unsigned>(static_cast<uint64_t>(d.B) * d.H * ((d.T + BMQ - 1) / BMQ));
}

}  // namespace

bool flash_attention_fits(const AttnDims &d, const HeadView *views, int n) {
  if (d.T == 0 || d.B == 0 || d.H == 0) return false;
  if (static_cast<uint64_t>(d.B) * d.H * ((d.T + BMQ - 1) / BMQ) > 0x7fffffffu) return false;
  if (d.T > 0x7fffffffu / 2) return false;
  for (int i = 0; i < n; ++i) {
    const HeadView &v = views[i];
    if (!v.p) continue;
    if (!aligned16(v.p) || v.ld % 4 || v.sh % 4 || v.sb % 4) return false;
  }
  return true;
}

int launch_flash_fwd(const AttnDims &d, const HeadView &q, const HeadView &k, const HeadView &v,
                     const float *divisor, const float *mask, const uint32_t *mask_flag,
                     const HeadView &o, float *lse, cudaStream_t s) {
  Maps maps{};
  Args a = base_args(d, divisor, mask, mask_flag, lse, nullptr);
  if (!a.status) return fail(TL_ERR_CUDA, "flash attention: no status word");
  a.out0 = view_of(o);
  const bool kt = k.trans;
  const bool ok = attn_maps::rows(&maps.a, q, d, HD, BMQ) &&
                  (kt ? attn_maps::trans(&maps.b, k, d, HD, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)
                      : attn_maps::rows(&maps.b, k, d, HD, BNK)) &&
                  attn_maps::rows_mn(&maps.c, v, d, HD, BNK);
  if (!ok) return fail(TL_ERR_UNSUPPORTED, "flash attention forward: tensor maps refused");
  static bool attr[2] = {false, false};
  int rc = kt ? set_smem(flash_fwd_kernel<true>, kFwdSmem, attr[1], "flash forward smem")
              : set_smem(flash_fwd_kernel<false>, kFwdSmem, attr[0], "flash forward smem");
  if (rc) return rc;
  if (kt) launch_pdl(flash_fwd_kernel<true>, grid_of(d), kThreads, kFwdSmem, s, maps, a);
  else launch_pdl(flash_fwd_kernel<false>, grid_of(d), kThreads, kFwdSmem, s, maps, a);
  return launch_status("flash attention forward");
}

int launch_flash_bwd(const AttnDims &d, const HeadView &q, const HeadView &k, const HeadView &v,
                     const HeadView &o, const HeadView &d_o, const float *divisor,
                     const float *mask, const uint32_t *mask_flag, const float *lse,
                     float *delta, const HeadView &dq, const HeadView &dk, const HeadView &dv,
                     cudaStream_t s) {
  Args a = base_args(d, divisor, mask, mask_flag, const_cast<float *>(lse), delta);
  if (!a.status) return fail(TL_ERR_CUDA, "flash attention: no status word");
  const uint64_t rows = static_cast<uint64_t>(d.B) * d.H * d.T;
  launch_pdl(flash_delta_kernel, grid_for(rows * 32, 256), 256, 0, s, view_of(d_o), view_of(o),
             d.T, d.H, rows, delta);
  int rc = launch_status("flash attention backward (delta)");
  if (rc) return rc;
  const bool kt = k.trans;
  constexpr CUtensorMapSwizzle mn = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  constexpr CUtensorMapSwizzle km = CU_TENSOR_MAP_SWIZZLE_128B;
  // query side: dQ
  {
    Maps maps{};
    a.out0 = view_of(dq);
    const bool ok =
        attn_maps::rows(&maps.a, q, d, HD, BMQ) && attn_maps::rows(&maps.b, d_o, d, HD, BMQ) &&
        (kt ? attn_maps::trans(&maps.c, k, d, HD, mn) : attn_maps::rows(&maps.c, k, d, HD, BNK)) &&
        (kt ? attn_maps::trans(&maps.d, k, d, HD, km) : attn_maps::rows_mn(&maps.d, k, d, HD, BNK)) &&
        attn_maps::rows(&maps.e, v, d, HD, BNK);
    if (!ok) return fail(TL_ERR_UNSUPPORTED, "flash attention backward: tensor maps refused");
    static bool attr[2] = {false, false};
    rc = kt ? set_smem(flash_bwd_q_kernel<true>, kBqSmem, attr[1], "flash backward smem")
            : set_smem(flash_bwd_q_kernel<false>, kBqSmem, attr[0], "flash backward smem");
    if (rc) return rc;
    if (kt) launch_pdl(flash_bwd_q_kernel<true>, grid_of(d), kThreads, kBqSmem, s, maps, a);
    else launch_pdl(flash_bwd_q_kernel<false>, grid_of(d), kThreads, kBqSmem, s, maps, a);
    rc = launch_status("flash attention backward (dQ)");
    if (rc) return rc;
  }
  // key side: dK, dV
  {
    Maps maps{};
    a.out0 = view_of(dk);
    a.out1 = view_of(dv);
    const bool ok =
        (kt ? attn_maps::trans(&maps.a, k, d, HD, mn) : attn_maps::rows(&maps.a, k, d, HD, BMQ)) &&
        attn_maps::rows(&maps.b, v, d, HD, BMQ) && attn_maps::rows(&maps.c, q, d, HD, BNK) &&
        attn_maps::rows(&maps.d, d_o, d, HD, BNK) && attn_maps::rows_mn(&maps.e, q, d, HD, BNK) &&
        attn_maps::rows_mn(&maps.f, d_o, d, HD, BNK);
    if (!ok) return fail(TL_ERR_UNSUPPORTED, "flash attention backward: tensor maps refused");
    static bool attr[2] = {false, false};
    rc = kt ? set_smem(flash_bwd_kv_kernel<true>, kBkSmem, attr[1], "flash backward smem")
            : set_smem(flash_bwd_kv_kernel<false>, kBkSmem, attr[0], "flash backward smem");
    if (rc) return rc;
    if (kt) launch_pdl(flash_bwd_kv_kernel<true>, grid_of(d), kThreads, kBkSmem, s, maps, a);
    else launch_pdl(flash_bwd_kv_kernel<false>, grid_of(d), kThreads, kBkSmem, s, maps, a);
    rc = launch_status("flash attention backward (dK, dV)");
  }
  return rc;
}

int launch_flash_probs(const AttnDims &d, const HeadView &q, const HeadView &k,
                       const float *divisor, const float *mask, const uint32_t *mask_flag,
                       const float *lse, float *p, cudaStream_t s) {
  // S = Q K^T per (batch, head) on the tensor cores, straight into p
  tl_gemm_desc g{};
  g.a = q.p;
  g.b = k.p;
  g.c = p;
  g.m = d.T;
  g.n = d.T;
  g.k = HD;
  g.trans_b = k.trans ? 0 : 1;  // K rows [T, D] are B stored [N, K]; K^T is [K, N]
  g.precision = TL_GEMM_TF32;
  g.batch_rank = 2;
  g.batch_shape[0] = d.B;
  g.batch_shape[1] = d.H;
  g.a_batch_stride[0] = q.sb;
  g.a_batch_stride[1] = q.sh;
  g.b_batch_stride[0] = k.sb;
  g.b_batch_stride[1] = k.sh;
  g.c_batch_stride[0] = static_cast<uint64_t>(d.H) * d.T * d.T;
  g.c_batch_stride[1] = static_cast<uint64_t>(d.T) * d.T;
  g.lda = q.ld;
  g.ldb = k.ld;
  g.ldc = d.T;
  int rc = tl_gemm(&g, s);
  if (rc) return rc;
  const uint64_t rows = static_cast<uint64_t>(d.B) * d.H * d.T;
  launch_pdl(flash_probs_rows_kernel, grid_for(rows * 32, 256), 256, 0, s, p, divisor, mask,
             mask ? mask_flag : nullptr, lse, d.T, rows);
  return launch_status("flash attention probabilities");
}

// Whether `mask` ([T, T]) is nn::causal_mask's (include/nn/attention.h:10-22:
// -inf above the diagonal, 0 elsewhere): *flag = 1 or 0.
__global__ void __launch_bounds__(1024)
flash_mask_check_kernel(const float *__restrict__ mask, uint32_t T, uint32_t *flag) {
  pdl_enter();
  // warp w takes rows w, w + 32, ...; its lanes read 32 consecutive columns
  // at a time, a batch of them in flight (no early exit, no division)
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  bool ok = true;
  for (uint32_t r = warp; r < T; r += blockDim.x >> 5) {
    const float *row = mask + static_cast<size_t>(r) * T;
#pragma unroll 8
    for (uint32_t c = lane; c < T; c += 32)
      ok = ok & (__ldg(row + c) == (c > r ? -INFINITY : 0.0f));
  }
  ok = __syncthreads_and(ok);
  if (threadIdx.x == 0) *flag = ok ? 1u : 0u;
}

int launch_mask_check(const float *mask, uint32_t T, uint32_t *flag, cudaStream_t s) {
  launch_pdl(flash_mask_check_kernel, 1, 1024, 0, s, mask, T, flag);
  return launch_status("attention mask check");
}

}  // namespace tl

// ------------------------------------------------------------------ C ABI
using namespace tl;

namespace {

HeadView head_view(const tl_attn_view &v) {
  return HeadView{v.p, v.batch_stride, v.head_stride, v.row_stride, v.transposed != 0};
}

int check_desc(const tl_flash_desc *d, bool backward) {
  if (!d) return fail(TL_ERR_INVALID, "flash attention: null descriptor");
  if (d->D != kFusedHeadDim)
    return fail(TL_ERR_UNSUPPORTED, "flash attention: head width must be 64");
  if (!d->q.p || !d->k.p || !d->v.p || !d->divisor || !d->lse || !d->o.p)
    return fail(TL_ERR_INVALID, "flash attention: null operand");
  if (backward && (!d->d_o.p || !d->dq.p || !d->dk.p || !d->dv.p || !d->delta))
    return fail(TL_ERR_INVALID, "flash attention backward: null operand");
  if (d->q.transposed || d->v.transposed || d->o.transposed || d->d_o.transposed ||
      d->dq.transposed || d->dk.transposed || d->dv.transposed)
    return fail(TL_ERR_UNSUPPORTED, "flash attention: only k may be stored transposed");
  if (tl_flash_attention_supported(d) != 1)
    return fail(TL_ERR_UNSUPPORTED, "flash attention: operands not 16-byte aligned or sizes "
                                    "out of range");
  return TL_OK;
}

}  // namespace

extern "C" int tl_flash_attention_supported(const tl_flash_desc *d) {
  if (!d || d->D != kFusedHeadDim) return 0;
  const AttnDims dims{d->B, d->T, d->H};
  const HeadView v[8] = {head_view(d->q),  head_view(d->k),  head_view(d->v),
                         head_view(d->o),  head_view(d->d_o), head_view(d->dq),
                         head_view(d->dk), head_view(d->dv)};
  return flash_attention_fits(dims, v, 8) ? 1 : 0;
}

extern "C" int tl_flash_attention_fwd(const tl_flash_desc *d, void *stream) {
  int rc = check_desc(d, false);
  if (rc) return rc;
  if (d->B == 0 || d->H == 0 || d->T == 0) return TL_OK;
  return launch_flash_fwd(AttnDims{d->B, d->T, d->H}, head_view(d->q), head_view(d->k),
                          head_view(d->v), d->divisor, d->mask, d->mask_flag, head_view(d->o),
                          d->lse, as_stream(stream));
}

extern "C" int tl_flash_attention_bwd(const tl_flash_desc *d, void *stream) {
  int rc = check_desc(d, true);
  if (rc) return rc;
  if (d->B == 0 || d->H == 0 || d->T == 0) return TL_OK;
  return launch_flash_bwd(AttnDims{d->B, d->T, d->H}, head_view(d->q), head_view(d->k),
                          head_view(d->v), head_view(d->o), head_view(d->d_o), d->divisor,
                          d->mask, d->mask_flag, d->lse, d->delta, head_view(d->dq),
                          head_view(d->dk), head_view(d->dv), as_stream(stream));
}

extern "C" int tl_flash_attention_probs(const tl_flash_desc *d, float *p, void *stream) {
  int rc = check_desc(d, false);
  if (rc) return rc;
  if (!p) return fail(TL_ERR_INVALID, "flash attention probabilities: null output");
  if (d->B == 0 || d->H == 0 || d->T == 0) return TL_OK;
  return launch_flash_probs(AttnDims{d->B, d->T, d->H}, head_view(d->q), head_view(d->k),
                            d->divisor, d->mask, d->mask_flag, d->lse, p, as_stream(stream));
}

extern "C" int tl_attention_mask_check(const float *mask, uint32_t T, uint32_t *flag,
                                       void *stream) {
  if (!mask || !flag) return fail(TL_ERR_INVALID, "attention mask check: null pointer");
  if (T == 0) return TL_OK;
  return launch_mask_check(mask, T, flag, as_stream(stream));
}

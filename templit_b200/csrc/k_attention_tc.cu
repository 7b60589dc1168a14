// Fused attention on the tensor cores for short sequences (T <= 192) and
// 64-wide heads: the executor's attention composite (include/nn/
// multi_head.h:45-52; softmax derivative include/passes/execute.h:291-308)
// without its T x T score and score-gradient tensors in HBM.
//
// Forward, one CTA per (batch, head, 128 query rows), 320 threads, two
// CTAs per SM:
//   warp 0       TMA: the Q tile, all of K, all of V; TMA stores of P
//   warp 1       TMEM owner, MMA issuer: S = Q K^T into TMEM (128 x nk fp32),
//                then O = P V block by block as the softmax hands over P
//   warps 2..9   softmax, two warps per TMEM lane quadrant on alternate
//                key pieces: one pass for the row max and the sum of
//                exponentials of S / divisor + mask (merged across the two
//                warps through shared memory), then P = exp(x - max) / sum
//                written in 32-key blocks into a two-slot shared-memory ring
//                in the MMA's K-major layout (also the TMA box of the P
//                store); finally O from TMEM to global.
// P leaves through TMA stores (the backward reads it); S never leaves TMEM.
//
// Backward, query side (same CTA shape): dP = dO V^T into TMEM; the softmax
// derivative dS = P * (dP - rowsum(dP * P)) / divisor overwrites this tile's
// P in shared memory and leaves through TMA stores; dQ = dS K.  Key side,
// one CTA per (batch, head, 128 keys): dK = dS^T Q and dV = P^T dO over
// 32-query blocks of a TMA ring, all four operands MN-major.
//
// Operand layouts follow storage, as in the GEMM: a [T, D] row block is
// K-major for a product over D and MN-major (TMA 32-byte-atom swizzle) for a
// product over T; K may also come stored transposed ([D, T], the executor's
// K^T), which swaps its two roles.
//
// Every wait is bounded (2 s): on timeout the CTA raises TL_FLAG_TIMEOUT,
// lets what it issued finish and returns.
#include "attention_tc.h"
#include "tc_ptx.cuh"

#include <cuda.h>

namespace tl {
namespace {

constexpr int kSoftWarps = 8;  // two per TMEM lane quadrant
constexpr int kThreads = 64 + 32 * kSoftWarps;
constexpr uint32_t BMQ = 128;  // query rows of a CTA
constexpr uint32_t HD = kFusedHeadDim;
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr float kLog2e = 1.4426950408889634f;

// Element strides of a head-strided output written from registers.
struct Out {
  float *p;
  uint64_t sb, sh, ld;
};

Out out_of(const HeadView &v) { return Out{const_cast<float *>(v.p), v.sb, v.sh, v.ld}; }

// Shared memory of the query-side kernels (offsets from a 1024-aligned
// base), small enough for two CTAs per SM.  Region A holds the operands of
// the first product (a 128-row tile of D = 64 in two 16 KB K-major blocks,
// then an nk-row operand, 48 KB at most), and, once that product is done,
// the second product's nk-row operand (48 KB) and a ring of two 128 x 32
// score blocks (P or dS) that the softmax warps fill, the MMA warp
// multiplies and warp 0 stores.  Then the row reductions and barriers.
constexpr uint32_t kBlock = BMQ * 128;                         // 16 KB
constexpr uint32_t kRegQ = 2 * kBlock;                         // 32 KB
constexpr uint32_t kRingOff = 2 * kMaxFusedKeys * 128;         // 48 KB
constexpr uint32_t kRegion = kRegQ + 2 * kMaxFusedKeys * 128;  // 80 KB
static_assert(kRingOff + 2 * kBlock <= kRegion, "ring exceeds region A");
constexpr uint32_t kRed = kRegion;
constexpr uint32_t kBars = kRed + 4 * BMQ * 4;
constexpr size_t kQuerySmem = 1024 + kBars + 256;
constexpr uint32_t kTmemCols = 256;  // scores (<= 192 columns) + a 64-column product
static_assert(kMaxFusedKeys + HD <= kTmemCols, "TMEM budget");
// The query-side backward takes all of the SM's TMEM.  With two of its CTAs
// holding 256 columns each, the softmax derivative's row sums came out
// wrong in a few rows of CTAs that started while the SM's other CTA was
// mid-way (dS differed from run to run in about 10 of 73,728 rows at
// configuration 3; never with one CTA's TMEM per SM, at one CTA per SM, or
// when every CTA started in the first wave).  The cause was not found; with
// 512 columns the second CTA on an SM sets up while the first runs and
// starts its tensor-core work when the first has freed the TMEM
// (configuration-3 backward 122 us instead of 105 us, deterministic).
constexpr uint32_t kTmemColsBwdQ = 512;

__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t j) {
  return r * 128u + ((j ^ (r & 7u)) << 4);
}

__device__ __forceinline__ uint8_t *align1024(uint8_t *p) {
  return reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(p) + 1023) &
                                     ~static_cast<uintptr_t>(1023));
}

// Row `row` of a 128 x 64 fp32 TMEM accumulator half (32 columns at col0)
// to out[row] columns col0.. (float4 stores).
__device__ __forceinline__ void store_row32(uint32_t taddr, const Out &o, int32_t b, int32_t h,
                                            uint32_t t, uint32_t col0, bool ok) {
  uint32_t r[32];
  ptx::tmem_load_32x32b_x32(taddr, r);
  ptx::tmem_load_wait();
  if (!ok) return;
  float4 *dst =
      reinterpret_cast<float4 *>(o.p + b * o.sb + h * o.sh + static_cast<uint64_t>(t) * o.ld + col0);
#pragma unroll
  for (int j = 0; j < 8; ++j)
    dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                         __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
}

// Scores of 16 columns of one row: s / divisor (as s * (1 / divisor)) +
// mask (a mask row, when given); columns from `lim` on (past T, or past the
// row under a causal mask) are -inf.  `open`: no mask row and every column
// below `lim` (warp-uniform), so neither is looked at.
__device__ __forceinline__ void score16(const uint32_t (&r)[16], float inv, const float *mrow,
                                        uint32_t col0, uint32_t T, uint32_t lim, bool open,
                                        float (&x)[16]) {
  if (open) {
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = __uint_as_float(r[j]) * inv;
    return;
  }
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    float4 mk = make_float4(0.f, 0.f, 0.f, 0.f);
    const uint32_t c = col0 + 4 * g;
    if (mrow && c + 4 <= T) mk = *reinterpret_cast<const float4 *>(mrow + c);
    const float mv[4] = {mk.x, mk.y, mk.z, mk.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t col = c + i;
      float v = __uint_as_float(r[4 * g + i]) * inv;
      if (mrow) v = v + (c + 4 <= T ? mv[i] : (col < T ? mrow[col] : 0.0f));
      x[4 * g + i] = col < lim ? v : -INFINITY;
    }
  }
}

// Loads of the nk-row operands.  A [T, D] block as a K-major operand of a
// product over D: two boxes of 32 columns x nk rows.  As an MN-major operand
// of a product over T: one box of (32 columns, nk rows, 2 chunks).  A
// transposed ([D, T]) block: nk / 32 boxes of 32 keys x 64 rows, K-major for
// a product over T (128-byte swizzle) or MN-major for one over D (32-byte
// atoms).
__device__ __forceinline__ void load_rows_kmajor(uint8_t *dst, const CUtensorMap *m, uint64_t *bar,
                                                 uint32_t nk, int32_t h, int32_t b) {
  for (int kb = 0; kb < 2; ++kb) {
    const int32_t c[4] = {32 * kb, 0, h, b};
    ptx::tma_load_rank(dst + kb * nk * 128, m, bar, 4, c);
  }
}

__device__ __forceinline__ void load_rows_mnmajor(uint8_t *dst, const CUtensorMap *m,
                                                  uint64_t *bar, int32_t h, int32_t b) {
  const int32_t c[5] = {0, 0, 0, h, b};
  ptx::tma_load_rank(dst, m, bar, 5, c);
}

__device__ __forceinline__ void load_trans_blocks(uint8_t *dst, const CUtensorMap *m,
                                                  uint64_t *bar, uint32_t nk, int32_t h,
                                                  int32_t b) {
  for (uint32_t c = 0; c < nk / 32; ++c) {
    const int32_t cc[4] = {static_cast<int32_t>(32 * c), 0, h, b};
    ptx::tma_load_rank(dst + c * HD * 128, m, bar, 4, cc);
  }
}

struct FwdMaps {
  CUtensorMap q, k, v, p;
};

struct FwdArgs {
  uint32_t T, H, nk, qtiles;
  const float *divisor, *mask;
  const uint32_t *mask_flag;  // nonzero: the mask is the causal one
  Out o;
  uint32_t *status;
};

// Whether `mask` ([T, T], T % 4 == 0) is the causal mask of nn::causal_mask
// (include/nn/attention.h:10-22: -inf above the diagonal, 0 elsewhere).
__global__ void __launch_bounds__(1024)
mask_causal_kernel(const float *__restrict__ mask, uint32_t T, uint32_t *flag) {
  pdl_enter();
  bool ok = true;
  const uint32_t n4 = T * T / 4;  // T <= 192
  for (uint32_t i = threadIdx.x; i < n4; i += blockDim.x) {
    const float4 m = reinterpret_cast<const float4 *>(mask)[i];
    const uint32_t r = (4 * i) / T, c = 4 * i - r * T;
    ok = ok && m.x == (c > r ? -INFINITY : 0.0f) && m.y == (c + 1 > r ? -INFINITY : 0.0f) &&
         m.z == (c + 2 > r ? -INFINITY : 0.0f) && m.w == (c + 3 > r ? -INFINITY : 0.0f);
  }
  ok = __syncthreads_and(ok);
  if (threadIdx.x == 0) *flag = ok ? 1u : 0u;
}

template <bool KT>
__global__ void __launch_bounds__(kThreads, 2)
attn_fwd_kernel(const __grid_constant__ FwdMaps maps, const FwdArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  // region A: Q and K for S, then V and the P ring for P V
  uint8_t *s_q = smem, *s_k = smem + kRegQ, *s_v = smem, *s_ring = smem + kRingOff;
  float *red_m = reinterpret_cast<float *>(smem + kRed);  // [2][128] row maxima
  float *red_s = red_m + 2 * BMQ;                          // [2][128] row sums
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kBars);
  uint64_t *bar_qk = bars, *bar_v = bars + 1, *bar_s = bars + 2, *bar_o = bars + 3;
  uint64_t *full = bars + 4, *mma_done = bars + 6, *store_done = bars + 8;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 10);
  volatile uint32_t *abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const uint32_t nkb = a.nk / 32;
  const uint32_t qt = blockIdx.x % a.qtiles;
  const uint32_t bh = blockIdx.x / a.qtiles;
  const int32_t hh = static_cast<int32_t>(bh % a.H), bb = static_cast<int32_t>(bh / a.H);
  const int32_t q0 = static_cast<int32_t>(qt * BMQ);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) ptx::mbar_init(&bars[i], 1);
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&full[i], kSoftWarps * 32);  // a block: every softmax thread
      ptx::mbar_init(&mma_done[i], 1);
      ptx::mbar_init(&store_done[i], 1);
    }
    *abort_flag = 0;
    ptx::fence_barrier_init();
    ptx::prefetch_tensormap(&maps.q);
    ptx::prefetch_tensormap(&maps.k);
    ptx::prefetch_tensormap(&maps.v);
    ptx::prefetch_tensormap(&maps.p);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem, tmem_o = tmem + kMaxFusedKeys;
  pdl_enter();
  // causal mask: applied arithmetically; key blocks past the tile's last
  // row are all masked (P = 0 there), so S and P V stop at nk_eff
  const bool causal = a.mask && a.mask_flag && *a.mask_flag != 0;
  const uint32_t nk_eff =
      causal ? min(a.nk, (min(a.T, static_cast<uint32_t>(q0) + BMQ) + 31) / 32 * 32) : a.nk;

  auto timeout = [&]() {
    *abort_flag = 1;
    raise_flag(a.status, TL_FLAG_TIMEOUT);
  };

  if (warp == 0) {
    // ------------------------------------------------ loads and P stores
    if (lane == 0) {
      const uint32_t kbytes = a.nk * HD * 4;
      bool ok = true;
      ptx::mbar_arrive_expect_tx(bar_qk, 2 * BMQ * 128 + kbytes);
      for (int kb = 0; kb < 2; ++kb) {
        const int32_t cq[4] = {32 * kb, q0, hh, bb};
        ptx::tma_load_rank(s_q + kb * BMQ * 128, &maps.q, bar_qk, 4, cq);
      }
      if (KT)
        load_trans_blocks(s_k, &maps.k, bar_qk, a.nk, hh, bb);
      else
        load_rows_kmajor(s_k, &maps.k, bar_qk, a.nk, hh, bb);
      // V replaces Q and K once S is computed
      ok = ptx::mbar_wait_bounded(bar_s, 0, kWaitLimitNs);
      if (ok) {
        ptx::mbar_arrive_expect_tx(bar_v, kbytes);
        load_rows_mnmajor(s_v, &maps.v, bar_v, hh, bb);
      }
      // each P block leaves by TMA store once written; its ring slot is
      // free again when the store has read it and its MMAs are done
      for (uint32_t c = 0; c < nkb && ok; ++c) {
        const uint32_t slot = c & 1, use = c >> 1;
        if (!ptx::mbar_wait_bounded(&full[slot], use & 1, kWaitLimitNs)) {
          ok = false;
          break;
        }
        ptx::tma_store_3d(&maps.p, s_ring + slot * kBlock, static_cast<int32_t>(c * 32), q0,
                          static_cast<int32_t>(bh));
        ptx::bulk_commit_group();
        ptx::bulk_wait_group_read<0>();
        ptx::mbar_arrive(&store_done[slot]);
      }
      if (ok) ok = ptx::mbar_wait_bounded(bar_v, 0, kWaitLimitNs);
      if (!ok) timeout();
      ptx::bulk_wait_group<0>();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMAs
    if (lane == 0) {
      bool issued = false;
      const uint32_t sq = ptx::smem_addr(s_q), sk = ptx::smem_addr(s_k);
      const uint32_t sv = ptx::smem_addr(s_v), sr = ptx::smem_addr(s_ring);
      bool ok = ptx::mbar_wait_bounded(bar_qk, 0, kWaitLimitNs);
      if (ok) {
        ptx::tc_fence_after();
        const uint32_t idesc_s = ptx::idesc_tf32(BMQ, nk_eff, false, KT);
#pragma unroll
        for (uint32_t kb = 0; kb < 2; ++kb)
#pragma unroll
          for (uint32_t kk = 0; kk < 4; ++kk) {
            const uint64_t bd =
                KT ? ptx::smem_desc(sk + (kb * 32 + kk * 8) * 128, HD * 128, 512,
                                    ptx::kSwizzle128B32BAtom)
                   : ptx::smem_desc(sk + kb * a.nk * 128 + kk * 32, 16, 1024, ptx::kSwizzle128B);
            ptx::mma_tf32(tmem_s,
                          ptx::smem_desc(sq + kb * BMQ * 128 + kk * 32, 16, 1024,
                                         ptx::kSwizzle128B),
                          bd, idesc_s, (kb | kk) ? 1u : 0u);
          }
        issued = true;
        ptx::mma_commit(bar_s);
        ok = ptx::mbar_wait_bounded(bar_v, 0, kWaitLimitNs);
      }
      const uint32_t idesc_o = ptx::idesc_tf32(BMQ, HD, false, true);
      for (uint32_t c = 0; c < nkb && ok; ++c) {
        const uint32_t slot = c & 1, use = c >> 1;
        if (!ptx::mbar_wait_bounded(&full[slot], use & 1, kWaitLimitNs)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        if (c < nk_eff / 32) {
#pragma unroll
          for (uint32_t kk = 0; kk < 4; ++kk)
            ptx::mma_tf32(tmem_o,
                          ptx::smem_desc(sr + slot * kBlock + kk * 32, 16, 1024,
                                         ptx::kSwizzle128B),
                          ptx::smem_desc(sv + (c * 32 + kk * 8) * 128, a.nk * 128, 512,
                                         ptx::kSwizzle128B32BAtom),
                          idesc_o, (c | kk) ? 1u : 0u);
        }
        ptx::mma_commit(&mma_done[slot]);  // (blocks of zeros: nothing to wait for)
      }
      if (!ok) timeout();
      if (issued) {
        ptx::mma_commit(bar_o);
        ptx::mbar_wait_bounded(bar_o, 0, kWaitLimitNs);  // before TMEM is released
        // The last blocks' mma_done arrivals are waited for nowhere else:
        // an arrival still in flight when the CTA exits would land on the
        // barrier of the next CTA to take this shared memory.
        for (uint32_t c = nkb > 2 ? nkb - 2 : 0; ok && c < nkb; ++c)
          ok = ptx::mbar_wait_bounded(&mma_done[c & 1], (c >> 1) & 1, kWaitLimitNs);
      } else {
        ptx::mbar_arrive(bar_o);
      }
    }
  } else {
    // --------------------------------------------------------- softmax
    // Warps 2..9: quadrant q = warp % 4 (the TMEM lanes a warp may read),
    // the two warps of a quadrant on alternate 16-key pieces.  Three passes
    // over S: max, sum of exponentials, P (through the ring).
    const int e = warp - 2;
    const uint32_t q = warp & 3, half = static_cast<uint32_t>(e) >> 2;
    const uint32_t row = q * 32 + lane;
    const uint32_t grow = qt * BMQ + row;
    const bool row_ok = grow < a.T;
    const float inv = 1.0f / *a.divisor;
    const float *mrow =
        (a.mask && !causal && row_ok) ? a.mask + static_cast<size_t>(grow) * a.T : nullptr;
    // keys from `lim` on are masked: past T, or (causal) past this row
    const uint32_t lim = causal ? min(a.T, grow + 1) : a.T;
    const uint32_t lane_base = (q * 32u) << 16;
    const uint32_t npieces = nk_eff / 16;
    bool ok = ptx::mbar_wait_bounded(bar_s, 0, kWaitLimitNs);
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0) timeout();
      ok = false;
    }
    // the row of lane 0 has the warp's smallest `lim`: pieces wholly below
    // it need no masking
    const uint32_t lim_lo = __shfl_sync(0xffffffffu, lim, 0);
    auto open = [&](uint32_t piece) { return !mrow && (piece + 1) * 16 <= lim_lo; };
    // one pass over S: an online (max, sum of 2^((x - max) log2 e)) per row,
    // rescaled once per 16-key piece
    float m = -INFINITY, sum = 0.0f;
    if (ok) {
      ptx::tc_fence_after();
      for (uint32_t c = half; c < npieces; c += 2) {
        uint32_t r[16];
        ptx::tmem_load_32x32b_x16(tmem_s + lane_base + c * 16, r);
        ptx::tmem_load_wait();
        float x[16];
        score16(r, inv, mrow, c * 16, a.T, lim, open(c), x);
        float pm = x[0];
#pragma unroll
        for (int j = 1; j < 16; ++j) pm = fmaxf(pm, x[j]);
        const float mn = fmaxf(m, pm);
        if (mn != -INFINITY) {
          const float ml = mn * kLog2e;
          float ps = 0.0f;
#pragma unroll
          for (int j = 0; j < 16; ++j) ps += ptx::ex2_approx(fmaf(x[j], kLog2e, -ml));
          sum = fmaf(sum, ptx::ex2_approx(fmaf(m, kLog2e, -ml)), ps);
          m = mn;
        }
      }
      red_m[half * BMQ + row] = m;
      red_s[half * BMQ + row] = sum;
    }
    ptx::named_bar_sync(1, 32 * kSoftWarps);
    if (ok) {
      // both halves merge in the same order, so they agree on (max, sum)
      const float m0 = red_m[row], m1 = red_m[BMQ + row];
      const float s0 = red_s[row], s1 = red_s[BMQ + row];
      m = fmaxf(m0, m1);
      const float ml0 = m * kLog2e;
      sum = m == -INFINITY ? 0.0f
                           : s0 * ptx::ex2_approx(fmaf(m0, kLog2e, -ml0)) +
                                 s1 * ptx::ex2_approx(fmaf(m1, kLog2e, -ml0));
      const float inv_sum = 1.0f / sum;
      const float ml = m * kLog2e;
      for (uint32_t c = 0; c < nkb; ++c) {
        const uint32_t slot = c & 1, use = c >> 1;
        const uint32_t piece = 2 * c + half;
        float4 v[4];
        if (piece < npieces) {
          uint32_t r[16];
          ptx::tmem_load_32x32b_x16(tmem_s + lane_base + piece * 16, r);
          ptx::tmem_load_wait();
          float x[16];
          score16(r, inv, mrow, piece * 16, a.T, lim, open(piece), x);
#pragma unroll
          for (int g = 0; g < 4; ++g)
            v[g] = make_float4(ptx::ex2_approx(fmaf(x[4 * g], kLog2e, -ml)) * inv_sum,
                               ptx::ex2_approx(fmaf(x[4 * g + 1], kLog2e, -ml)) * inv_sum,
                               ptx::ex2_approx(fmaf(x[4 * g + 2], kLog2e, -ml)) * inv_sum,
                               ptx::ex2_approx(fmaf(x[4 * g + 3], kLog2e, -ml)) * inv_sum);
        } else {
#pragma unroll
          for (int g = 0; g < 4; ++g) v[g] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (use > 0) {  // the slot's previous block is stored and multiplied
          const bool freed = ptx::mbar_wait_bounded(&mma_done[slot], (use - 1) & 1, kWaitLimitNs) &&
                             ptx::mbar_wait_bounded(&store_done[slot], (use - 1) & 1, kWaitLimitNs);
          if (!__all_sync(0xffffffffu, freed)) {
            if (lane == 0) timeout();
            ok = false;
            break;
          }
        }
        uint8_t *blk = s_ring + slot * kBlock;
#pragma unroll
        for (int g = 0; g < 4; ++g)
          *reinterpret_cast<float4 *>(blk + swz(row, half * 4 + g)) = v[g];
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(&full[slot]);
      }
    }
    // O: TMEM -> global, each warp of a quadrant 32 of the 64 columns
    ok = ok && ptx::mbar_wait_bounded(bar_o, 0, kWaitLimitNs);
    if (__all_sync(0xffffffffu, ok) && !*abort_flag) {
      ptx::tc_fence_after();
      store_row32(tmem_o + lane_base + half * 32, a.o, bb, hh, grow, half * 32, row_ok);
    } else if (lane == 0 && !ok) {
      timeout();
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------ backward, query side
struct BwdQMaps {
  CUtensorMap d_o, v, k, p, ds;
};

struct BwdQArgs {
  uint32_t T, H, nk, qtiles;
  const float *divisor;
  Out dq;
  uint32_t *status;
};

// Rows of P stream through the two-slot ring twice: once for rowsum(dP * P),
// once to turn each block into dS in place (then multiplied by K for dQ and
// TMA-stored).  Use i of the ring (i = 0 .. 2 nkb - 1) loads P block
// i % nkb into slot i % 2; pass-2 block c is use nkb + c.
template <bool KT>
__global__ void __launch_bounds__(kThreads, 2)
attn_bwd_q_kernel(const __grid_constant__ BwdQMaps maps, const BwdQArgs a) {
  constexpr uint32_t S = 2;  // ring slots
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  // region A: dO and V for dP, then K and the ring for dQ
  uint8_t *s_do = smem, *s_v = smem + kRegQ, *s_k = smem, *s_ring = smem + kRingOff;
  float *red = reinterpret_cast<float *>(smem + kRed);  // [2][128] partial row sums
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kBars);
  uint64_t *bar_a = bars, *bar_k = bars + 1, *bar_dp = bars + 2, *bar_dq = bars + 3;
  uint64_t *loaded = bars + 4, *consumed = bars + 6, *full = bars + 8, *mma_done = bars + 10;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 12);
  volatile uint32_t *abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const uint32_t nkb = a.nk / 32;
  const uint32_t qt = blockIdx.x % a.qtiles;
  const uint32_t bh = blockIdx.x / a.qtiles;
  const int32_t hh = static_cast<int32_t>(bh % a.H), bb = static_cast<int32_t>(bh / a.H);
  const int32_t q0 = static_cast<int32_t>(qt * BMQ);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) ptx::mbar_init(&bars[i], 1);
    for (uint32_t i = 0; i < S; ++i) {
      ptx::mbar_init(&loaded[i], 1);
      ptx::mbar_init(&consumed[i], kSoftWarps * 32);
      ptx::mbar_init(&full[i], kSoftWarps * 32);
      ptx::mbar_init(&mma_done[i], 1);
    }
    *abort_flag = 0;
    ptx::fence_barrier_init();
    ptx::prefetch_tensormap(&maps.d_o);
    ptx::prefetch_tensormap(&maps.v);
    ptx::prefetch_tensormap(&maps.k);
    ptx::prefetch_tensormap(&maps.p);
    ptx::prefetch_tensormap(&maps.ds);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, kTmemColsBwdQ);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_dp = tmem, tmem_dq = tmem + kMaxFusedKeys;
  pdl_enter();

  auto timeout = [&]() {
    *abort_flag = 1;
    raise_flag(a.status, TL_FLAG_TIMEOUT);
  };

  if (warp == 0) {
    // ------------------------------ loads, the P stream and the dS stores
    if (lane == 0) {
      const uint32_t kbytes = a.nk * HD * 4;
      ptx::mbar_arrive_expect_tx(bar_a, 2 * BMQ * 128 + kbytes);
      for (int kb = 0; kb < 2; ++kb) {
        const int32_t cd[4] = {32 * kb, q0, hh, bb};
        ptx::tma_load_rank(s_do + kb * BMQ * 128, &maps.d_o, bar_a, 4, cd);
      }
      load_rows_kmajor(s_v, &maps.v, bar_a, a.nk, hh, bb);
      bool ok = ptx::mbar_wait_bounded(bar_dp, 0, kWaitLimitNs);  // dO, V consumed
      if (ok) {
        ptx::mbar_arrive_expect_tx(bar_k, kbytes);
        if (KT)
          load_trans_blocks(s_k, &maps.k, bar_k, a.nk, hh, bb);
        else
          load_rows_mnmajor(s_k, &maps.k, bar_k, hh, bb);
      }
      uint32_t stored = 0;  // pass-2 blocks stored so far
      auto store = [&](uint32_t c) -> bool {
        const uint32_t slot = (nkb + c) % S;
        if (!ptx::mbar_wait_bounded(&full[slot], (c / S) & 1, kWaitLimitNs)) return false;
        ptx::tma_store_3d(&maps.ds, s_ring + slot * kBlock, static_cast<int32_t>(c * 32), q0,
                          static_cast<int32_t>(bh));
        ptx::bulk_commit_group();
        ++stored;
        return true;
      };
      for (uint32_t i = 0; i < 2 * nkb && ok; ++i) {
        const uint32_t slot = i % S;
        if (i >= S) {  // the slot's previous use is over
          const uint32_t ip = i - S;
          if (ip < nkb) {
            ok = ptx::mbar_wait_bounded(&consumed[slot], (ip / S) & 1, kWaitLimitNs);
          } else {
            const uint32_t cp = ip - nkb;
            ok = store(cp);
            if (ok) {
              ptx::bulk_wait_group_read<0>();
              ok = ptx::mbar_wait_bounded(&mma_done[slot], (cp / S) & 1, kWaitLimitNs);
            }
          }
          if (!ok) break;
        }
        ptx::mbar_arrive_expect_tx(&loaded[slot], kBlock);
        ptx::tma_load_3d(s_ring + slot * kBlock, &maps.p, &loaded[slot],
                         static_cast<int32_t>((i % nkb) * 32), q0, static_cast<int32_t>(bh));
      }
      while (ok && stored < nkb) ok = store(stored);
      if (ok) ok = ptx::mbar_wait_bounded(bar_k, 0, kWaitLimitNs);
      if (!ok) timeout();
      ptx::bulk_wait_group<0>();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool issued = false;
      const uint32_t sdo = ptx::smem_addr(s_do), sv = ptx::smem_addr(s_v);
      const uint32_t sk = ptx::smem_addr(s_k), sr = ptx::smem_addr(s_ring);
      bool ok = ptx::mbar_wait_bounded(bar_a, 0, kWaitLimitNs);
      if (ok) {
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
        ok = ptx::mbar_wait_bounded(bar_k, 0, kWaitLimitNs);
      }
      const uint32_t idesc_q = ptx::idesc_tf32(BMQ, HD, false, !KT);
      for (uint32_t c = 0; c < nkb && ok; ++c) {
        const uint32_t slot = (nkb + c) % S;
        if (!ptx::mbar_wait_bounded(&full[slot], (c / S) & 1, kWaitLimitNs)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
#pragma unroll
        for (uint32_t kk = 0; kk < 4; ++kk) {
          const uint64_t bd =
              KT ? ptx::smem_desc(sk + c * HD * 128 + kk * 32, 16, 1024, ptx::kSwizzle128B)
                 : ptx::smem_desc(sk + (c * 32 + kk * 8) * 128, a.nk * 128, 512,
                                  ptx::kSwizzle128B32BAtom);
          ptx::mma_tf32(tmem_dq,
                        ptx::smem_desc(sr + slot * kBlock + kk * 32, 16, 1024, ptx::kSwizzle128B),
                        bd, idesc_q, (c | kk) ? 1u : 0u);
        }
        ptx::mma_commit(&mma_done[slot]);
      }
      if (!ok) timeout();
      if (issued) {
        ptx::mma_commit(bar_dq);
        ptx::mbar_wait_bounded(bar_dq, 0, kWaitLimitNs);
        // The last S blocks' mma_done arrivals are waited for nowhere else:
        // one still in flight when the CTA exits would land on the barrier
        // of the next CTA to take this shared memory (seen as dS rows that
        // changed from run to run in CTAs that started mid-launch).
        for (uint32_t c = nkb > S ? nkb - S : 0; ok && c < nkb; ++c)
          ok = ptx::mbar_wait_bounded(&mma_done[(nkb + c) % S], (c / S) & 1, kWaitLimitNs);
      } else {
        ptx::mbar_arrive(bar_dq);
      }
    }
  } else {
    // ----------------------------------------------- softmax derivative
    const int e = warp - 2;
    const uint32_t q = warp & 3, half = static_cast<uint32_t>(e) >> 2;
    const uint32_t row = q * 32 + lane;
    const uint32_t grow = qt * BMQ + row;
    const float inv = 1.0f / *a.divisor;
    const uint32_t lane_base = (q * 32u) << 16;
    bool ok = ptx::mbar_wait_bounded(bar_dp, 0, kWaitLimitNs);
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0) timeout();
      ok = false;
    }
    float sum = 0.0f;
    if (ok) {
      ptx::tc_fence_after();
      for (uint32_t c = 0; c < nkb; ++c) {
        const uint32_t slot = c % S, piece = 2 * c + half;
        const bool got = ptx::mbar_wait_bounded(&loaded[slot], (c / S) & 1, kWaitLimitNs);
        uint32_t r[16];
        ptx::tmem_load_32x32b_x16(tmem_dp + lane_base + piece * 16, r);
        ptx::tmem_load_wait();
        if (!__all_sync(0xffffffffu, got)) {
          if (lane == 0) timeout();
          ok = false;
          break;
        }
        const uint8_t *blk = s_ring + slot * kBlock;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const float4 p4 = *reinterpret_cast<const float4 *>(blk + swz(row, half * 4 + g));
          sum = fmaf(__uint_as_float(r[4 * g]), p4.x, sum);
          sum = fmaf(__uint_as_float(r[4 * g + 1]), p4.y, sum);
          sum = fmaf(__uint_as_float(r[4 * g + 2]), p4.z, sum);
          sum = fmaf(__uint_as_float(r[4 * g + 3]), p4.w, sum);
        }
        ptx::mbar_arrive(&consumed[slot]);
      }
      red[half * BMQ + row] = sum;
    }
    ptx::named_bar_sync(1, 32 * kSoftWarps);
    if (ok) {
      sum = red[row] + red[BMQ + row];  // same order in both halves
      for (uint32_t c = 0; c < nkb; ++c) {
        const uint32_t i = nkb + c, slot = i % S, piece = 2 * c + half;
        const bool got = ptx::mbar_wait_bounded(&loaded[slot], (i / S) & 1, kWaitLimitNs);
        uint32_t r[16];
        ptx::tmem_load_32x32b_x16(tmem_dp + lane_base + piece * 16, r);
        ptx::tmem_load_wait();
        if (!__all_sync(0xffffffffu, got)) {
          if (lane == 0) timeout();
          ok = false;
          break;
        }
        uint8_t *blk = s_ring + slot * kBlock;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          float4 *slot4 = reinterpret_cast<float4 *>(blk + swz(row, half * 4 + g));
          const float4 p4 = *slot4;
          *slot4 = make_float4(p4.x * (__uint_as_float(r[4 * g]) - sum) * inv,
                               p4.y * (__uint_as_float(r[4 * g + 1]) - sum) * inv,
                               p4.z * (__uint_as_float(r[4 * g + 2]) - sum) * inv,
                               p4.w * (__uint_as_float(r[4 * g + 3]) - sum) * inv);
        }
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(&full[slot]);
      }
    }
    ok = ok && ptx::mbar_wait_bounded(bar_dq, 0, kWaitLimitNs);
    if (__all_sync(0xffffffffu, ok) && !*abort_flag) {
      ptx::tc_fence_after();
      store_row32(tmem_dq + lane_base + half * 32, a.dq, bb, hh, grow, half * 32, grow < a.T);
    } else if (lane == 0 && !ok) {
      timeout();
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem, kTmemColsBwdQ);
}

// -------------------------------------------------------- backward, key side
constexpr int kKvThreads = 64 + 128;
constexpr int kKvStages = 4;
constexpr uint32_t kKvA = 128 * 32 * 4;  // 128 keys x 32 queries
constexpr uint32_t kKvB = 32 * HD * 4;   // 32 queries x 64
constexpr uint32_t kKvPart = kKvA + kKvB;  // one product's share of a stage
constexpr size_t kv_smem(uint32_t products) { return 1024 + kKvStages * products * kKvPart + 256; }

struct BwdKvMaps {
  CUtensorMap ds, p, q, d_o;
};

struct BwdKvArgs {
  uint32_t T, H, ktiles, qblocks;
  bool with_dk, with_dv;
  uint32_t stage_bytes, dv_off;  // products x kKvPart; dV's part in a stage
  Out dk, dv;
  uint32_t *status;
};

__global__ void __launch_bounds__(kKvThreads, 2)
attn_bwd_kv_kernel(const __grid_constant__ BwdKvMaps maps, const BwdKvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kKvStages * a.stage_bytes);
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
    if (a.with_dk) {
      ptx::prefetch_tensormap(&maps.ds);
      ptx::prefetch_tensormap(&maps.q);
    }
    if (a.with_dv) {
      ptx::prefetch_tensormap(&maps.p);
      ptx::prefetch_tensormap(&maps.d_o);
    }
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
      const uint32_t bytes = a.stage_bytes;
      uint32_t stage = 0, phase = 0, issued = 0;
      for (uint32_t qb = 0; qb < a.qblocks; ++qb) {
        if (!ptx::mbar_wait_bounded(&empty[stage], phase ^ 1, kWaitLimitNs)) {
          timeout();
          break;
        }
        uint8_t *st = smem + stage * a.stage_bytes;
        ptx::mbar_arrive_expect_tx(&full[stage], bytes);
        const int32_t y = static_cast<int32_t>(qb * 32);
        for (int j = 0; j < 4; ++j) {
          if (a.with_dk)
            ptx::tma_load_3d(st + j * 4096, &maps.ds, &full[stage], k0 + 32 * j, y,
                             static_cast<int32_t>(bh));
          if (a.with_dv)
            ptx::tma_load_3d(st + a.dv_off + j * 4096, &maps.p, &full[stage], k0 + 32 * j, y,
                             static_cast<int32_t>(bh));
        }
        for (int j = 0; j < 2; ++j) {
          const int32_t c[4] = {32 * j, y, hh, bb};
          if (a.with_dk) ptx::tma_load_rank(st + kKvA + j * 4096, &maps.q, &full[stage], 4, c);
          if (a.with_dv)
            ptx::tma_load_rank(st + a.dv_off + kKvA + j * 4096, &maps.d_o, &full[stage], 4, c);
        }
        ++issued;
        if (++stage == kKvStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      // every issued stage has landed before the CTA may exit
      const uint32_t back = issued < kKvStages ? issued : kKvStages;
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
      uint32_t stage = 0, phase = 0, committed = 0;
      bool issued = false;
      for (uint32_t qb = 0; qb < a.qblocks && !*abort_flag; ++qb) {
        if (!ptx::mbar_wait_bounded(&full[stage], phase, kWaitLimitNs)) {
          timeout();
          break;
        }
        ptx::tc_fence_after();
        const uint32_t st = ptx::smem_addr(smem + stage * a.stage_bytes);
#pragma unroll
        for (uint32_t kk = 0; kk < 4; ++kk) {
          const uint32_t acc = (qb | kk) ? 1u : 0u;
          if (a.with_dk)
            ptx::mma_tf32(tmem,
                          ptx::smem_desc(st + kk * 1024, 4096, 512, ptx::kSwizzle128B32BAtom),
                          ptx::smem_desc(st + kKvA + kk * 1024, 4096, 512,
                                         ptx::kSwizzle128B32BAtom),
                          idesc, acc);
          if (a.with_dv)
            ptx::mma_tf32(tmem + HD,
                          ptx::smem_desc(st + a.dv_off + kk * 1024, 4096, 512,
                                         ptx::kSwizzle128B32BAtom),
                          ptx::smem_desc(st + a.dv_off + kKvA + kk * 1024, 4096, 512,
                                         ptx::kSwizzle128B32BAtom),
                          idesc, acc);
        }
        issued = true;
        ++committed;
        ptx::mma_commit(&empty[stage]);
        if (++stage == kKvStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (issued) {
        ptx::mma_commit(done);
        if (!ptx::mbar_wait_bounded(done, 0, kWaitLimitNs)) timeout();
        // the releases of the last stages (their arrivals must not be in
        // flight when the CTA exits: they would reach the next CTA's barriers)
        const uint32_t back = committed < kKvStages ? committed : kKvStages;
        uint32_t s = stage, p = phase;
        for (uint32_t i = 0; i < back; ++i) {
          if (s == 0) {
            s = kKvStages - 1;
            p ^= 1;
          } else {
            --s;
          }
          if (!ptx::mbar_wait_bounded(&empty[s], p, kWaitLimitNs)) {
            timeout();
            break;
          }
        }
      } else {
        ptx::mbar_arrive(done);  // nothing issued: release the epilogue
      }
    }
  } else {
    const uint32_t q = warp & 3;
    const uint32_t key = kt * 128 + q * 32 + lane;
    const bool ok = ptx::mbar_wait_bounded(done, 0, kWaitLimitNs);
    if (__all_sync(0xffffffffu, ok) && !*abort_flag) {
      ptx::tc_fence_after();
      const uint32_t lane_base = (q * 32u) << 16;
      if (a.with_dk)
        for (uint32_t c = 0; c < 2; ++c)
          store_row32(tmem + lane_base + c * 32, a.dk, bb, hh, key, c * 32, key < a.T);
      if (a.with_dv)
        for (uint32_t c = 0; c < 2; ++c)
          store_row32(tmem + lane_base + HD + c * 32, a.dv, bb, hh, key, c * 32, key < a.T);
    } else if (lane == 0 && !ok) {
      timeout();
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc(tmem, 128);
}

// ---------------------------------------------------------------- host side
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

// A [T, D] head block as [D, T, H, B], box 32 columns x `rows`.
bool rows_map(CUtensorMap *map, const HeadView &v, const AttnDims &d, uint32_t rows,
              CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  const cuuint64_t dims[4] = {HD, d.T, d.H, d.B};
  const cuuint64_t st[3] = {v.ld * 4, v.sh * 4, v.sb * 4};
  const cuuint32_t box[4] = {32, rows, 1, 1};
  return encode(map, v.p, 4, dims, st, box, swz);
}

// A [T, D] head block as [32, T, D / 32, H, B] (32-wide column chunks of
// rows, the MN-major operand layout), box 32 x rows x D / 32.
bool rows_map_mn(CUtensorMap *map, const HeadView &v, const AttnDims &d, uint32_t rows) {
  const cuuint64_t dims[5] = {32, d.T, HD / 32, d.H, d.B};
  const cuuint64_t st[4] = {v.ld * 4, 128, v.sh * 4, v.sb * 4};
  const cuuint32_t box[5] = {32, rows, HD / 32, 1, 1};
  return encode(map, v.p, 5, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
}

// A transposed [D, T] head block as [T, D, H, B], box 32 keys x D rows.
bool trans_map(CUtensorMap *map, const HeadView &v, const AttnDims &d, CUtensorMapSwizzle swz) {
  const cuuint64_t dims[4] = {d.T, HD, d.H, d.B};
  const cuuint64_t st[3] = {v.ld * 4, v.sh * 4, v.sb * 4};
  const cuuint32_t box[4] = {32, HD, 1, 1};
  return encode(map, v.p, 4, dims, st, box, swz);
}

// Dense [B, H, T, T] scores as [T, T, B * H], box 32 x rows.
bool scores_map(CUtensorMap *map, const float *base, const AttnDims &d, uint32_t rows,
                CUtensorMapSwizzle swz) {
  const cuuint64_t dims[3] = {d.T, d.T, static_cast<cuuint64_t>(d.B) * d.H};
  const cuuint64_t st[2] = {static_cast<cuuint64_t>(d.T) * 4,
                            static_cast<cuuint64_t>(d.T) * d.T * 4};
  const cuuint32_t box[3] = {32, rows, 1};
  return encode(map, base, 3, dims, st, box, swz);
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

uint32_t keys_of(const AttnDims &d) { return (d.T + 31) / 32 * 32; }

}  // namespace

bool fused_attention_fits(const AttnDims &d, const HeadView *views, const bool *may_trans,
                          int n) {
  if (d.T == 0 || d.T > kMaxFusedKeys || d.T % 4 != 0 || d.B == 0 || d.H == 0) return false;
  if (static_cast<uint64_t>(d.B) * d.H * ((d.T + BMQ - 1) / BMQ) > 0x7fffffffu) return false;
  for (int i = 0; i < n; ++i) {
    const HeadView &v = views[i];
    if (!v.p) continue;
    if (!aligned16(v.p) || v.ld % 4 || v.sh % 4 || v.sb % 4) return false;
    if (v.trans && !may_trans[i]) return false;
  }
  return true;
}

int launch_attention_fwd_tc(const AttnDims &d, const HeadView &q, const HeadView &k,
                            const HeadView &v, const float *divisor, const float *mask, float *p,
                            const HeadView &o, uint32_t *mask_flag, cudaStream_t s,
                            bool mask_checked) {
  FwdMaps maps{};
  FwdArgs a{};
  if (mask && !aligned16(mask))  // rows of the mask are read as float4
    return fail(TL_ERR_UNSUPPORTED, "attention forward: mask not 16-byte aligned");
  a.mask_flag = mask ? mask_flag : nullptr;
  a.T = d.T;
  a.H = d.H;
  a.nk = keys_of(d);
  a.qtiles = (d.T + BMQ - 1) / BMQ;
  a.divisor = divisor;
  a.mask = mask;
  a.o = out_of(o);
  a.status = device_status_ptr();
  if (!a.status) return fail(TL_ERR_CUDA, "attention forward: no status word");
  const bool kt = k.trans;
  const bool maps_ok =
      rows_map(&maps.q, q, d, BMQ) &&
      (kt ? trans_map(&maps.k, k, d, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)
          : rows_map(&maps.k, k, d, a.nk)) &&
      rows_map_mn(&maps.v, v, d, a.nk) &&
      scores_map(&maps.p, p, d, BMQ, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!maps_ok) return fail(TL_ERR_UNSUPPORTED, "attention forward: tensor maps refused");
  static bool attr[2] = {false, false};
  int rc = kt ? set_smem(attn_fwd_kernel<true>, kQuerySmem, attr[1], "attention forward: smem")
              : set_smem(attn_fwd_kernel<false>, kQuerySmem, attr[0], "attention forward: smem");
  if (rc) return rc;
  if (a.mask_flag && !mask_checked) {
    launch_pdl(mask_causal_kernel, 1, 1024, 0, s, mask, d.T, mask_flag);
    rc = launch_status("attention forward (mask check)");
    if (rc) return rc;
  }
  const unsigned grid = static_cast<unsigned>(static_cast<uint64_t>(d.B) * d.H * a.qtiles);
  if (kt)
    launch_pdl(attn_fwd_kernel<true>, grid, kThreads, kQuerySmem, s, maps, a);
  else
    launch_pdl(attn_fwd_kernel<false>, grid, kThreads, kQuerySmem, s, maps, a);
  return launch_status("attention forward");
}

int launch_attention_bwd_q_tc(const AttnDims &d, const HeadView &d_o, const HeadView &v,
                              const HeadView &k, const float *p, const float *divisor, float *ds,
                              const HeadView &dq, cudaStream_t s) {
  BwdQMaps maps{};
  BwdQArgs a{};
  a.T = d.T;
  a.H = d.H;
  a.nk = keys_of(d);
  a.qtiles = (d.T + BMQ - 1) / BMQ;
  a.divisor = divisor;
  a.dq = out_of(dq);
  a.status = device_status_ptr();
  if (!a.status) return fail(TL_ERR_CUDA, "attention backward: no status word");
  const bool kt = k.trans;
  const bool maps_ok = rows_map(&maps.d_o, d_o, d, BMQ) && rows_map(&maps.v, v, d, a.nk) &&
                       (kt ? trans_map(&maps.k, k, d, CU_TENSOR_MAP_SWIZZLE_128B)
                           : rows_map_mn(&maps.k, k, d, a.nk)) &&
                       scores_map(&maps.p, p, d, BMQ, CU_TENSOR_MAP_SWIZZLE_128B) &&
                       scores_map(&maps.ds, ds, d, BMQ, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!maps_ok) return fail(TL_ERR_UNSUPPORTED, "attention backward: tensor maps refused");
  static bool attr[2] = {false, false};
  int rc = kt ? set_smem(attn_bwd_q_kernel<true>, kQuerySmem, attr[1], "attention backward: smem")
              : set_smem(attn_bwd_q_kernel<false>, kQuerySmem, attr[0], "attention backward: smem");
  if (rc) return rc;
  const unsigned grid = static_cast<unsigned>(static_cast<uint64_t>(d.B) * d.H * a.qtiles);
  if (kt)
    launch_pdl(attn_bwd_q_kernel<true>, grid, kThreads, kQuerySmem, s, maps, a);
  else
    launch_pdl(attn_bwd_q_kernel<false>, grid, kThreads, kQuerySmem, s, maps, a);
  return launch_status("attention backward (dQ)");
}

int launch_attention_bwd_kv_tc(const AttnDims &d, const float *ds, const HeadView &q,
                               const HeadView &dk, const float *p, const HeadView &d_o,
                               const HeadView &dv, cudaStream_t s) {
  BwdKvMaps maps{};
  BwdKvArgs a{};
  a.T = d.T;
  a.H = d.H;
  a.ktiles = (d.T + 127) / 128;
  a.qblocks = (d.T + 31) / 32;
  a.with_dk = dk.p != nullptr;
  a.with_dv = dv.p != nullptr;
  a.dk = out_of(dk);
  a.dv = out_of(dv);
  a.status = device_status_ptr();
  if (!a.status) return fail(TL_ERR_CUDA, "attention backward: no status word");
  if (!a.with_dk && !a.with_dv) return TL_OK;
  constexpr CUtensorMapSwizzle mn = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  bool maps_ok = true;
  if (a.with_dk)
    maps_ok = scores_map(&maps.ds, ds, d, 32, mn) && rows_map(&maps.q, q, d, 32, mn);
  if (a.with_dv)
    maps_ok = maps_ok && scores_map(&maps.p, p, d, 32, mn) && rows_map(&maps.d_o, d_o, d, 32, mn);
  if (!maps_ok) return fail(TL_ERR_UNSUPPORTED, "attention backward: tensor maps refused");
  a.stage_bytes = ((a.with_dk ? 1u : 0u) + (a.with_dv ? 1u : 0u)) * kKvPart;
  a.dv_off = a.with_dk ? kKvPart : 0;
  const size_t smem = kv_smem(a.stage_bytes / kKvPart);
  static bool attr = false;
  int rc = set_smem(attn_bwd_kv_kernel, kv_smem(2), attr, "attention backward: smem");
  if (rc) return rc;
  const unsigned grid = static_cast<unsigned>(static_cast<uint64_t>(d.B) * d.H * a.ktiles);
  launch_pdl(attn_bwd_kv_kernel, grid, kKvThreads, smem, s, maps, a);
  return launch_status("attention backward (dK, dV)");
}

}  // namespace tl

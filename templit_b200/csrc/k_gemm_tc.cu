// Tensor-core GEMM for sm_100a: tcgen05.mma kind::tf32 with fp32
// accumulation in TMEM, operands staged by TMA (no multicast).
//
// Persistent, warp-specialised CTA of 320 threads (one CTA per SM):
//   warp 0      TMA producer: STAGES-deep ring of (A, B) k-tiles in smem
//   warp 1      TMEM owner + MMA issuer (one thread issues tcgen05.mma)
//   warps 2..9  epilogue, two warps per TMEM lane quadrant on alternate
//               32-column chunks: tcgen05.ld of the accumulator, bias /
//               addend / GELU, swizzled smem boxes, TMA stores to C
// Two TMEM accumulators (2 x BN columns) let the epilogue of tile i overlap
// the MMAs of tile i+1.  CTA tile 128 x BN x 32 (32 fp32 = one 128-byte
// swizzle row).  Operand majorness follows the stored layout:
//   A [M,K] row-major  -> K-major, TMA SWIZZLE_128B
//   A stored [K,M]     -> MN-major, TMA SWIZZLE_128B_ATOM_32B (tf32 MN-major
//                         operands only accept this 32-byte-atom swizzle)
//   B [K,N] row-major  -> MN-major;  B stored [N,K] -> K-major
// so the executor's NN, NT (transposed B) and TN (transposed A) products
// need no transpose pass.  Batched operands use a 3-D tensor map whose third
// dimension walks whole matrices, so a k-tile never reads a neighbour's rows.
//
// 3xTF32 (TL_GEMM_3XTF32, SPLIT): four more warps split every landed k-tile
// in shared memory into its tf32-rounded big part (written in place) and the
// tf32-rounded remainder (written to a second half of the stage), and the
// MMA warp accumulates big*small + small*big + big*big per k-step, which
// keeps about 21 of fp32's 24 significand bits of every product.
//
// Every mbarrier wait is bounded (2 s): on timeout the CTA raises
// TL_FLAG_TIMEOUT in the device status word, drains what it issued and
// returns instead of hanging the GPU.
#include "gemm_common.cuh"
#include "tc_ptx.cuh"

#include <cuda.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

namespace tl {

EncodeTiledFn tensor_map_encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

namespace {

constexpr int kEpiWarps = 8;  // two warps per TMEM lane quadrant
constexpr int kConvWarps = 4;  // 3xTF32 operand splitters
constexpr int BM = 128, BK = 32;
constexpr uint32_t kA_BYTES = BM * BK * 4;  // 16 KB
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr uint32_t kFlagTimeout = TL_FLAG_TIMEOUT;

struct OpMap {
  int32_t nb;       // batch dims in the map (0..3)
  int32_t dim[3];   // product batch dim of its batch map dim i
  int32_t chunked;  // MN-major: one load of `chunked` 32-wide chunks (map
                    // dims 32 x K x MN/32 [x batch]), 0: one load per chunk
};

// Tensor maps of one launch: per group the A, B and C maps (N groups share
// A; K groups share C), plus GELU output and addend (C's layout).
struct TcMaps {
  CUtensorMap a[TL_GEMM_MAX_GROUPS];
  CUtensorMap b[TL_GEMM_MAX_GROUPS];
  CUtensorMap c[TL_GEMM_MAX_GROUPS];
  CUtensorMap gelu;
  CUtensorMap addend;
};

struct TcArgs {
  GemmArgs g;
  uint32_t mt, nt;        // tiles along M and N
  uint64_t num_tiles;     // groups (N) * batch * splits * mt * nt
  uint32_t tiles_per_group;  // batch * splits * mt * nt
  bool kgroups;              // K-grouped: k-tiles run through the groups
  uint32_t kb_per_group;     // k-tiles of one group
  // batch dims each operand's tensor map walks (those with a nonzero
  // stride), as indices into the product's batch dims
  OpMap ma, mb, mc;
  uint32_t *status;
  // split-K: the K range is cut into `splits` slices of kb_per_split k-tiles;
  // slice s writes its raw fp32 product to partial + s * M * N (batch 1 only)
  // and a second kernel sums the slices in order and applies the epilogue.
  uint32_t splits, kb_per_split;
  float *partial;
  // epilogue through shared memory and TMA stores (C, or the split-K
  // partials, dense per matrix with rows of a multiple of 16 bytes)
  bool tma_epi;
  // the TMA epilogue reads an addend / GELU-input box per chunk: the
  // producer prefetches each tile's boxes into L2 when it starts the tile
  bool aux_prefetch;
};

// PAIR: a CTA pair (cluster of 2) computes a 256 x BN tile with cta_group::2
// products; each CTA loads its 128 rows of A and BN / 2 columns of B and
// holds its 128 rows of the accumulator.
// BX: staging boxes per epilogue warp, 0 for the default (one for 256-wide
// and 3xTF32 tiles, else two); 2 gives 256-wide tiles two (one fewer
// pipeline stage, for the GELU-output products, whose chunks leave by two
// stores); 1 gives narrower tiles one (one more pipeline stage, for
// products whose epilogue reads no box).
template <int BN, bool SPLIT, bool PAIR = false, int BX = 0>
struct Cfg {
  static_assert(!(SPLIT && PAIR), "3xTF32 runs on single CTAs");
  static constexpr int THREADS = 64 + 32 * kEpiWarps + (SPLIT ? 32 * kConvWarps : 0);
  static constexpr int BN_LOAD = PAIR ? BN / 2 : BN;  // columns of B this CTA loads
  static constexpr uint32_t BMT = PAIR ? 256 : 128;    // rows of a tile
  static constexpr uint32_t B_BYTES = BN_LOAD * BK * 4;
  // bytes TMA brings per stage (A then B); a 3xTF32 stage holds their
  // small parts after them in the same layout
  static constexpr uint32_t LOAD_BYTES = kA_BYTES + B_BYTES;
  static constexpr uint32_t STAGE_BYTES = SPLIT ? 2 * LOAD_BYTES : LOAD_BYTES;
  // staging boxes for the TMA stores: per epilogue warp two 32 x 32 fp32
  // boxes (4 KB each, 128-byte swizzled rows), one for the widest tile and
  // for 3xTF32 (whose stages are twice as large)
  static constexpr int BOXES = BX ? BX : ((BN == 256 || SPLIT) ? 1 : 2);
  static constexpr uint32_t OUT_BYTES = kEpiWarps * BOXES * 4096;
  static constexpr uint32_t BAR_BYTES = 384;
  static constexpr int STAGES_FIT =
      static_cast<int>((232448u - 1024u - BAR_BYTES - OUT_BYTES) / STAGE_BYTES);
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  // second accumulator at a power-of-two column; allocation a power of two
  static constexpr uint32_t ACC_COLS = BN == 192 ? 256 : BN;
  static constexpr uint32_t TMEM_COLS = 2 * ACC_COLS < 32 ? 32 : 2 * ACC_COLS;
  static constexpr size_t SMEM = 1024 + STAGES * STAGE_BYTES + OUT_BYTES + BAR_BYTES;
  // barriers: full, empty, conv (STAGES each), tfull, tempty (2 each),
  // abar (per epilogue warp), then the TMEM slot and the abort word
  static_assert((3 * STAGES + 4 + kEpiWarps) * 8 + 8 <= BAR_BYTES, "barrier area");
};

// tile = ((z * splits + s) * nt + nb) * mt + mb: consecutive CTAs take
// consecutive row blocks of the same column block and K slice, so they
// share the B tiles in L2.
__device__ __forceinline__ void decode_tile(const TcArgs &t, uint64_t tile, uint64_t &z,
                                            uint32_t &s, uint32_t &mb, uint32_t &nb,
                                            uint32_t &grp) {
  // fewer than 2^32 tiles (checked at launch): 32-bit divisions
  uint32_t tl = static_cast<uint32_t>(tile);
  grp = tl / t.tiles_per_group;  // N groups: group-major
  tl -= grp * t.tiles_per_group;
  mb = tl % t.mt;
  uint32_t r = tl / t.mt;
  nb = r % t.nt;
  r /= t.nt;
  s = r % t.splits;
  z = r / t.splits;
}

__device__ __forceinline__ void k_range(const TcArgs &t, uint32_t ktiles, uint32_t s,
                                        uint32_t &kb0, uint32_t &kb1) {
  kb0 = s * t.kb_per_split;
  kb1 = min(ktiles, kb0 + t.kb_per_split);
}

// Coordinates of flattened batch index z in the product's batch dims.
__device__ __forceinline__ void batch_coords(const GemmArgs &g, uint64_t z,
                                             int32_t (&cz)[TL_GEMM_MAX_BATCH_RANK]) {
  uint32_t r = static_cast<uint32_t>(z);
  for (int d = static_cast<int>(g.batch_rank) - 1; d >= 0; --d) {
    cz[d] = static_cast<int32_t>(r % g.batch_shape[d]);
    r /= g.batch_shape[d];
  }
}

__device__ __forceinline__ void map_coords(const OpMap &m, const int32_t (&cz)[TL_GEMM_MAX_BATCH_RANK],
                                           int32_t (&out)[3]) {
#pragma unroll
  for (int i = 0; i < 3; ++i) out[i] = i < m.nb ? cz[m.dim[i]] : 0;
}

// Byte offset of 16-byte group j of row r in a 128-byte-swizzled box.
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t j) {
  return r * 128u + ((j ^ (r & 7u)) << 4);
}

template <int BN, bool A_MN, bool B_MN, bool SPLIT, bool PAIR, int BX = 0>
__global__ void __launch_bounds__(Cfg<BN, SPLIT, PAIR, BX>::THREADS, 1)
tc_gemm_kernel(const __grid_constant__ TcMaps maps, const TcArgs t) {
  using C = Cfg<BN, SPLIT, PAIR, BX>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *stage_base = smem;
  uint8_t *out_base = smem + C::STAGES * C::STAGE_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(out_base + C::OUT_BYTES);
  uint64_t *full = bars;
  uint64_t *empty = bars + C::STAGES;
  uint64_t *tfull = bars + 2 * C::STAGES;
  uint64_t *tempty = tfull + 2;
  uint64_t *abar = tempty + 2;  // one per epilogue warp: addend box loaded
  uint64_t *conv = abar + kEpiWarps;  // 3xTF32: stage split into big / small parts
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(conv + C::STAGES);
  volatile uint32_t *abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const GemmArgs &g = t.g;
  // CTA pairs: rank in the pair, and the pair's place in the tile loop
  const uint32_t rank = PAIR ? ptx::cluster_rank() : 0u;
  const uint64_t tile0 = PAIR ? blockIdx.x / 2 : blockIdx.x;
  const uint64_t tile_step = PAIR ? gridDim.x / 2 : gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
      if (SPLIT) ptx::mbar_init(&conv[s], kConvWarps);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&tfull[a], 1);
      // a pair's accumulator is free once the epilogues of both CTAs read it
      ptx::mbar_init(&tempty[a], (PAIR ? 2 : 1) * 32 * kEpiWarps);
    }
    for (int w = 0; w < kEpiWarps; ++w) ptx::mbar_init(&abar[w], 1);
    *abort_flag = 0;
    ptx::fence_barrier_init();
    ptx::fence_proxy_async_smem();
    for (uint32_t i = 0; i < t.g.groups; ++i) {
      if (i == 0 || t.kgroups) ptx::prefetch_tensormap(&maps.a[i]);
      ptx::prefetch_tensormap(&maps.b[i]);
      if (t.tma_epi && (i == 0 || !t.kgroups)) ptx::prefetch_tensormap(&maps.c[i]);
    }
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      ptx::tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
      ptx::tmem_relinquish_pair();
    } else {
      ptx::tmem_alloc(tmem_slot, C::TMEM_COLS);
      ptx::tmem_relinquish();
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  // a pair: both CTAs' barriers exist before either signals the other's
  if constexpr (PAIR) ptx::cluster_sync();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t ktiles = t.kgroups ? t.g.groups * t.kb_per_group : (g.k + BK - 1) / BK;
  // the setup above overlaps the previous kernel's tail
  pdl_enter();

  auto timeout = [&]() {
    *abort_flag = 1;
    raise_flag(t.status, kFlagTimeout);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      uint64_t issued = 0;
      for (uint64_t tile = tile0; tile < t.num_tiles && !*abort_flag; tile += tile_step) {
        uint64_t z;
        uint32_t s, mb, nb, kb0, kb1, grp;
        decode_tile(t, tile, z, s, mb, nb, grp);
        k_range(t, ktiles, s, kb0, kb1);
        int32_t cz[TL_GEMM_MAX_BATCH_RANK], za[3], zb[3];
        batch_coords(g, z, cz);
        map_coords(t.ma, cz, za);
        map_coords(t.mb, cz, zb);
        // this CTA's rows of A; its columns of B (a pair splits them)
        const int32_t m0 = static_cast<int32_t>(mb * C::BMT + rank * BM);
        const int32_t n0 = static_cast<int32_t>(nb * BN);
        const int32_t nl = n0 + static_cast<int32_t>(rank * C::BN_LOAD);
        if (t.aux_prefetch) {
          // the epilogue's addend / GELU-input boxes of this tile: into L2
          // while the mainloop runs, so its per-chunk loads hit L2
          int32_t zc[3];
          map_coords(t.mc, cz, zc);
          for (int c = 0; c < BN / 32; ++c)
            for (int q = 0; q < BM / 32; ++q)
              ptx::tma_prefetch_nd(&maps.addend, n0 + 32 * c, m0 + 32 * q, t.mc.nb, zc);
        }
        for (uint32_t kb = kb0; kb < kb1; ++kb) {
          if (!ptx::mbar_wait_bounded(&empty[stage], phase ^ 1, kWaitLimitNs)) {
            timeout();
            break;
          }
          uint8_t *sa = stage_base + stage * C::STAGE_BYTES;
          uint8_t *sb = sa + kA_BYTES;
          if constexpr (PAIR) {
            // both CTAs' loads count on the first CTA's barrier
            if (rank == 0) ptx::mbar_arrive_expect_tx(&full[stage], 2 * C::LOAD_BYTES);
          } else {
            ptx::mbar_arrive_expect_tx(&full[stage], C::LOAD_BYTES);
          }
          // K groups walk group after group; N groups use their own B
          uint32_t kg = 0, kl = kb;
          if (t.kgroups) {
            kg = kb / t.kb_per_group;
            kl = kb - kg * t.kb_per_group;
          }
          const CUtensorMap *tmA = &maps.a[kg];
          const CUtensorMap *tmB = &maps.b[t.kgroups ? kg : grp];
          const int32_t k0 = static_cast<int32_t>(kl * BK);
          // a box at (x, y) (+ batch coordinates z) of map m into dst
          auto load2 = [&](void *dst, const CUtensorMap *m, int32_t x, int32_t y, int nz,
                           const int32_t *zz) {
            if constexpr (PAIR) {
              const int32_t c[5] = {x, y, zz[0], zz[1], zz[2]};
              ptx::tma_load_pair(dst, m, ptx::mapa_shared(&full[stage], 0), 2 + nz, c);
            } else {
              ptx::tma_load_nd(dst, m, &full[stage], x, y, nz, zz);
            }
          };
          auto loadr = [&](void *dst, const CUtensorMap *m, int r, const int32_t *c) {
            if constexpr (PAIR) ptx::tma_load_pair(dst, m, ptx::mapa_shared(&full[stage], 0), r, c);
            else ptx::tma_load_rank(dst, m, &full[stage], r, c);
          };
          if (!A_MN) {
            load2(sa, tmA, k0, m0, t.ma.nb, za);
          } else if (t.ma.chunked) {
            const int32_t c[5] = {0, k0, m0 / 32, za[0], za[1]};
            loadr(sa, tmA, 3 + t.ma.nb, c);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 32; ++j) load2(sa + j * 4096, tmA, m0 + 32 * j, k0, t.ma.nb, za);
          }
          if (!B_MN) {
            load2(sb, tmB, k0, nl, t.mb.nb, zb);
          } else if (t.mb.chunked) {
            const int32_t c[5] = {0, k0, nl / 32, zb[0], zb[1]};
            loadr(sb, tmB, 3 + t.mb.nb, c);
          } else {
#pragma unroll
            for (int j = 0; j < C::BN_LOAD / 32; ++j)
              load2(sb + j * 4096, tmB, nl + 32 * j, k0, t.mb.nb, zb);
          }
          ++issued;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: every issued k-tile must have landed (full; a pair's second
      // CTA: its loads count on the first CTA's barriers, which that CTA
      // drains) and, unless aborting, been released by the MMAs (empty: the
      // commit's arrival must not be in flight when the CTA exits, or it
      // would land on the barrier of the next CTA to take this shared
      // memory; a pair's commits reach both CTAs).
      const uint64_t back = issued < static_cast<uint64_t>(C::STAGES) ? issued : C::STAGES;
      uint32_t s = stage, p = phase;
      for (uint64_t i = 0; i < back; ++i) {
        if (s == 0) {
          s = C::STAGES - 1;
          p ^= 1;
        } else {
          --s;
        }
        if ((!PAIR || rank == 0) && !ptx::mbar_wait_bounded(&full[s], p, kWaitLimitNs)) {
          timeout();
          break;
        }
        if (!*abort_flag && !ptx::mbar_wait_bounded(&empty[s], p, kWaitLimitNs)) {
          timeout();
          break;
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    // (a pair's products are issued by its first CTA)
    if (lane == 0 && (!PAIR || rank == 0)) {
      constexpr uint32_t idesc = ptx::idesc_tf32(C::BMT, BN, A_MN, B_MN);
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool issued_any = false;
      for (uint64_t tile = tile0; tile < t.num_tiles && !*abort_flag; tile += tile_step) {
        if (!ptx::mbar_wait_bounded(&tempty[acc], acc_phase ^ 1, kWaitLimitNs)) {
          timeout();
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::ACC_COLS;
        bool ok = true;
        uint64_t z;
        uint32_t s, mb, nb, kb0, kb1, grp;
        decode_tile(t, tile, z, s, mb, nb, grp);
        k_range(t, ktiles, s, kb0, kb1);
        for (uint32_t kb = kb0; kb < kb1; ++kb) {
          if (!ptx::mbar_wait_bounded(SPLIT ? &conv[stage] : &full[stage], phase,
                                      kWaitLimitNs)) {
            timeout();
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t sa = ptx::smem_addr(stage_base + stage * C::STAGE_BYTES);
          const uint32_t sb = sa + kA_BYTES;
          auto a_desc = [&](uint32_t base, int kk) {
            return A_MN ? ptx::smem_desc(base + kk * 1024, 4096, 512, ptx::kSwizzle128B32BAtom)
                        : ptx::smem_desc(base + kk * 32, 16, 1024, ptx::kSwizzle128B);
          };
          auto b_desc = [&](uint32_t base, int kk) {
            return B_MN ? ptx::smem_desc(base + kk * 1024, 4096, 512, ptx::kSwizzle128B32BAtom)
                        : ptx::smem_desc(base + kk * 32, 16, 1024, ptx::kSwizzle128B);
          };
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk) {
            const uint64_t ad = a_desc(sa, kk), bd = b_desc(sb, kk);
            const uint32_t acc_in = (kb != kb0 || kk != 0) ? 1u : 0u;
            if constexpr (SPLIT) {
              // small terms first, then the big product
              ptx::mma_tf32(d_tmem, ad, b_desc(sb + C::LOAD_BYTES, kk), idesc, acc_in);
              ptx::mma_tf32(d_tmem, a_desc(sa + C::LOAD_BYTES, kk), bd, idesc, 1u);
              ptx::mma_tf32(d_tmem, ad, bd, idesc, 1u);
            } else if constexpr (PAIR) {
              ptx::mma_tf32_pair(d_tmem, ad, bd, idesc, acc_in);
            } else {
              ptx::mma_tf32(d_tmem, ad, bd, idesc, acc_in);
            }
          }
          issued_any = true;
          // stage reusable (in both CTAs of a pair) once these MMAs finish
          if constexpr (PAIR) ptx::mma_commit_pair(&empty[stage], 0x3);
          else ptx::mma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        // accumulator ready for the epilogue (of both CTAs of a pair)
        if constexpr (PAIR) ptx::mma_commit_pair(&tfull[acc], 0x3);
        else ptx::mma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (*abort_flag && issued_any) {
        // let in-flight MMAs finish before TMEM is released
        if constexpr (PAIR) ptx::mma_commit_pair(&tfull[acc], 0x1);
        else ptx::mma_commit(&tfull[acc]);
        ptx::mbar_wait_bounded(&tfull[acc], acc_phase, kWaitLimitNs);
      }
    }
  } else if (SPLIT && warp >= 2 + kEpiWarps) {
    // ------------------------------------------------ 3xTF32 operand split
    // Each landed stage: x -> big = tf32(x) in place, small = tf32(x - big)
    // at the same offset in the stage's second half (x - big is exact).
    const uint32_t ct = threadIdx.x - (64 + 32 * kEpiWarps);
    uint32_t stage = 0, phase = 0;
    bool stop = false;
    for (uint64_t tile = blockIdx.x; tile < t.num_tiles && !stop && !*abort_flag;
         tile += gridDim.x) {
      uint64_t z;
      uint32_t s, mb, nb, kb0, kb1, grp;
      decode_tile(t, tile, z, s, mb, nb, grp);
      k_range(t, ktiles, s, kb0, kb1);
      for (uint32_t kb = kb0; kb < kb1; ++kb) {
        const bool got = ptx::mbar_wait_bounded(&full[stage], phase, kWaitLimitNs);
        if (!__all_sync(0xffffffffu, got)) {
          if (lane == 0) timeout();
          stop = true;
          break;
        }
        float4 *big = reinterpret_cast<float4 *>(stage_base + stage * C::STAGE_BYTES);
        float4 *small = big + C::LOAD_BYTES / 16;
#pragma unroll 4
        for (uint32_t i = ct; i < C::LOAD_BYTES / 16; i += 32 * kConvWarps) {
          const float4 x = big[i];
          const float4 h = make_float4(ptx::round_tf32(x.x), ptx::round_tf32(x.y),
                                       ptx::round_tf32(x.z), ptx::round_tf32(x.w));
          big[i] = h;
          small[i] = make_float4(ptx::round_tf32(x.x - h.x), ptx::round_tf32(x.y - h.y),
                                 ptx::round_tf32(x.z - h.z), ptx::round_tf32(x.w - h.w));
        }
        // generic-proxy writes, read next by the tensor cores (async proxy)
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&conv[stage]);
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------- epilogue
    // Warps 2..9: quadrant q = warp % 4 (the TMEM lanes a warp may read),
    // two warps per quadrant taking alternate 32-column chunks.
    const int q = warp & 3;
    const int e = warp - 2;
    const int c0 = e >> 2;
    uint32_t acc = 0, acc_phase = 0;
    uint8_t *obuf = out_base + e * C::BOXES * 4096;  // this warp's staging boxes
    uint32_t nbuf = 0, a_phase = 0;
    uint64_t *my_abar = &abar[e];
    // Tiles of at most 128 columns give a warp at most two chunks, one per
    // staging box, so the addend / GELU-backward boxes of the whole tile
    // are loaded before its accumulator is ready.
    constexpr bool kBoxPerChunk = C::BOXES == 2 && BN <= 128;
    const bool early_aux = kBoxPerChunk && t.tma_epi && t.partial == nullptr &&
                           (g.addend != nullptr || g.gelu_grad_x != nullptr) &&
                           g.gelu_out == nullptr;
    // a pair's first CTA counts both CTAs' releases of an accumulator
    auto release_acc = [&](uint32_t a) {
      if (PAIR && rank != 0) ptx::mbar_arrive_cluster(ptx::mapa_shared(&tempty[a], 0));
      else ptx::mbar_arrive(&tempty[a]);
    };
    for (uint64_t tile = tile0; tile < t.num_tiles; tile += tile_step) {
      uint64_t z;
      uint32_t s, mb, nb, grp;
      decode_tile(t, tile, z, s, mb, nb, grp);
      const uint32_t row0 = mb * C::BMT + rank * BM;  // this CTA's rows of the tile
      int32_t zc[3];
      int ncz;
      {
        int32_t cz[TL_GEMM_MAX_BATCH_RANK];
        batch_coords(g, z, cz);
        map_coords(t.mc, cz, zc);
        ncz = t.mc.nb;
      }
      uint32_t early_chunks = 0;
      if (early_aux) {
        for (int c = c0; c < BN / 32; c += 2) early_chunks += nb * BN + c * 32 < g.n;
        if (lane == 0 && early_chunks) {
          ptx::bulk_wait_group_read<0>();  // both boxes' stores have read them
          ptx::mbar_arrive_expect_tx(my_abar, early_chunks * 4096);
          for (uint32_t i = 0; i < early_chunks; ++i)
            ptx::tma_load_nd(obuf + i * 4096, &maps.addend, my_abar,
                             static_cast<int32_t>(nb * BN + (c0 + 2 * i) * 32),
                             static_cast<int32_t>(row0 + q * 32), ncz, zc);
        }
        __syncwarp();
      }
      // warp-uniform decisions: tcgen05.ld below needs all 32 lanes
      const bool got = ptx::mbar_wait_bounded(&tfull[acc], acc_phase, kWaitLimitNs);
      const bool aborting = !__all_sync(0xffffffffu, got) ||
                            __any_sync(0xffffffffu, *abort_flag != 0);
      if (early_chunks) {
        // the boxes are needed now, and must not be in flight at exit
        const bool got_add = ptx::mbar_wait_bounded(my_abar, a_phase, kWaitLimitNs);
        a_phase ^= 1;
        if (!__all_sync(0xffffffffu, got_add)) {
          if (lane == 0) timeout();
          break;
        }
      }
      if (!__all_sync(0xffffffffu, got)) {
        if (lane == 0) timeout();
        break;
      }
      if (aborting) break;
      ptx::tc_fence_after();
      uint64_t oa, ob, oc;
      batch_offsets(g, z, oa, ob, oc);
      // split-K slices store their raw partial product; the epilogue
      // (bias, accumulate, GELU) runs once in the slice-summing kernel
      const bool raw = t.partial != nullptr;
      const uint32_t slice = grp * t.splits + s;  // [groups][splits][M][N]
      float *Cb = raw ? t.partial + static_cast<size_t>(slice) * g.m * g.n : g.c + oc;
      // N groups: this tile's product has its own output and bias
      const float *bias = t.g.groups > 1 && !t.kgroups ? t.g.biasg[grp] : g.bias;
      const uint32_t m = row0 + q * 32 + lane;
      const uint32_t n_base = nb * BN;
      const bool row_ok = m < g.m;
      // 128-bit path: raw partials, or the full epilogue on float4 groups
      // (bias, accumulate and GELU in the same order as epilogue_store)
      const uint64_t ldo = raw ? g.n : g.ldc;  // split-K slices are dense
      const bool fast = (g.n % 4) == 0 && (ldo % 4) == 0 && aligned16(Cb) &&
                        (raw || ((!g.bias || aligned16(g.bias)) &&
                                 (!g.addend || aligned16(g.addend + oc)) &&
                                 (!g.gelu_grad_x || aligned16(g.gelu_grad_x + oc)) &&
                                 (!g.gelu_out || aligned16(g.gelu_out + oc))));
      if (t.tma_epi) {
        // Each chunk of 32 columns: TMEM -> registers (+ bias, + addend box
        // loaded by TMA into the staging box) -> swizzled staging box -> TMA
        // store of the 32 x 32 box (rows and columns past M, N are clipped).
        // A warp's boxes alternate (two per warp; one for 256-wide tiles) so
        // a store is in flight while the next box is filled.
        const int32_t y0 = static_cast<int32_t>(row0 + q * 32);
        if (raw) {  // split-K slices: [groups x splits][M][N]
          zc[0] = static_cast<int32_t>(slice);
          zc[1] = zc[2] = 0;
          ncz = 1;
        }
        // the addend box, or the GELU-backward input box (same map slot),
        // loaded by TMA into the staging box (L2 hits: the producer
        // prefetched the tile's boxes)
        const bool with_add = !raw && (g.addend != nullptr || g.gelu_grad_x != nullptr);
        const bool gelu_grad = !raw && g.gelu_grad_x != nullptr;
        const bool with_gelu = !raw && g.gelu_out != nullptr;
        bool failed = false;
#pragma unroll 1
        for (int c = c0; c < BN / 32; c += 2) {
          const uint32_t n0 = n_base + c * 32;
          if (n0 >= g.n) break;  // warp-uniform
          uint8_t *box;
          if (early_aux) {
            box = obuf + ((c - c0) >> 1) * 4096;  // loaded before the tile began
          } else {
            box = obuf + (C::BOXES == 2 ? (nbuf++ & 1u) * 4096 : 0);
            if (lane == 0) {  // the box's previous store has read it
              if constexpr (C::BOXES == 2) ptx::bulk_wait_group_read<1>();
              else ptx::bulk_wait_group_read<0>();
            }
            __syncwarp();
          }
          if (with_add && !early_aux) {
            if (lane == 0) {
              ptx::mbar_arrive_expect_tx(my_abar, 4096);
              ptx::tma_load_nd(box, &maps.addend, my_abar, static_cast<int32_t>(n0), y0, ncz, zc);
            }
            const bool got_add = ptx::mbar_wait_bounded(my_abar, a_phase, kWaitLimitNs);
            a_phase ^= 1;
            if (!__all_sync(0xffffffffu, got_add)) {
              if (lane == 0) timeout();
              failed = true;
            }
          }
          uint32_t r[32];
          ptx::tmem_load_32x32b_x32(tmem_base + acc * C::ACC_COLS + c * 32 + ((q * 32u) << 16), r);
          ptx::tmem_load_wait();
          if (failed) break;
          float4 v[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            v[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                               __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
            if (!raw && bias) {
              const uint32_t nb4 = n0 + 4 * j;
              if (nb4 + 4 <= g.n) {
                const float4 b = *reinterpret_cast<const float4 *>(bias + nb4);
                v[j] = make_float4(v[j].x + b.x, v[j].y + b.y, v[j].z + b.z, v[j].w + b.w);
              }
            }
            float4 *slot = reinterpret_cast<float4 *>(box + swz(lane, j));
            if (gelu_grad) {
              const float4 a = *slot;
              v[j] = make_float4(gelu_deriv_f(a.x) * v[j].x, gelu_deriv_f(a.y) * v[j].y,
                                 gelu_deriv_f(a.z) * v[j].z, gelu_deriv_f(a.w) * v[j].w);
            } else if (with_add) {
              const float4 a = *slot;
              v[j] = make_float4(a.x + v[j].x, a.y + v[j].y, a.z + v[j].z, a.w + v[j].w);
            }
            *slot = v[j];
          }
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (t.g.c_heads) {  // (head column, row in the head, head, row block)
              const uint32_t dh = g.n / g.c_heads, yr = static_cast<uint32_t>(y0);
              const int32_t hz[2] = {static_cast<int32_t>(n0 / dh),
                                     static_cast<int32_t>(yr / g.c_head_rows)};
              ptx::tma_store_nd(&maps.c[grp], box, static_cast<int32_t>(n0 % dh),
                                static_cast<int32_t>(yr % g.c_head_rows), 2, hz);
            } else {
              ptx::tma_store_nd(&maps.c[raw ? 0 : grp], box, static_cast<int32_t>(n0), y0, ncz,
                                zc);
            }
            ptx::bulk_commit_group();
          }
          if (with_gelu) {
            // the activations are computed while the store above reads
            // the box (the only one of a 256-wide tile's warp)
#pragma unroll
            for (int j = 0; j < 8; ++j)
              v[j] = make_float4(gelu_f(v[j].x), gelu_f(v[j].y), gelu_f(v[j].z), gelu_f(v[j].w));
            uint8_t *gbox = obuf + (C::BOXES == 2 ? (nbuf++ & 1u) * 4096 : 0);
            if (lane == 0) {
              if constexpr (C::BOXES == 2) ptx::bulk_wait_group_read<1>();
              else ptx::bulk_wait_group_read<0>();
            }
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 8; ++j) *reinterpret_cast<float4 *>(gbox + swz(lane, j)) = v[j];
            ptx::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              ptx::tma_store_nd(&maps.gelu, gbox, static_cast<int32_t>(n0), y0, ncz, zc);
              ptx::bulk_commit_group();
            }
          }
        }
        ptx::tc_fence_before();
        release_acc(acc);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
        if (failed) break;
        continue;
      }
#pragma unroll 1
      for (int c = c0; c < BN / 32; c += 2) {
        uint32_t r[32];
        ptx::tmem_load_32x32b_x32(tmem_base + acc * C::ACC_COLS + c * 32 + ((q * 32u) << 16), r);
        ptx::tmem_load_wait();
        const uint32_t n0 = n_base + c * 32;
        if (!row_ok || n0 >= g.n) continue;
        const size_t rowoff = static_cast<size_t>(m) * ldo;
        if (fast && n0 + 32 <= g.n) {
          float4 *dst = reinterpret_cast<float4 *>(Cb + rowoff + n0);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float4 v = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                   __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
            if (!raw) {
              if (g.bias) {
                const float4 b = *reinterpret_cast<const float4 *>(g.bias + n0 + 4 * j);
                v = make_float4(v.x + b.x, v.y + b.y, v.z + b.z, v.w + b.w);
              }
              if (g.addend) {
                const float4 o =
                    *reinterpret_cast<const float4 *>(g.addend + oc + rowoff + n0 + 4 * j);
                v = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
              }
              if (g.gelu_grad_x) {
                const float4 x =
                    *reinterpret_cast<const float4 *>(g.gelu_grad_x + oc + rowoff + n0 + 4 * j);
                v = make_float4(gelu_deriv_f(x.x) * v.x, gelu_deriv_f(x.y) * v.y,
                                gelu_deriv_f(x.z) * v.z, gelu_deriv_f(x.w) * v.w);
              }
            }
            dst[j] = v;
            if (!raw && g.gelu_out)
              *reinterpret_cast<float4 *>(g.gelu_out + oc + rowoff + n0 + 4 * j) =
                  make_float4(gelu_f(v.x), gelu_f(v.y), gelu_f(v.z), gelu_f(v.w));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const uint32_t n = n0 + j;
            if (n >= g.n) continue;
            if (raw) Cb[rowoff + n] = __uint_as_float(r[j]);
            else epilogue_store(g, Cb, oc, rowoff + n, n, __uint_as_float(r[j]));
          }
        }
      }
      ptx::tc_fence_before();
      release_acc(acc);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  // every TMA store issued by this CTA has written its box before exit
  if (warp >= 2 && lane == 0) ptx::bulk_wait_group<0>();
  ptx::tc_fence_before();
  __syncthreads();
  // a pair: neither CTA leaves while the other may still use its shared
  // memory (products) or barriers (loads, releases)
  if constexpr (PAIR) ptx::cluster_sync();
  ptx::tc_fence_after();
  if (warp == 1) {
    if constexpr (PAIR) ptx::tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    else ptx::tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side
EncodeTiledFn encode_fn() { return tensor_map_encoder(); }

// Map of a stored matrix [outer][inner] (row stride ld elements) and the
// batch dims of `strides` that are not broadcast (stride 0), box
// box_inner x box_outer.  Fills `om` with those dims; false when TMA cannot
// describe the operand (more than three such dims, or encoding refused).
bool make_operand_map(CUtensorMap *map, const float *base, uint64_t inner, uint64_t outer,
                      uint64_t ld, const GemmArgs &g, const uint64_t *strides,
                      uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz,
                      OpMap &om, uint32_t chunks = 0) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  om = OpMap{};
  int nb = 0;
  for (uint32_t d = 0; d < g.batch_rank; ++d)
    if (strides[d] != 0) {
      if (nb == 3) return false;
      om.dim[nb++] = static_cast<int32_t>(d);
    }
  om.nb = nb;
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  if (chunks && inner % 32 == 0 && nb <= 2) {
    // [MN/32 chunks][K][32]: one load brings `chunks` 32 x 32 boxes, laid
    // out one after another exactly as `chunks` separate loads would
    cuuint64_t dims[5] = {32, outer, inner / 32, 1, 1};
    cuuint64_t st[4] = {ld * 4, 128, 0, 0};
    int rank = 3;
    for (int i = 0; i < nb; ++i) {
      dims[rank] = g.batch_shape[om.dim[i]];
      st[rank - 1] = strides[om.dim[i]] * 4;
      ++rank;
    }
    const cuuint32_t box[5] = {32, box_outer, chunks, 1, 1};
    if (enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, const_cast<float *>(base), dims, st, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS) {
      om.chunked = static_cast<int32_t>(chunks);
      return true;
    }
  }
  cuuint64_t dims[5] = {inner, outer, 1, 1, 1};
  cuuint64_t st[4] = {ld * 4, 0, 0, 0};
  int rank = 2;
  for (int i = 0; i < nb; ++i) {
    dims[rank] = g.batch_shape[om.dim[i]];
    st[rank - 1] = strides[om.dim[i]] * 4;
    ++rank;
  }
  const cuuint32_t box[5] = {box_inner, box_outer, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, const_cast<float *>(base), dims, st,
             box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Slice sums of a split-K product in slice order, then the epilogue; one
// launch for all groups of an N-grouped product (blockIdx.y: group, whose
// slices follow the previous group's).  VEC: four columns per thread (N,
// ldc and every epilogue operand 16-byte aligned).
template <bool VEC>
__global__ void __launch_bounds__(256)
splitk_epilogue_kernel(const float *__restrict__ part, uint32_t splits, uint32_t ngroups,
                       const GemmArgs g) {
  pdl_enter();
  const uint32_t grp = blockIdx.y;
  float *C = ngroups > 1 ? g.cg[grp] : g.c;
  const float *bias = ngroups > 1 ? g.biasg[grp] : g.bias;
  const uint64_t mn = static_cast<uint64_t>(g.m) * g.n;
  const float *P = part + static_cast<uint64_t>(grp) * splits * mn;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  const uint64_t count = VEC ? mn / 4 : mn;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += stride) {
    if constexpr (VEC) {
      const uint64_t e = 4 * i;
      float4 v = __ldcg(reinterpret_cast<const float4 *>(P + e));
      for (uint32_t s = 1; s < splits; ++s) {
        const float4 w = __ldcg(reinterpret_cast<const float4 *>(P + s * mn + e));
        v.x += w.x;
        v.y += w.y;
        v.z += w.z;
        v.w += w.w;
      }
      const uint32_t n = static_cast<uint32_t>(e % g.n);
      const size_t idx = (e / g.n) * g.ldc + n;
      epilogue_store(g, C, bias, 0, idx, n, v.x);
      epilogue_store(g, C, bias, 0, idx + 1, n + 1, v.y);
      epilogue_store(g, C, bias, 0, idx + 2, n + 2, v.z);
      epilogue_store(g, C, bias, 0, idx + 3, n + 3, v.w);
    } else {
      float v = P[i];
      for (uint32_t s = 1; s < splits; ++s) v += P[s * mn + i];
      const uint32_t n = static_cast<uint32_t>(i % g.n);
      epilogue_store(g, C, bias, 0, (i / g.n) * g.ldc + n, n, v);
    }
  }
}

struct TcPlan {
  int bn;
  uint32_t splits, kb_per_split;
  size_t workspace;
  bool pair;  // 256-row tiles on CTA pairs (cta_group::2)
};

TcPlan plan_width(const GemmArgs &g, int max_bn) {
  TcPlan p{};
  p.bn = g.n > 128 ? max_bn : (g.n > 64 ? 128 : 64);
  // Enough tiles for every SM: pick the tile width with the least work per
  // SM, waves x (width + a fixed per-tile cost of ~64 columns), so N = 384
  // runs as 3 x 128 instead of 2 x 256 with a quarter of the MMAs wasted,
  // and the attention products (N = 192) as one 192-wide tile.
  const uint64_t mt = (g.m + BM - 1) / BM;
  const bool kgroups = g.groups > 1 && g.group_mode == TL_GEMM_GROUP_K;
  const uint64_t outs = g.batch_count * (g.groups > 1 && !kgroups ? g.groups : 1);
  if (outs * mt * ((g.n + 255) / 256) >= static_cast<uint64_t>(kNumSMs) / 2) {
    uint64_t best = ~0ull;
    for (int bn : {64, 128, 192, 256}) {
      if (bn > max_bn) continue;
      const uint64_t tiles = outs * mt * ((g.n + bn - 1) / bn);
      const uint64_t cost = (tiles + kNumSMs - 1) / kNumSMs * (bn + 64);
      if (cost < best) {
        best = cost;
        p.bn = bn;
      }
    }
  }
  const uint64_t tiles = outs * ((g.m + BM - 1) / BM) * ((g.n + p.bn - 1) / p.bn);
  const uint32_t ktiles = (g.k + BK - 1) / BK * (kgroups ? g.groups : 1);
  p.splits = 1;
  p.kb_per_split = ktiles;
  // Few output tiles but a long K (weight gradients: K = every token of the
  // batch): cut K into slices of at least 8 k-tiles (256 of K).  The grid
  // is persistent, one CTA per SM, so tiles x slices stay within one wave
  // (148 + 14 CTAs would run a second pass of 14); the tile width and the
  // slice count are picked together for the least work per SM, waves x
  // k-tiles per slice x (width + ~64 columns of fixed cost): N = 384 as two
  // 192-wide tiles, not two 256-wide ones with a quarter of the MMAs wasted.
  if (g.batch_count == 1 && tiles < static_cast<uint64_t>(kNumSMs) / 2 && ktiles >= 16 &&
      !g.c_heads) {
    uint64_t best = ~0ull;
    const uint64_t mt = (g.m + BM - 1) / BM;
    for (int bn : {64, 128, 192, 256}) {
      if (bn > max_bn || (bn < p.bn && bn < 128) || (bn >= 2 * static_cast<int>(g.n) && bn > 64))
        continue;
      const uint64_t tl = outs * mt * ((g.n + bn - 1) / bn);
      uint64_t want = kNumSMs / tl;
      if (want > ktiles / 8) want = ktiles / 8;
      if (want < 1) want = 1;
      const uint64_t kb = (ktiles + want - 1) / want;
      const uint64_t splits = (ktiles + kb - 1) / kb;
      const uint64_t waves = (tl * splits + kNumSMs - 1) / kNumSMs;
      const uint64_t cost = waves * kb * static_cast<uint64_t>(bn + 64);
      if (cost < best) {
        best = cost;
        p.bn = bn;
        p.kb_per_split = static_cast<uint32_t>(kb);
        p.splits = static_cast<uint32_t>(splits);
      }
    }
    if (p.splits > 1)
      p.workspace = static_cast<size_t>(p.splits) * (outs / g.batch_count) * g.m * g.n *
                    sizeof(float);
  }
  return p;
}

// Map of a head-split C ([M / R, H, R, Dh], tl_gemm_desc.c_heads) as the
// 4-D tensor (Dh, R, H, M / R), boxes of 32 x 32 (head columns x rows).
bool make_head_map(CUtensorMap *map, float *base, const GemmArgs &g) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  const uint64_t H = g.c_heads, R = g.c_head_rows, Dh = g.n / g.c_heads;
  const cuuint64_t dims[4] = {Dh, R, H, g.m / R};
  const cuuint64_t st[3] = {Dh * 4, R * Dh * 4, H * R * Dh * 4};
  const cuuint32_t box[4] = {32, 32, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, dims, st, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// Whether CTA pairs should take the product: 256-row tiles halve the B
// columns each SM loads per k-step (the operand fill from L2 bounds the
// small-K products), for unsplit TF32 products with many full 256-row
// tiles: at least one wave of pairs.
bool use_pairs(const GemmArgs &g, const TcPlan &p) {
  if (g.split_tf32 || p.splits != 1 || g.m % 256 || (p.bn != 128 && p.bn != 256)) return false;
  static const bool enabled = [] {
    const char *e = std::getenv("TL_GEMM_PAIRS");
    return e && std::strcmp(e, "1") == 0;
  }();
  if (!enabled) return false;
  const bool kgroups = g.groups > 1 && g.group_mode == TL_GEMM_GROUP_K;
  const uint64_t outs = g.batch_count * (g.groups > 1 && !kgroups ? g.groups : 1);
  const uint64_t tiles = outs * (g.m / 256) * ((g.n + p.bn - 1) / p.bn);
  return tiles >= static_cast<uint64_t>(kNumSMs) / 2;
}

TcPlan plan_tc(const GemmArgs &g) {
  // 3xTF32 stages are twice as large: tiles of at most 128 columns
  TcPlan p = plan_width(g, g.split_tf32 ? 128 : 256);
  if (p.bn == 192) {  // pairs split the columns of B in halves of 32-multiples
    const TcPlan q = plan_width(g, 128);
    if (use_pairs(g, q)) p = q;
  }
  p.pair = use_pairs(g, p);
  // An epilogue that loads a box per chunk (addend, GELU-backward input)
  // loads all of a tile's boxes while the tile's MMAs run when it has a
  // staging box per chunk, which only tiles up to 128 wide have.  Only
  // unsplit products narrow their tiles: the K slicing, and so the
  // summation order, stays the one the same product has without epilogue.
  // TL_GEMM_EPI_TILES (tuning): 0 keeps the widest tile for these products
  // too, 2 also narrows the GELU-output products (two staging boxes per
  // warp: the pre-activation and the activation stores overlap).
  static const int epi_tiles = [] {
    const char *e = std::getenv("TL_GEMM_EPI_TILES");
    return e ? std::atoi(e) : 1;
  }();
  const bool narrow = epi_tiles >= 1 && (g.addend || g.gelu_grad_x) && !g.gelu_out;
  const bool narrow_gelu = epi_tiles >= 2 && g.gelu_out;
  if (p.splits == 1 && (narrow || narrow_gelu)) {
    TcPlan q = plan_width(g, 128);
    q.pair = use_pairs(g, q);
    if (q.splits == 1) return q;
  }
  return p;
}

template <int BN, bool A_MN, bool B_MN, bool SPLIT, bool PAIR, int BX = 0>
int launch_variant(const GemmArgs &g, const TcPlan &plan, float *partial, cudaStream_t s) {
  using C = Cfg<BN, SPLIT, PAIR, BX>;
  TcArgs t{};
  t.g = g;
  t.mt = (g.m + C::BMT - 1) / C::BMT;
  t.nt = (g.n + BN - 1) / BN;
  t.kgroups = g.groups > 1 && g.group_mode == TL_GEMM_GROUP_K;
  t.kb_per_group = (g.k + BK - 1) / BK;
  const uint32_t ktiles = t.kgroups ? g.groups * t.kb_per_group : t.kb_per_group;
  if (t.kgroups && g.k % BK) return fail(TL_ERR_UNSUPPORTED, "tl_gemm: K groups need k % 32 == 0");
  t.splits = partial ? plan.splits : 1;
  t.kb_per_split = partial ? plan.kb_per_split : ktiles;
  t.partial = partial;
  const uint64_t per_group = g.batch_count * t.splits * t.mt * t.nt;
  const uint32_t ngroups = g.groups > 1 && !t.kgroups ? g.groups : 1;
  t.num_tiles = per_group * ngroups;
  if (t.num_tiles >= (1ull << 32)) return fail(TL_ERR_UNSUPPORTED, "tl_gemm: too many tiles");
  t.tiles_per_group = static_cast<uint32_t>(per_group);
  t.status = device_status_ptr();
  if (!t.status) return fail(TL_ERR_CUDA, "tl_gemm: no status word");
  TcMaps maps{};
  bool ok = true;
  for (uint32_t i = 0; i < g.groups && ok; ++i) {
    if (i == 0 || t.kgroups)
      ok = A_MN ? make_operand_map(&maps.a[i], g.ag[i] ? g.ag[i] : g.a, g.m, g.k, g.lda, g, g.sa,
                                   32, 32, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, t.ma, BM / 32)
                : make_operand_map(&maps.a[i], g.ag[i] ? g.ag[i] : g.a, g.k, g.m, g.lda, g, g.sa,
                                   32, BM, CU_TENSOR_MAP_SWIZZLE_128B, t.ma);
    ok = ok && (B_MN ? make_operand_map(&maps.b[i], g.bg[i] ? g.bg[i] : g.b, g.n, g.k, g.ldb, g,
                                        g.sb, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, t.mb,
                                        C::BN_LOAD / 32)
                     : make_operand_map(&maps.b[i], g.bg[i] ? g.bg[i] : g.b, g.k, g.n, g.ldb, g,
                                        g.sb, 32, C::BN_LOAD, CU_TENSOR_MAP_SWIZZLE_128B, t.mb));
  }
  if (!ok) return fail(TL_ERR_UNSUPPORTED, "tl_gemm: tensor map rejected");
  // epilogue through TMA stores when C (and gelu_out, addend: same layout)
  // have 16-byte rows; otherwise per-thread stores
  if (partial) {
    GemmArgs slices = g;  // [groups x splits][M][N], dense
    slices.batch_rank = 1;
    slices.batch_shape[0] = t.splits * ngroups;
    const uint64_t mn = static_cast<uint64_t>(g.m) * g.n;
    OpMap unused;
    t.tma_epi = g.n % 4 == 0 &&
                make_operand_map(&maps.c[0], partial, g.n, g.m, g.n, slices, &mn, 32, 32,
                                 CU_TENSOR_MAP_SWIZZLE_128B, unused);
  } else {
    bool strides_ok = g.ldc % 4 == 0;
    for (uint32_t d = 0; d < g.batch_rank; ++d) strides_ok = strides_ok && g.sc[d] % 4 == 0;
    const float *aux = g.addend ? g.addend : g.gelu_grad_x;  // one epilogue input box
    OpMap og{}, od{};
    t.tma_epi = g.n % 4 == 0 && strides_ok && aligned16(g.c) &&
                (!g.bias || aligned16(g.bias)) && (!g.gelu_out || aligned16(g.gelu_out)) &&
                (!g.addend || aligned16(g.addend)) &&
                (!g.gelu_grad_x || aligned16(g.gelu_grad_x)) &&
                (!g.gelu_out || make_operand_map(&maps.gelu, g.gelu_out, g.n, g.m, g.ldc, g,
                                                 g.sc, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B, og)) &&
                (!aux || make_operand_map(&maps.addend, aux, g.n, g.m, g.ldc, g, g.sc, 32, 32,
                                          CU_TENSOR_MAP_SWIZZLE_128B, od));
    for (uint32_t i = 0; i < ngroups && t.tma_epi; ++i) {
      float *ci = g.cg[i] ? g.cg[i] : g.c;
      const float *bi = g.groups > 1 ? g.biasg[i] : g.bias;
      t.tma_epi = aligned16(ci) && (!bi || aligned16(bi)) &&
                  (g.c_heads ? make_head_map(&maps.c[i], ci, g)
                             : make_operand_map(&maps.c[i], ci, g.n, g.m, g.ldc, g, g.sc, 32,
                                                32, CU_TENSOR_MAP_SWIZZLE_128B, t.mc));
    }
  }
  if (g.c_heads && !t.tma_epi)
    return fail(TL_ERR_UNSUPPORTED, "tl_gemm: head-split store needs the TMA epilogue");
  t.aux_prefetch = t.tma_epi && !partial && (g.addend || g.gelu_grad_x);
  // grouped outputs leave only through the TMA epilogue
  if (ngroups > 1 && !t.tma_epi)
    return fail(TL_ERR_UNSUPPORTED, "tl_gemm: grouped outputs need 16-byte rows");
  static bool attr_set = false;
  if (!attr_set) {
    int rc = check_cuda(cudaFuncSetAttribute(tc_gemm_kernel<BN, A_MN, B_MN, SPLIT, PAIR, BX>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(C::SMEM)),
                        "tl_gemm smem attribute");
    if (rc) return rc;
    attr_set = true;
  }
  if constexpr (PAIR) {
    const uint64_t pairs = kNumSMs / 2;
    const uint64_t grid = 2 * (t.num_tiles < pairs ? t.num_tiles : pairs);
    launch_pdl_cluster(tc_gemm_kernel<BN, A_MN, B_MN, SPLIT, PAIR, BX>, static_cast<unsigned>(grid),
                       C::THREADS, C::SMEM, s, 2u, maps, t);
  } else {
    const uint64_t grid = t.num_tiles < static_cast<uint64_t>(kNumSMs) ? t.num_tiles : kNumSMs;
    launch_pdl(tc_gemm_kernel<BN, A_MN, B_MN, SPLIT, PAIR, BX>, static_cast<unsigned>(grid),
               C::THREADS, C::SMEM, s, maps, t);
  }
  int rc = launch_status("tl_gemm tf32");
  if (rc || !partial) return rc;
  const uint64_t mn = static_cast<uint64_t>(g.m) * g.n;
  bool vec = g.n % 4 == 0 && g.ldc % 4 == 0;
  for (uint32_t i = 0; i < ngroups && vec; ++i) {
    const float *ci = ngroups > 1 ? g.cg[i] : g.c;
    const float *bi = ngroups > 1 ? g.biasg[i] : g.bias;
    vec = aligned16(ci) && (!bi || aligned16(bi));
  }
  vec = vec && (!g.addend || aligned16(g.addend)) && (!g.gelu_out || aligned16(g.gelu_out)) &&
        (!g.gelu_grad_x || aligned16(g.gelu_grad_x));
  const dim3 grid(vec ? grid_for(mn / 4, 256) : grid_for(mn, 256), ngroups);
  if (vec)
    launch_pdl(splitk_epilogue_kernel<true>, grid, 256, 0, s, partial, t.splits, ngroups, g);
  else
    launch_pdl(splitk_epilogue_kernel<false>, grid, 256, 0, s, partial, t.splits, ngroups, g);
  return launch_status("tl_gemm split-K sum");
}

template <int BN, bool SPLIT = false, bool PAIR = false>
int launch_bn(const GemmArgs &g, const TcPlan &plan, float *partial, cudaStream_t s) {
  const bool a_mn = g.trans_a != 0, b_mn = g.trans_b == 0;
  if (a_mn && b_mn) return launch_variant<BN, true, true, SPLIT, PAIR>(g, plan, partial, s);
  if (a_mn) return launch_variant<BN, true, false, SPLIT, PAIR>(g, plan, partial, s);
  if (b_mn) return launch_variant<BN, false, true, SPLIT, PAIR>(g, plan, partial, s);
  return launch_variant<BN, false, false, SPLIT, PAIR>(g, plan, partial, s);
}

}  // namespace

bool tc_gemm_supported(const GemmArgs &g) {
  // TMA rules: 16-byte aligned bases, row strides and batch strides; at
  // most three walked batch dims per operand.
  if (g.k == 0 || g.lda % 4 || g.ldb % 4 || !aligned16(g.a) || !aligned16(g.b)) return false;
  for (uint32_t i = 0; i < g.groups; ++i)
    if ((g.ag[i] && !aligned16(g.ag[i])) || (g.bg[i] && !aligned16(g.bg[i]))) return false;
  int na = 0, nb = 0;
  for (uint32_t d = 0; d < g.batch_rank; ++d) {
    if (g.sa[d] % 4 || g.sb[d] % 4) return false;
    na += g.sa[d] != 0;
    nb += g.sb[d] != 0;
  }
  return na <= 3 && nb <= 3 && g.m <= 0x7fffffffu && g.n <= 0x7fffffffu &&
         g.k <= 0x7fffffffu;
}

size_t tc_gemm_workspace(const GemmArgs &g) {
  return tc_gemm_supported(g) ? plan_tc(g).workspace : 0;
}

int launch_tc_gemm(const GemmArgs &g, void *workspace, size_t workspace_bytes, cudaStream_t s) {
  if (!tc_gemm_supported(g)) return TL_ERR_UNSUPPORTED;
  const TcPlan plan = plan_tc(g);
  // without room for the slices the product runs unsplit (same result)
  float *partial = plan.splits > 1 && workspace && workspace_bytes >= plan.workspace &&
                           aligned16(workspace)
                       ? static_cast<float *>(workspace)
                       : nullptr;
  if (g.split_tf32)
    return plan.bn == 128 ? launch_bn<128, true>(g, plan, partial, s)
                          : launch_bn<64, true>(g, plan, partial, s);
  if (plan.pair)
    return plan.bn == 256 ? launch_bn<256, false, true>(g, plan, partial, s)
                          : launch_bn<128, false, true>(g, plan, partial, s);
  // the FFN's first product (NN, unsplit, GELU output) with two boxes per
  // warp: opt-in (TL_GEMM_EPI2=1), measured no faster than one box (63.5 us
  // both at 12288 x 1536 x 384, 96.2 us both at 8192 x 3072 x 768)
  static const bool epi2 = [] {
    const char *e = std::getenv("TL_GEMM_EPI2");
    return e && std::strcmp(e, "1") == 0;
  }();
  if (plan.bn == 256 && epi2 && g.gelu_out && !g.trans_a && !g.trans_b && !partial)
    return launch_variant<256, false, true, false, false, 2>(g, plan, partial, s);
  if (plan.bn == 256) return launch_bn<256>(g, plan, partial, s);
  if (plan.bn == 192) return launch_bn<192>(g, plan, partial, s);
  // 128-wide products whose epilogue reads no box: one staging box per
  // warp and one more pipeline stage (TL_GEMM_BOX1=1, tuning)
  static const bool box1 = [] {
    const char *e = std::getenv("TL_GEMM_BOX1");
    return e && std::strcmp(e, "1") == 0;
  }();
  if (plan.bn == 128 && box1 && !g.addend && !g.gelu_grad_x && !g.gelu_out) {
    const bool a_mn = g.trans_a != 0, b_mn = g.trans_b == 0;
    if (a_mn && b_mn) return launch_variant<128, true, true, false, false, 1>(g, plan, partial, s);
    if (a_mn) return launch_variant<128, true, false, false, false, 1>(g, plan, partial, s);
    if (b_mn) return launch_variant<128, false, true, false, false, 1>(g, plan, partial, s);
    return launch_variant<128, false, false, false, false, 1>(g, plan, partial, s);
  }
  if (plan.bn == 128) return launch_bn<128>(g, plan, partial, s);
  return launch_bn<64>(g, plan, partial, s);
}

}  // namespace tl

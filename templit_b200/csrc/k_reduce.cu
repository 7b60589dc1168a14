// Shape reductions (sum_to_shape / max_to_shape / sum) and argmax.
//
// The reference reduces with one thread per output element walking every
// reduced element serially (include/my_metal/math.metal:618-714), and argmax
// with 16-element chunks over several dispatches (math.metal:715-777).  Here
// the host classifies the kept (K) and reduced (R) dimensions after merging
// neighbours of the same class:
//   [K, R]      row reduction   - one warp per row, or split rows + a second pass
//   [K1, R, K2] column reduction - threads along K2 (4-wide), R split over CTAs
//               with a second pass when the output alone cannot fill the GPU
//   other       generic         - one thread per output (rare shapes)
// Every plan is deterministic: partial results land in a workspace and are
// combined in a fixed order.
#include "tl_common.cuh"

#include <atomic>
#include <mutex>

#include <cfloat>

namespace tl {
namespace {

template <int OP>
__device__ __forceinline__ float rinit() {
  return OP == TL_REDUCE_SUM ? 0.0f : -INFINITY;
}
template <int OP>
__device__ __forceinline__ float rcomb(float a, float b) {
  return OP == TL_REDUCE_SUM ? a + b : fmaxf(a, b);
}
template <int OP>
__device__ __forceinline__ float warp_reduce(float v) {
  return OP == TL_REDUCE_SUM ? warp_sum(v) : warp_max(v);
}

// out[row * out_stride + split] = reduce(x[row, split chunk]).
// One warp per (row, split); chunk = ceil(cols / splits) rounded to 4.
template <int OP>
__global__ void __launch_bounds__(256)
rows_kernel(const float *__restrict__ x, float *out, uint32_t rows,
            uint32_t cols, uint32_t splits, uint32_t chunk, bool vec) {
  pdl_enter();
  const uint32_t warps = (blockDim.x / 32) * gridDim.x;
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t total = static_cast<uint64_t>(rows) * splits;
  for (uint64_t w = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; w < total;
       w += warps) {
    const uint32_t row = static_cast<uint32_t>(w / splits);
    const uint32_t sp = static_cast<uint32_t>(w % splits);
    const uint32_t c0 = sp * chunk;
    const uint32_t c1 = min(cols, c0 + chunk);
    const float *xr = x + static_cast<size_t>(row) * cols;
    float acc = rinit<OP>();
    if (vec) {
      for (uint32_t c = c0 + lane * 4; c < c1; c += 128) {
        const float4 v = *reinterpret_cast<const float4 *>(xr + c);
        acc = rcomb<OP>(acc, rcomb<OP>(rcomb<OP>(v.x, v.y), rcomb<OP>(v.z, v.w)));
      }
    } else {
      for (uint32_t c = c0 + lane; c < c1; c += 32) acc = rcomb<OP>(acc, xr[c]);
    }
    acc = warp_reduce<OP>(acc);
    if (lane == 0) out[w] = acc;
  }
}

// out[k1, k2] (+ split s: part[s, k1, k2]) = reduce over r in [r0, r1) of
// x[k1, r, k2].  Threads own 4 consecutive k2 when vec.
template <int OP, int V>
__global__ void __launch_bounds__(256)
cols_kernel(const float *__restrict__ x, float *out, uint32_t K1, uint32_t R,
            uint32_t K2, uint32_t splits, uint32_t rchunk) {
  pdl_enter();
  const uint32_t k2v = K2 / V;
  const uint64_t per_split = static_cast<uint64_t>(K1) * k2v;
  const uint64_t total = per_split * splits;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       t < total; t += stride) {
    const uint32_t s = static_cast<uint32_t>(t / per_split);
    const uint64_t rem = t % per_split;
    const uint32_t k1 = static_cast<uint32_t>(rem / k2v);
    const uint32_t k2 = static_cast<uint32_t>(rem % k2v) * V;
    const uint32_t r0 = s * rchunk;
    const uint32_t r1 = min(R, r0 + rchunk);
    const float *base = x + (static_cast<size_t>(k1) * R) * K2 + k2;
    if constexpr (V == 4) {
      float4 acc = make_float4(rinit<OP>(), rinit<OP>(), rinit<OP>(), rinit<OP>());
#pragma unroll 8
      for (uint32_t r = r0; r < r1; ++r) {
        const float4 v = *reinterpret_cast<const float4 *>(base + static_cast<size_t>(r) * K2);
        acc.x = rcomb<OP>(acc.x, v.x);
        acc.y = rcomb<OP>(acc.y, v.y);
        acc.z = rcomb<OP>(acc.z, v.z);
        acc.w = rcomb<OP>(acc.w, v.w);
      }
      *reinterpret_cast<float4 *>(out + s * static_cast<size_t>(K1) * K2 +
                                  static_cast<size_t>(k1) * K2 + k2) = acc;
    } else {
      float acc = rinit<OP>();
      for (uint32_t r = r0; r < r1; ++r) acc = rcomb<OP>(acc, base[static_cast<size_t>(r) * K2]);
      out[s * static_cast<size_t>(K1) * K2 + static_cast<size_t>(k1) * K2 + k2] = acc;
    }
  }
}

// Arrival counters of the single-launch column reduction: one per (k1,
// column block), back at zero after every launch (atomicInc wraps), so the
// launches of a stream reuse them; reductions that run concurrently on
// several streams must not share the library (documented in the header).
constexpr uint32_t kColTickets = 1u << 16;
static __device__ unsigned int g_col_tickets[kColTickets];

// [K1, R, K2] column reduction by blocks: CTA (c, k1, cb) folds rows
// [c * rchunk, (c + 1) * rchunk) of columns [128 cb, 128 cb + 128): warp w
// takes rows w, w + 8, ... (float4 per lane, 128-byte rows per warp) and the
// 8 warp results are folded in warp order, so each split costs one pass over
// its rows with all 8 warps' loads in flight and the order is fixed.  With
// `fold` (several splits), the partial goes to part[c]; the last CTA of the
// (k1, column block) to finish folds all splits' partials in split order
// into out, in the same launch.
// Grouped (g.grouped): blockIdx.y picks one of up to TL_REDUCE_MAX_GROUPS
// independent [R, K2] reductions (K1 = 1), each with its own input,
// partials and output; otherwise blockIdx.y is k1 of the one reduction.
struct ColsGroups {
  const float *x[TL_REDUCE_MAX_GROUPS];
  float *part[TL_REDUCE_MAX_GROUPS];      // partials (`out` below)
  float *fold_out[TL_REDUCE_MAX_GROUPS];  // null: no in-launch fold
  uint32_t grouped;
};

template <int OP>
__global__ void __launch_bounds__(256)
cols_block_kernel(const __grid_constant__ ColsGroups g, uint32_t K1, uint32_t R, uint32_t K2,
                  uint32_t rchunk) {
  pdl_enter();
  __shared__ float4 part[8][32];
  __shared__ bool last;
  const uint32_t gi = g.grouped ? blockIdx.y : 0;
  const float *__restrict__ x = g.x[gi];
  float *out = g.part[gi];
  float *fold_out = g.fold_out[gi];
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t c = blockIdx.x, k1 = g.grouped ? 0 : blockIdx.y;
  const uint32_t col = blockIdx.z * 128 + lane * 4;
  const uint32_t r0 = c * rchunk, r1 = min(R, r0 + rchunk);
  float4 acc = make_float4(rinit<OP>(), rinit<OP>(), rinit<OP>(), rinit<OP>());
  if (col < K2) {
    const float *base = x + static_cast<size_t>(k1) * R * K2 + col;
    // 16 rows per warp in flight: loads first, then the adds in row order
    uint32_t r = r0 + warp;
    for (; r + 15 * 8 < r1; r += 16 * 8) {
      float4 v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        v[i] = __ldcs(reinterpret_cast<const float4 *>(base + static_cast<size_t>(r + 8 * i) * K2));
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        acc.x = rcomb<OP>(acc.x, v[i].x);
        acc.y = rcomb<OP>(acc.y, v[i].y);
        acc.z = rcomb<OP>(acc.z, v[i].z);
        acc.w = rcomb<OP>(acc.w, v[i].w);
      }
    }
    for (; r < r1; r += 8) {
      const float4 v = *reinterpret_cast<const float4 *>(base + static_cast<size_t>(r) * K2);
      acc.x = rcomb<OP>(acc.x, v.x);
      acc.y = rcomb<OP>(acc.y, v.y);
      acc.z = rcomb<OP>(acc.z, v.z);
      acc.w = rcomb<OP>(acc.w, v.w);
    }
  }
  part[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && col < K2) {
    float4 r = part[0][lane];
#pragma unroll
    for (int w = 1; w < 8; ++w) {
      const float4 v = part[w][lane];
      r.x = rcomb<OP>(r.x, v.x);
      r.y = rcomb<OP>(r.y, v.y);
      r.z = rcomb<OP>(r.z, v.z);
      r.w = rcomb<OP>(r.w, v.w);
    }
    *reinterpret_cast<float4 *>(out + static_cast<size_t>(c) * K1 * K2 +
                                static_cast<size_t>(k1) * K2 + col) = r;
  }
  if (!fold_out) return;
  // publish this split's partial, then count arrivals of the column block
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned slot = blockIdx.y * gridDim.z + blockIdx.z;
    last = ticket_acq_rel(&g_col_tickets[slot], gridDim.x - 1) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  // fold the splits: warp w takes splits w, w + 8, ... in order, then the
  // warp results in warp order (the order is fixed: deterministic)
  const size_t plane = static_cast<size_t>(K1) * K2;
  float4 a = make_float4(rinit<OP>(), rinit<OP>(), rinit<OP>(), rinit<OP>());
  if (col < K2) {
    const float *src = out + static_cast<size_t>(k1) * K2 + col;
    // up to 16 of the warp's partials loaded at once, then added in order
    for (uint32_t sp0 = warp; sp0 < gridDim.x; sp0 += 16 * 8) {
      float4 v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t sp = sp0 + 8 * i;
        v[i] = sp < gridDim.x ? __ldcg(reinterpret_cast<const float4 *>(src + sp * plane))
                              : make_float4(rinit<OP>(), rinit<OP>(), rinit<OP>(), rinit<OP>());
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        a.x = rcomb<OP>(a.x, v[i].x);
        a.y = rcomb<OP>(a.y, v[i].y);
        a.z = rcomb<OP>(a.z, v[i].z);
        a.w = rcomb<OP>(a.w, v[i].w);
      }
    }
  }
  part[warp][lane] = a;
  __syncthreads();
  if (warp != 0 || col >= K2) return;
  float4 r = part[0][lane];
#pragma unroll
  for (int w = 1; w < 8; ++w) {
    const float4 v = part[w][lane];
    r.x = rcomb<OP>(r.x, v.x);
    r.y = rcomb<OP>(r.y, v.y);
    r.z = rcomb<OP>(r.z, v.z);
    r.w = rcomb<OP>(r.w, v.w);
  }
  *reinterpret_cast<float4 *>(fold_out + static_cast<size_t>(k1) * K2 + col) = r;
}

// Sums `splits` partial planes part[s, i] into out[i].  A CTA of W warps
// owns 32 consecutive outputs; warp w folds splits w, w + W, w + 2W, ... in
// order and warp 0 then folds the W warp results in warp order, so the
// summation order is fixed (deterministic).  Many splits take W = 32, so
// each thread has only a few loads in its dependent chain.
template <int OP, int W>
__global__ void __launch_bounds__(W * 32)
combine_kernel(const float *__restrict__ part, float *out, uint64_t n,
               uint32_t splits) {
  pdl_enter();
  __shared__ float acc_w[W][33];
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t i = static_cast<uint64_t>(blockIdx.x) * 32 + lane;
  float acc = rinit<OP>();
  if (i < n) {
#pragma unroll 4
    for (uint32_t s = warp; s < splits; s += W) acc = rcomb<OP>(acc, part[s * n + i]);
  }
  acc_w[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && i < n) {
    float r = acc_w[0][lane];
#pragma unroll
    for (int w = 1; w < W; ++w) r = rcomb<OP>(r, acc_w[w][lane]);
    out[i] = r;
  }
}

struct GenericParams {
  int rank;                      // merged dims
  uint32_t shape[TL_MAX_RANK];
  uint32_t xstride[TL_MAX_RANK];
  uint32_t reduced[TL_MAX_RANK];  // 1 if reduced
  uint32_t out_count;
  uint32_t red_count;
};

// One thread per output element; walks the reduced index space.
template <int OP>
__global__ void generic_kernel(const float *__restrict__ x, float *out,
                               GenericParams p) {
  pdl_enter();
  for (uint32_t o = blockIdx.x * blockDim.x + threadIdx.x; o < p.out_count;
       o += gridDim.x * blockDim.x) {
    // decode o over kept dims (row-major over kept dims)
    uint32_t base = 0, rem = o;
    for (int d = p.rank - 1; d >= 0; --d) {
      if (p.reduced[d]) continue;
      const uint32_t c = rem % p.shape[d];
      rem /= p.shape[d];
      base += c * p.xstride[d];
    }
    float acc = rinit<OP>();
    for (uint32_t i = 0; i < p.red_count; ++i) {
      uint32_t off = 0, ri = i;
      for (int d = p.rank - 1; d >= 0; --d) {
        if (!p.reduced[d]) continue;
        const uint32_t c = ri % p.shape[d];
        ri /= p.shape[d];
        off += c * p.xstride[d];
      }
      acc = rcomb<OP>(acc, x[base + off]);
    }
    out[o] = acc;
  }
}

enum PlanKind { kCopy, kRows, kCols, kGeneric };

struct ReducePlan {
  PlanKind kind;
  uint64_t numel;     // input elements
  uint64_t out_count;
  // rows: rows x cols; cols: K1 x R x K2
  uint32_t rows, cols, K1, R, K2;
  uint32_t splits, chunk;
  bool block = false;  // kCols by cols_block_kernel
  size_t workspace;   // bytes
  GenericParams gp;
};

int make_plan(const uint32_t *x_shape, int x_rank, const uint32_t *out_shape,
              int out_rank, ReducePlan &pl) {
  if (x_rank < 0 || x_rank > TL_MAX_RANK || out_rank < 0 || out_rank > x_rank)
    return fail(TL_ERR_INVALID, "reduce: cannot reduce to a shape with a higher rank");
  uint32_t aligned[TL_MAX_RANK];
  const int off = x_rank - out_rank;
  for (int i = 0; i < x_rank; ++i) aligned[i] = i < off ? 1u : out_shape[i - off];
  pl = ReducePlan{};
  pl.numel = 1;
  pl.out_count = 1;
  for (int i = 0; i < x_rank; ++i) {
    if (x_shape[i] != aligned[i] && aligned[i] != 1)
      return fail(TL_ERR_INVALID, "invalid reduce_to_shape");
    pl.numel *= x_shape[i];
    pl.out_count *= aligned[i];
  }
  // merge neighbouring dims of the same class (size-1 dims dropped)
  uint32_t gs[TL_MAX_RANK], gr[TL_MAX_RANK];
  int g = 0;
  for (int i = 0; i < x_rank; ++i) {
    if (x_shape[i] == 1) continue;
    const uint32_t red = aligned[i] == 1 ? 1u : 0u;
    if (g > 0 && gr[g - 1] == red) {
      gs[g - 1] *= x_shape[i];
    } else {
      gs[g] = x_shape[i];
      gr[g] = red;
      ++g;
    }
  }
  const size_t target_threads = static_cast<size_t>(kNumSMs) * 1024;
  if (pl.numel == 0 || g == 0 || (g == 1 && !gr[0]) ||
      (g >= 1 && [&] { for (int i = 0; i < g; ++i) if (gr[i]) return false; return true; }())) {
    pl.kind = kCopy;
    return TL_OK;
  }
  if ((g == 1 && gr[0]) || (g == 2 && !gr[0] && gr[1])) {
    pl.kind = kRows;
    pl.rows = g == 1 ? 1u : gs[0];
    pl.cols = g == 1 ? gs[0] : gs[1];
    // enough warps from rows alone, else split each row
    const uint64_t warps_wanted = target_threads / 32;
    uint32_t splits = 1;
    if (pl.rows < warps_wanted) {
      uint64_t want = warps_wanted / pl.rows;
      uint64_t max_splits = (pl.cols + 1023) / 1024;  // >= 1024 columns per split
      splits = static_cast<uint32_t>(want < max_splits ? want : max_splits);
      if (splits < 1) splits = 1;
    }
    uint32_t chunk = (pl.cols + splits - 1) / splits;
    chunk = (chunk + 3) & ~3u;
    splits = (pl.cols + chunk - 1) / chunk;
    pl.splits = splits;
    pl.chunk = chunk;
    pl.workspace = splits > 1 ? static_cast<size_t>(pl.rows) * splits * sizeof(float) : 0;
    return TL_OK;
  }
  if ((g == 2 && gr[0] && !gr[1]) || (g == 3 && !gr[0] && gr[1] && !gr[2])) {
    pl.kind = kCols;
    pl.K1 = g == 2 ? 1u : gs[0];
    pl.R = g == 2 ? gs[0] : gs[1];
    pl.K2 = g == 2 ? gs[1] : gs[2];
    const uint64_t outs = static_cast<uint64_t>(pl.K1) * pl.K2;
    if (pl.K2 % 4 == 0 && pl.K1 <= 65535 && pl.K2 / 128 < 65535) {
      // blocks of 8 warps x 128 columns: about two CTAs per SM, >= 128 rows
      // (the last CTA of a column block folds the splits' partials)
      const uint64_t colblocks = (pl.K2 + 127) / 128;
      uint64_t want = (2ull * kNumSMs + pl.K1 * colblocks - 1) / (pl.K1 * colblocks);
      const uint64_t max_splits = (pl.R + 127) / 128;
      if (want > max_splits) want = max_splits;
      if (want < 1) want = 1;
      uint32_t chunk = static_cast<uint32_t>((pl.R + want - 1) / want);
      chunk = (chunk + 7) & ~7u;
      pl.splits = (pl.R + chunk - 1) / chunk;
      pl.chunk = chunk;
      pl.block = true;
      pl.workspace = pl.splits > 1 ? outs * pl.splits * sizeof(float) : 0;
      return TL_OK;
    }
    const uint64_t lanes = pl.K2 % 4 == 0 ? outs / 4 : outs;
    uint32_t splits = 1;
    if (lanes < target_threads) {
      uint64_t want = (target_threads + lanes - 1) / lanes;
      uint64_t max_splits = (pl.R + 31) / 32;  // >= 32 rows per split
      splits = static_cast<uint32_t>(want < max_splits ? want : max_splits);
      if (splits < 1) splits = 1;
    }
    uint32_t chunk = (pl.R + splits - 1) / splits;
    splits = (pl.R + chunk - 1) / chunk;
    pl.splits = splits;
    pl.chunk = chunk;
    pl.workspace = splits > 1 ? outs * splits * sizeof(float) : 0;
    return TL_OK;
  }
  pl.kind = kGeneric;
  GenericParams &p = pl.gp;
  p.rank = g;
  uint32_t st = 1;
  uint64_t red = 1;
  for (int i = g; i-- > 0;) {
    p.shape[i] = gs[i];
    p.xstride[i] = st;
    p.reduced[i] = gr[i];
    st *= gs[i];
    if (gr[i]) red *= gs[i];
  }
  p.out_count = static_cast<uint32_t>(pl.out_count);
  p.red_count = static_cast<uint32_t>(red);
  return TL_OK;
}

template <int OP>
int run_plan(const ReducePlan &pl, const float *x, float *out, void *ws,
             cudaStream_t s) {
  switch (pl.kind) {
    case kCopy:
      return check_cuda(cudaMemcpyAsync(out, x, pl.numel * sizeof(float),
                                        cudaMemcpyDeviceToDevice, s),
                        "reduce copy");
    case kRows: {
      const bool vec = pl.cols % 4 == 0 && aligned16(x);
      float *dst = pl.splits > 1 ? static_cast<float *>(ws) : out;
      const uint64_t warps = static_cast<uint64_t>(pl.rows) * pl.splits;
      launch_pdl(rows_kernel<OP>, grid_for(warps * 32, 256, 16), 256, 0, s, 
          x, dst, pl.rows, pl.cols, pl.splits, pl.chunk, vec);
      int rc = launch_status("reduce rows");
      if (rc || pl.splits == 1) return rc;
      // dst is [rows, splits]: a second row pass over the partials
      launch_pdl(rows_kernel<OP>, grid_for(static_cast<uint64_t>(pl.rows) * 32, 256, 16), 256, 0, s, 
          dst, out, pl.rows, pl.splits, 1, pl.splits, false);
      return launch_status("reduce rows combine");
    }
    case kCols: {
      const bool vec = pl.K2 % 4 == 0 && aligned16(x) && aligned16(out) && aligned16(ws);
      float *dst = pl.splits > 1 ? static_cast<float *>(ws) : out;
      const uint64_t outs = static_cast<uint64_t>(pl.K1) * pl.K2;
      const uint64_t work = (vec ? outs / 4 : outs) * pl.splits;
      const uint64_t slots = static_cast<uint64_t>(pl.K1) * ((pl.K2 + 127) / 128);
      ColsGroups cg{};
      cg.x[0] = x;
      cg.part[0] = dst;
      if (pl.block && vec && pl.splits > 1 && slots <= kColTickets) {
        // one launch: the last CTA of each column block folds the splits
        cg.fold_out[0] = out;
        launch_pdl(cols_block_kernel<OP>, dim3(pl.splits, pl.K1, (pl.K2 + 127) / 128), 256, 0, s,
                   cg, pl.K1, pl.R, pl.K2, pl.chunk);
        return launch_status("reduce cols");
      }
      if (pl.block && vec)
        launch_pdl(cols_block_kernel<OP>, dim3(pl.splits, pl.K1, (pl.K2 + 127) / 128), 256, 0, s,
                   cg, pl.K1, pl.R, pl.K2, pl.chunk);
      else if (vec)
        launch_pdl(cols_kernel<OP, 4>, grid_for(work, 256, 16), 256, 0, s, x, dst, pl.K1, pl.R, pl.K2, pl.splits, pl.chunk);
      else
        launch_pdl(cols_kernel<OP, 1>, grid_for(work, 256, 16), 256, 0, s, x, dst, pl.K1, pl.R, pl.K2, pl.splits, pl.chunk);
      int rc = launch_status("reduce cols");
      if (rc || pl.splits == 1) return rc;
      if (pl.splits >= 64)
        launch_pdl(combine_kernel<OP, 32>, static_cast<unsigned>((outs + 31) / 32), 1024, 0, s,
                   dst, out, outs, pl.splits);
      else
        launch_pdl(combine_kernel<OP, 8>, static_cast<unsigned>((outs + 31) / 32), 256, 0, s,
                   dst, out, outs, pl.splits);
      return launch_status("reduce cols combine");
    }
    default:
      launch_pdl(generic_kernel<OP>, grid_for(pl.out_count, 128), 128, 0, s, x, out, pl.gp);
      return launch_status("reduce generic");
  }
}

// ---------------------------------------------------------------- argmax
struct ArgBest {
  float v;
  uint32_t i;
};

__device__ __forceinline__ void arg_merge(float &v, uint32_t &i, float v2, uint32_t i2) {
  // candidates must be > -inf (NaN never is); ties keep the lower index
  if (v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

__device__ __forceinline__ void arg_warp(float &v, uint32_t &i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    const uint32_t i2 = __shfl_xor_sync(0xffffffffu, i, o);
    arg_merge(v, i, v2, i2);
  }
}

__global__ void __launch_bounds__(256)
argmax_partial_kernel(const float *__restrict__ x, uint64_t n, ArgBest *part,
                      uint32_t *out_index, bool final_pass) {
  pdl_enter();
  float v = -INFINITY;
  uint32_t idx = 0xffffffffu;
  for (uint64_t j = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; j < n;
       j += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const float xv = x[j];
    if (xv > -INFINITY) arg_merge(v, idx, xv, static_cast<uint32_t>(j));
  }
  arg_warp(v, idx);
  __shared__ float sv[8];
  __shared__ uint32_t si[8];
  const int w = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[w] = v;
    si[w] = idx;
  }
  __syncthreads();
  if (w == 0) {
    v = lane < blockDim.x / 32 ? sv[lane] : -INFINITY;
    idx = lane < blockDim.x / 32 ? si[lane] : 0xffffffffu;
    arg_warp(v, idx);
    if (lane == 0) {
      if (final_pass) *out_index = idx == 0xffffffffu ? 0u : idx;
      else part[blockIdx.x] = ArgBest{v, idx};
    }
  }
}

__global__ void __launch_bounds__(256)
argmax_final_kernel(const ArgBest *part, uint32_t count, uint32_t *out_index) {
  pdl_enter();
  float v = -INFINITY;
  uint32_t idx = 0xffffffffu;
  for (uint32_t j = threadIdx.x; j < count; j += blockDim.x)
    if (part[j].i != 0xffffffffu) arg_merge(v, idx, part[j].v, part[j].i);
  arg_warp(v, idx);
  __shared__ float sv[8];
  __shared__ uint32_t si[8];
  const int w = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[w] = v;
    si[w] = idx;
  }
  __syncthreads();
  if (w == 0) {
    v = lane < blockDim.x / 32 ? sv[lane] : -INFINITY;
    idx = lane < blockDim.x / 32 ? si[lane] : 0xffffffffu;
    arg_warp(v, idx);
    if (lane == 0) *out_index = idx == 0xffffffffu ? 0u : idx;
  }
}

uint32_t argmax_blocks(size_t count) {
  return grid_for(count, 256, 4);
}

}  // namespace
}  // namespace tl

using namespace tl;

extern "C" {

size_t tl_reduce_workspace_size(const uint32_t *x_shape, int x_rank,
                                const uint32_t *out_shape, int out_rank) {
  ReducePlan pl;
  if (make_plan(x_shape, x_rank, out_shape, out_rank, pl)) return 0;
  return pl.workspace;
}

int tl_reduce(int op, const float *x, const uint32_t *x_shape, int x_rank,
              float *out, const uint32_t *out_shape, int out_rank,
              void *workspace, size_t workspace_bytes, void *stream) {
  if (op != TL_REDUCE_SUM && op != TL_REDUCE_MAX)
    return fail(TL_ERR_INVALID, "tl_reduce: unknown op");
  ReducePlan pl;
  int rc = make_plan(x_shape, x_rank, out_shape, out_rank, pl);
  if (rc) return rc;
  if (pl.numel == 0 || pl.out_count == 0) return TL_OK;
  if (!x || !out) return fail(TL_ERR_INVALID, "tl_reduce: null pointer");
  if (pl.workspace > workspace_bytes || (pl.workspace && !workspace))
    return fail(TL_ERR_INVALID, "tl_reduce: workspace too small");
  if (pl.numel > 0xffffffffull) return fail(TL_ERR_RANGE, "tl_reduce: more than 2^32-1 elements");
  cudaStream_t s = as_stream(stream);
  return op == TL_REDUCE_SUM ? run_plan<TL_REDUCE_SUM>(pl, x, out, workspace, s)
                             : run_plan<TL_REDUCE_MAX>(pl, x, out, workspace, s);
}

size_t tl_reduce_group_workspace_size(uint32_t groups, const uint32_t *x_shape, int x_rank,
                                      const uint32_t *out_shape, int out_rank) {
  return groups * tl_reduce_workspace_size(x_shape, x_rank, out_shape, out_rank);
}

int tl_reduce_group(int op, uint32_t groups, const float *const *x, const uint32_t *x_shape,
                    int x_rank, float *const *out, const uint32_t *out_shape, int out_rank,
                    void *workspace, size_t workspace_bytes, void *stream) {
  if (op != TL_REDUCE_SUM && op != TL_REDUCE_MAX)
    return fail(TL_ERR_INVALID, "tl_reduce_group: unknown op");
  if (groups < 1 || groups > TL_REDUCE_MAX_GROUPS)
    return fail(TL_ERR_INVALID, "tl_reduce_group: 1 to TL_REDUCE_MAX_GROUPS groups");
  if (!x || !out) return fail(TL_ERR_INVALID, "tl_reduce_group: null pointer");
  ReducePlan pl;
  int rc = make_plan(x_shape, x_rank, out_shape, out_rank, pl);
  if (rc) return rc;
  if (pl.numel == 0 || pl.out_count == 0) return TL_OK;
  for (uint32_t i = 0; i < groups; ++i)
    if (!x[i] || !out[i]) return fail(TL_ERR_INVALID, "tl_reduce_group: null pointer");
  if (groups * pl.workspace > workspace_bytes || (pl.workspace && !workspace))
    return fail(TL_ERR_INVALID, "tl_reduce_group: workspace too small");
  if (pl.numel > 0xffffffffull)
    return fail(TL_ERR_RANGE, "tl_reduce_group: more than 2^32-1 elements");
  cudaStream_t s = as_stream(stream);
  float *ws = static_cast<float *>(workspace);
  const size_t ws_floats = pl.workspace / sizeof(float);
  // one launch when every group folds its split partials in-launch: the
  // same plan, grid and fold order as tl_reduce of each group alone
  const uint64_t colblocks = (pl.K2 + 127) / 128;
  bool one = pl.kind == kCols && pl.block && pl.K1 == 1 && pl.splits > 1 && pl.K2 % 4 == 0 &&
             groups * colblocks <= kColTickets && aligned16(ws);
  for (uint32_t i = 0; i < groups && one; ++i) one = aligned16(x[i]) && aligned16(out[i]);
  if (one) {
    ColsGroups cg{};
    cg.grouped = 1;
    for (uint32_t i = 0; i < groups; ++i) {
      cg.x[i] = x[i];
      cg.part[i] = ws + i * ws_floats;
      cg.fold_out[i] = out[i];
    }
    const dim3 grid(pl.splits, groups, static_cast<unsigned>(colblocks));
    if (op == TL_REDUCE_SUM)
      launch_pdl(cols_block_kernel<TL_REDUCE_SUM>, grid, 256, 0, s, cg, 1u, pl.R, pl.K2, pl.chunk);
    else
      launch_pdl(cols_block_kernel<TL_REDUCE_MAX>, grid, 256, 0, s, cg, 1u, pl.R, pl.K2, pl.chunk);
    return launch_status("reduce cols grouped");
  }
  for (uint32_t i = 0; i < groups; ++i) {
    float *wi = pl.workspace ? ws + i * ws_floats : nullptr;
    rc = op == TL_REDUCE_SUM ? run_plan<TL_REDUCE_SUM>(pl, x[i], out[i], wi, s)
                             : run_plan<TL_REDUCE_MAX>(pl, x[i], out[i], wi, s);
    if (rc) return rc;
  }
  return TL_OK;
}

size_t tl_argmax_workspace_size(size_t count) {
  const uint32_t b = argmax_blocks(count);
  return b > 1 ? b * sizeof(ArgBest) : 0;
}

int tl_argmax(const float *x, size_t count, uint32_t *out_index, void *workspace,
              size_t workspace_bytes, void *stream) {
  if (count == 0) return fail(TL_ERR_INVALID, "argmax requires a non-empty tensor");
  if (!x || !out_index) return fail(TL_ERR_INVALID, "tl_argmax: null pointer");
  if (count > 0xffffffffull) return fail(TL_ERR_RANGE, "tl_argmax: more than 2^32-1 elements");
  const uint32_t blocks = argmax_blocks(count);
  cudaStream_t s = as_stream(stream);
  if (blocks == 1) {
    launch_pdl(argmax_partial_kernel, 1, 256, 0, s, x, count, nullptr, out_index, true);
    return launch_status("tl_argmax");
  }
  if (!workspace || workspace_bytes < blocks * sizeof(ArgBest))
    return fail(TL_ERR_INVALID, "tl_argmax: workspace too small");
  ArgBest *part = static_cast<ArgBest *>(workspace);
  launch_pdl(argmax_partial_kernel, blocks, 256, 0, s, x, count, part, nullptr, false);
  int rc = launch_status("tl_argmax partial");
  if (rc) return rc;
  launch_pdl(argmax_final_kernel, 1, 256, 0, s, part, blocks, out_index);
  return launch_status("tl_argmax final");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of tl_reduce (no counterpart in the reference).
//
// Some callers cannot allocate device memory at the moment they need a
// reduction: code running while a CUDA stream is being captured into a graph
// (where cudaMalloc is not allowed), hosts whose whole device-memory budget
// is owned by another allocator (a framework's caching pool or a fixed
// arena, where an extra cudaMalloc would exceed the budget or fragment it),
// and foreign-language callers that bind this C ABI without binding the
// CUDA allocator.  tl_reduce_noalloc takes no workspace: the split partial
// sums live in the file-scope device array below, which every GPU that
// loads this library holds until the process exits.
namespace tl {
namespace {

// 4 MiB of partials.  The planner's largest workspace is about 3.1 MB
// (3 x 2^18 floats: a column plan over more than 65535 column groups, whose
// lanes are split at most three ways); the GPT step's largest, a
// [12288, 1536] -> [1536] bias gradient, uses about 0.3 MB.
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;
static __device__ __align__(256) unsigned char g_reduce_scratch[kNoAllocScratchBytes];

// Device address of g_reduce_scratch on the current device.  In host code
// the array's name is only a host-side stand-in, so the address is looked
// up once per device (with that device current) and cached.  The cache is
// safe for concurrent first calls from several host threads; after
// cudaDeviceReset the cached address is stale, so the process must not
// call this entry point again on a device it has reset.
int noalloc_scratch(void **ptr) {
  static std::atomic<void *> cached[64];
  static std::mutex lookup;
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "tl_reduce_noalloc: cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= 64) return fail(TL_ERR_RANGE, "tl_reduce_noalloc: device id above 63");
  void *p = cached[dev].load(std::memory_order_acquire);
  if (!p) {
    std::lock_guard<std::mutex> hold(lookup);
    p = cached[dev].load(std::memory_order_relaxed);
    if (!p) {
      rc = check_cuda(cudaGetSymbolAddress(&p, g_reduce_scratch),
                      "tl_reduce_noalloc: cudaGetSymbolAddress of the scratch array");
      if (rc) return rc;
      cached[dev].store(p, std::memory_order_release);
    }
  }
  *ptr = p;
  return TL_OK;
}

}  // namespace
}  // namespace tl

extern "C" size_t tl_reduce_noalloc_max_workspace(void) { return tl::kNoAllocScratchBytes; }

extern "C" int tl_reduce_noalloc(int op, const float *x, const uint32_t *x_shape, int x_rank,
                                 float *out, const uint32_t *out_shape, int out_rank,
                                 void *stream) {
  if (op != TL_REDUCE_SUM && op != TL_REDUCE_MAX)
    return fail(TL_ERR_INVALID, "tl_reduce_noalloc: unknown op");
  ReducePlan pl;
  int rc = make_plan(x_shape, x_rank, out_shape, out_rank, pl);
  if (rc) return rc;
  if (pl.numel == 0 || pl.out_count == 0) return TL_OK;
  if (!x || !out) return fail(TL_ERR_INVALID, "tl_reduce_noalloc: null pointer");
  if (pl.numel > 0xffffffffull)
    return fail(TL_ERR_RANGE, "tl_reduce_noalloc: more than 2^32-1 elements");
  if (pl.workspace > kNoAllocScratchBytes)
    return fail(TL_ERR_RANGE, "tl_reduce_noalloc: this reduction needs " +
                                  std::to_string(pl.workspace) +
                                  " bytes of partials, above the built-in 4 MiB scratch; use "
                                  "tl_reduce with a caller workspace");
  void *scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  // Partial planes are written in full by the first pass before the second
  // pass reads them, so the previous call's contents need no clearing.
  cudaStream_t s = as_stream(stream);
  return op == TL_REDUCE_SUM ? run_plan<TL_REDUCE_SUM>(pl, x, out, scratch, s)
                             : run_plan<TL_REDUCE_MAX>(pl, x, out, scratch, s);
}

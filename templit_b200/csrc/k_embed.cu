// Embedding gather and deterministic scatter-add
// (Runtime::embedding_lookup / scatter_add_rows / scatter_index,
// src/my_metal/runtime.cpp:920-1030; math.metal:778-820).
//
// The reference scatters with one float atomic per element, so its result
// depends on arrival order.  Here the scatter runs in two deterministic
// phases: every chunk of 64 ids is sorted in shared memory and summed per
// distinct id (position order), then every destination row folds its chunk
// partials in a fixed order.  Every run is bit-identical, and a hot id (a
// frequent token) is spread over all chunks instead of one serial loop.  Ids outside the table never touch memory:
// they raise TL_FLAG_INDEX_RANGE in the device status word instead.
#include "tl_common.cuh"

#include <type_traits>

namespace tl {
namespace {

template <int V>
__global__ void __launch_bounds__(256)
gather_kernel(const float *__restrict__ w, uint32_t n_rows, uint32_t dim,
              const uint32_t *__restrict__ ids, uint32_t n_ids, float *out,
              uint32_t *status) {
  pdl_enter();
  const uint32_t per_row = dim / V;
  const uint64_t total = static_cast<uint64_t>(n_ids) * per_row;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       t < total; t += stride) {
    const uint32_t i = static_cast<uint32_t>(t / per_row);
    const uint32_t c = static_cast<uint32_t>(t % per_row) * V;
    const uint32_t id = ids[i];
    float *dst = out + static_cast<size_t>(i) * dim + c;
    if (id >= n_rows) {
      if (c == 0) raise_flag(status, TL_FLAG_INDEX_RANGE);
      if constexpr (V == 4) *reinterpret_cast<float4 *>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
      else *dst = 0.0f;
      continue;
    }
    const float *src = w + static_cast<size_t>(id) * dim + c;
    if constexpr (V == 4) *reinterpret_cast<float4 *>(dst) = *reinterpret_cast<const float4 *>(src);
    else *dst = *src;
  }
}

constexpr uint32_t kChunk = 64;      // ids per chunk (phase 1 CTA)
constexpr uint32_t kThreads = 256;   // threads per CTA, both phases
constexpr uint32_t kInvalid = 0xffffffffu;

// Phase 1: CTA p takes ids [p * kChunk, (p + 1) * kChunk), sorts the
// (id, position) pairs of its chunk (bitonic, in shared memory), and for each
// distinct id u of the chunk (ascending) writes
//   partial[p * kChunk + u, :] = sum of values[i, :] over the chunk's i with
//                                ids[i] == id, in position order,
//   uid[p * kChunk + u] = id, and ucount[p] = number of distinct ids.
// The sums spread (distinct id, column group) items over all threads, four
// items at a time so their first loads are in flight together.
template <int V>
__global__ void __launch_bounds__(kThreads)
chunk_sum_kernel(const float *__restrict__ values, const uint32_t *__restrict__ ids,
                 uint32_t n_ids, uint32_t dim, uint32_t n_rows, float *partial,
                 uint32_t *uid, uint32_t *ucount, uint32_t *status) {
  pdl_enter();
  __shared__ unsigned long long key[kChunk];
  __shared__ uint32_t gstart[kChunk + 1];
  __shared__ uint32_t warp_heads[kChunk / 32], warp_valid[kChunk / 32];
  __shared__ uint32_t n_groups;
  const uint32_t t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const uint64_t first = static_cast<uint64_t>(blockIdx.x) * kChunk;
  if (t < kChunk) {
    uint32_t id = kInvalid;
    if (first + t < n_ids) {
      id = ids[first + t];
      if (id >= n_rows) {
        raise_flag(status, TL_FLAG_INDEX_RANGE);
        id = kInvalid;
      }
    }
    key[t] = (static_cast<unsigned long long>(id) << 32) | t;
  }
  __syncthreads();
  for (uint32_t k = 2; k <= kChunk; k <<= 1) {
    for (uint32_t j = k >> 1; j > 0; j >>= 1) {
      const uint32_t o = t ^ j;
      if (t < kChunk && o > t) {
        const unsigned long long a = key[t], b = key[o];
        if ((a > b) == ((t & k) == 0)) {
          key[t] = b;
          key[o] = a;
        }
      }
      __syncthreads();
    }
  }
  // group heads and their ranks (warps covering the chunk)
  if (t < kChunk) {
    const uint32_t my = static_cast<uint32_t>(key[t] >> 32);
    const bool valid = my != kInvalid;
    const bool head = valid && (t == 0 || static_cast<uint32_t>(key[t - 1] >> 32) != my);
    const uint32_t hb = __ballot_sync(0xffffffffu, head), vb = __ballot_sync(0xffffffffu, valid);
    if (lane == 0) {
      warp_heads[warp] = __popc(hb);
      warp_valid[warp] = __popc(vb);
    }
  }
  __syncthreads();
  if (t < kChunk) {
    const uint32_t my = static_cast<uint32_t>(key[t] >> 32);
    const bool valid = my != kInvalid;
    const bool head = valid && (t == 0 || static_cast<uint32_t>(key[t - 1] >> 32) != my);
    const uint32_t hb = __ballot_sync(0xffffffffu, head);
    uint32_t before = 0, groups = 0, n_valid = 0;
    for (uint32_t w = 0; w < kChunk / 32; ++w) {
      if (w < warp) before += warp_heads[w];
      groups += warp_heads[w];
      n_valid += warp_valid[w];
    }
    const uint32_t g = before + __popc(hb & ((1u << lane) - 1u));
    if (head) {
      gstart[g] = t;
      uid[first + g] = my;
    }
    if (t == 0) {
      gstart[groups] = n_valid;
      ucount[blockIdx.x] = groups;
      n_groups = groups;
    }
  }
  __syncthreads();
  const uint32_t cols = dim / V, total = n_groups * cols;
  for (uint32_t base = t; base < total; base += 4 * kThreads) {
    float acc[4][V];
    uint32_t q[4], col[4], b[4], e[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t item = base + u * kThreads;
      q[u] = item / cols;
      col[u] = (item % cols) * V;
      b[u] = e[u] = 0;
#pragma unroll
      for (int v = 0; v < V; ++v) acc[u][v] = 0.0f;
      if (item < total) {
        b[u] = gstart[q[u]];
        e[u] = gstart[q[u] + 1];
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      for (uint32_t k = b[u]; k < e[u]; ++k) {
        const uint32_t pos = static_cast<uint32_t>(key[k] & 0xffffffffu);
        const float *src = values + (first + pos) * dim + col[u];
        if constexpr (V == 4) {
          const float4 x = *reinterpret_cast<const float4 *>(src);
          acc[u][0] += x.x;
          acc[u][1] += x.y;
          acc[u][2] += x.z;
          acc[u][3] += x.w;
        } else {
          acc[u][0] += *src;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (b[u] == e[u]) continue;
      float *dst = partial + (first + q[u]) * dim + col[u];
      if constexpr (V == 4)
        *reinterpret_cast<float4 *>(dst) = make_float4(acc[u][0], acc[u][1], acc[u][2], acc[u][3]);
      else
        *dst = acc[u][0];
    }
  }
}

// Phase 2: CTA (r, slice) writes dst[r, slice] = base[r, slice] + the chunk
// partials of row r.  Thread t binary-searches chunk t of each round of 256
// chunks; warp w folds the chunks c with c % 8 == w in increasing order, and
// warp 0 folds the 8 warp sums in warp order: a fixed summation order.
template <int V>
__global__ void __launch_bounds__(kThreads)
row_combine_kernel(const float *__restrict__ partial, const uint32_t *__restrict__ uid,
                   const uint32_t *__restrict__ ucount, uint32_t n_chunks, uint32_t dim,
                   const float *base, float *dst) {
  pdl_enter();
  using Vec = typename std::conditional<V == 4, float4, float>::type;
  __shared__ int slot[kThreads];
  __shared__ Vec wsum[kThreads / 32][32];
  const uint32_t t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const uint32_t r = blockIdx.x;
  const uint32_t d = blockIdx.y * 32 * V + lane * V;
  const bool in = d < dim;
  float acc[V];
#pragma unroll
  for (int v = 0; v < V; ++v) acc[v] = 0.0f;
  for (uint32_t round = 0; round < n_chunks; round += kThreads) {
    const uint32_t c = round + t;
    int found = -1;
    if (c < n_chunks) {
      const uint32_t *u = uid + static_cast<uint64_t>(c) * kChunk;
      uint32_t lo = 0, hi = ucount[c];
      while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        if (u[mid] < r) lo = mid + 1;
        else hi = mid;
      }
      if (lo < ucount[c] && u[lo] == r) found = static_cast<int>(lo);
    }
    slot[t] = found;
    __syncthreads();
    const uint32_t in_round = min(kThreads, n_chunks - round);
    for (uint32_t q = warp; q < in_round; q += kThreads / 32) {
      const int u = slot[q];
      if (u < 0 || !in) continue;
      const float *src = partial + ((static_cast<uint64_t>(round + q)) * kChunk + u) * dim + d;
      if constexpr (V == 4) {
        const float4 v = *reinterpret_cast<const float4 *>(src);
        acc[0] += v.x;
        acc[1] += v.y;
        acc[2] += v.z;
        acc[3] += v.w;
      } else {
        acc[0] += *src;
      }
    }
    __syncthreads();
  }
  if constexpr (V == 4) wsum[warp][lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  else wsum[warp][lane] = acc[0];
  __syncthreads();
  if (warp != 0 || !in) return;
  float s[V];
#pragma unroll
  for (int v = 0; v < V; ++v) s[v] = 0.0f;
  for (uint32_t w = 0; w < kThreads / 32; ++w) {
    const float *x = reinterpret_cast<const float *>(&wsum[w][lane]);
#pragma unroll
    for (int v = 0; v < V; ++v) s[v] += x[v];
  }
  const size_t o = static_cast<size_t>(r) * dim + d;
  if constexpr (V == 4) {
    float4 out = make_float4(s[0], s[1], s[2], s[3]);
    if (base) {
      const float4 b = *reinterpret_cast<const float4 *>(base + o);
      out = make_float4(b.x + s[0], b.y + s[1], b.z + s[2], b.w + s[3]);
    }
    *reinterpret_cast<float4 *>(dst + o) = out;
  } else {
    dst[o] = base ? base[o] + s[0] : s[0];
  }
}

}  // namespace
}  // namespace tl

using namespace tl;

extern "C" {

int tl_embedding_gather(const float *weights, uint32_t n_rows, uint32_t dim,
                        const uint32_t *ids, uint32_t n_ids, float *out,
                        void *stream) {
  if (n_ids == 0 || dim == 0) return TL_OK;
  if (!weights || !ids || !out) return fail(TL_ERR_INVALID, "tl_embedding_gather: null pointer");
  uint32_t *status = device_status_ptr();
  if (!status) return fail(TL_ERR_CUDA, "tl_embedding_gather: no status word");
  cudaStream_t s = as_stream(stream);
  const uint64_t total = static_cast<uint64_t>(n_ids) * dim;
  if (dim % 4 == 0 && aligned16(weights) && aligned16(out))
    launch_pdl(gather_kernel<4>, grid_for(total / 4, 256), 256, 0, s, weights, n_rows, dim, ids, n_ids, out, status);
  else
    launch_pdl(gather_kernel<1>, grid_for(total, 256), 256, 0, s, weights, n_rows, dim, ids, n_ids, out, status);
  return launch_status("tl_embedding_gather");
}

namespace {
uint32_t scatter_chunks(uint32_t n_ids) { return (n_ids + kChunk - 1) / kChunk; }
}  // namespace

size_t tl_embedding_scatter_workspace_size(uint32_t n_ids, uint32_t n_rows, uint32_t dim) {
  (void)n_rows;
  const size_t slots = static_cast<size_t>(scatter_chunks(n_ids)) * kChunk;
  // partial rows, then uid per slot, then one count per chunk
  return slots * dim * sizeof(float) + slots * sizeof(uint32_t) +
         scatter_chunks(n_ids) * sizeof(uint32_t);
}

int tl_embedding_scatter_add(const float *values, const uint32_t *ids,
                             uint32_t n_ids, uint32_t dim, const float *base,
                             float *dst, uint32_t n_rows, void *workspace,
                             size_t workspace_bytes, void *stream) {
  if (n_rows == 0 || dim == 0) return TL_OK;
  if (!dst || (n_ids && (!values || !ids)))
    return fail(TL_ERR_INVALID, "tl_embedding_scatter_add: null pointer");
  if (n_ids && (!workspace ||
                workspace_bytes < tl_embedding_scatter_workspace_size(n_ids, n_rows, dim)))
    return fail(TL_ERR_INVALID, "tl_embedding_scatter_add: workspace too small");
  uint32_t *status = device_status_ptr();
  if (!status) return fail(TL_ERR_CUDA, "tl_embedding_scatter_add: no status word");
  cudaStream_t s = as_stream(stream);
  const uint32_t chunks = scatter_chunks(n_ids);
  const size_t slots = static_cast<size_t>(chunks) * kChunk;
  float *partial = static_cast<float *>(workspace);
  uint32_t *uid = reinterpret_cast<uint32_t *>(partial + slots * dim);
  uint32_t *ucount = uid + slots;
  const bool vec = dim % 4 == 0 && aligned16(values) && aligned16(dst) &&
                   (!base || aligned16(base)) && aligned16(workspace);
  if (chunks) {
    if (vec)
      launch_pdl(chunk_sum_kernel<4>, chunks, kThreads, 0, s, values, ids, n_ids, dim, n_rows, partial, uid, ucount, status);
    else
      launch_pdl(chunk_sum_kernel<1>, chunks, kThreads, 0, s, values, ids, n_ids, dim, n_rows, partial, uid, ucount, status);
    const int rc = launch_status("tl_embedding_scatter_add chunks");
    if (rc) return rc;
  }
  const uint32_t per = 32 * (vec ? 4 : 1);
  const dim3 grid(n_rows, (dim + per - 1) / per);
  if (vec)
    launch_pdl(row_combine_kernel<4>, grid, kThreads, 0, s, partial, uid, ucount, chunks, dim, base, dst);
  else
    launch_pdl(row_combine_kernel<1>, grid, kThreads, 0, s, partial, uid, ucount, chunks, dim, base, dst);
  return launch_status("tl_embedding_scatter_add rows");
}

}  // extern "C"

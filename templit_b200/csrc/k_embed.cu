// Embedding gather and deterministic scatter-add
// (Runtime::embedding_lookup / scatter_add_rows / scatter_index,
// src/my_metal/runtime.cpp:920-1030; math.metal:778-820).
//
// The reference scatters with one float atomic per element, so its result
// depends on arrival order.  Here the scatter runs in two deterministic
// phases: every chunk of 64 ids is sorted in shared memory and summed per
// distinct id (position order), then every destination row folds its chunk
// partials in a fixed order.  Every run is bit-identical, and a hot id (a
// frequent token) is spread over all chunks instead of one serial loop.
// Both phases keep 16 row loads per thread in flight (the sums are
// latency-bound otherwise), and a slot table (row, chunk) -> slot lets a
// destination row find its partials with one load per chunk.  Ids outside
// the table never touch memory: they raise TL_FLAG_INDEX_RANGE in the device
// status word instead.
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
constexpr uint32_t kThreads1 = 128;  // phase 1: one thread per column group
constexpr uint32_t kThreads2 = 256;  // phase 2
constexpr uint32_t kBatch = 16;      // loads in flight per thread
constexpr uint32_t kInvalid = 0xffffffffu;
// the slot table (n_rows x chunks words) is used up to this size; larger
// problems find a row's chunk slots by binary search instead
constexpr size_t kMaxSlotTable = size_t(64) << 20;

template <int V> struct VecOf { using T = float; };
template <> struct VecOf<4> { using T = float4; };

template <int V> __device__ __forceinline__ void vadd(float (&acc)[V], const typename VecOf<V>::T &x) {
  if constexpr (V == 4) {
    acc[0] += x.x;
    acc[1] += x.y;
    acc[2] += x.z;
    acc[3] += x.w;
  } else {
    acc[0] += x;
  }
}

template <int V> __device__ __forceinline__ void vstore(float *dst, const float (&acc)[V]) {
  if constexpr (V == 4) *reinterpret_cast<float4 *>(dst) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  else *dst = acc[0];
}

// Phase 1: CTA p takes ids [p * kChunk, (p + 1) * kChunk).  Thread i < 64
// ranks its (id, position) key among the chunk's keys (a stable sort by id),
// the distinct ids get slots u = 0, 1, ... in ascending id order, and
//   partial[p * kChunk + u, :] = sum of values[i, :] over the chunk's i with
//                                ids[i] == id, in position order,
//   uid[p * kChunk + u] = id, ucount[p] = number of distinct ids, and
//   (with a slot table) slots[id * chunks + p] = u.
// The sum is a segmented pass over the chunk's rows in sorted order: each
// thread owns V columns and keeps kBatch row loads in flight.
template <int V>
__global__ void __launch_bounds__(kThreads1)
chunk_sum_kernel(const float *__restrict__ values, const uint32_t *__restrict__ ids,
                 uint32_t n_ids, uint32_t dim, uint32_t n_rows, float *partial,
                 uint32_t *uid, uint32_t *ucount, uint32_t *slots, uint32_t chunks,
                 uint32_t *status) {
  pdl_enter();
  using Vec = typename VecOf<V>::T;
  __shared__ uint32_t key_id[kChunk], s_id[kChunk], s_pos[kChunk], s_slot[kChunk];
  __shared__ uint32_t warp_heads[kChunk / 32], warp_valid[kChunk / 32];
  const uint32_t t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const uint32_t c = blockIdx.x;
  const uint64_t first = static_cast<uint64_t>(c) * kChunk;
  const uint64_t left = n_ids - first;
  const uint32_t in_chunk = left < kChunk ? static_cast<uint32_t>(left) : kChunk;
  if (t < kChunk) {
    uint32_t id = kInvalid;
    if (t < in_chunk) {
      id = ids[first + t];
      if (id >= n_rows) {
        raise_flag(status, TL_FLAG_INDEX_RANGE);
        id = kInvalid;
      }
    }
    key_id[t] = id;
  }
  __syncthreads();
  if (t < kChunk) {
    // rank of (id, t) among the chunk's keys: invalid ids sort last
    const uint32_t my = key_id[t];
    uint32_t rank = 0;
#pragma unroll 8
    for (uint32_t j = 0; j < kChunk; ++j) {
      const uint32_t o = key_id[j];
      rank += (o < my) || (o == my && j < t);
    }
    s_id[rank] = my;
    s_pos[rank] = t;
  }
  __syncthreads();
  if (t < kChunk) {
    const uint32_t my = s_id[t];
    const bool valid = my != kInvalid;
    const bool head = valid && (t == 0 || s_id[t - 1] != my);
    const uint32_t hb = __ballot_sync(0xffffffffu, head);
    const uint32_t vb = __ballot_sync(0xffffffffu, valid);
    if (lane == 0) {
      warp_heads[warp] = __popc(hb);
      warp_valid[warp] = __popc(vb);
    }
  }
  __syncthreads();
  if (t < kChunk) {
    const uint32_t my = s_id[t];
    const bool valid = my != kInvalid;
    const bool head = valid && (t == 0 || s_id[t - 1] != my);
    const uint32_t hb = __ballot_sync(0xffffffffu, head);
    // slot of t's id: the heads at or before t, minus one ((2 << 31) - 1
    // wraps to all lanes)
    const uint32_t u = (warp ? warp_heads[0] : 0u) + __popc(hb & ((2u << lane) - 1u)) - 1u;
    if (valid) s_slot[t] = u;
    if (head) {
      uid[first + u] = my;
      if (slots) slots[static_cast<size_t>(my) * chunks + c] = u;
    }
    if (t == 0) ucount[c] = warp_heads[0] + warp_heads[1];
  }
  __syncthreads();
  // valid keys (ids inside the table) are a prefix of the sorted order
  const uint32_t n_valid = warp_valid[0] + warp_valid[1];
  const uint32_t cols = dim / V;
  for (uint32_t col = t; col < cols; col += kThreads1) {
    float acc[V];
#pragma unroll
    for (int v = 0; v < V; ++v) acc[v] = 0.0f;
    for (uint32_t k0 = 0; k0 < n_valid; k0 += kBatch) {
      Vec x[kBatch];
#pragma unroll
      for (uint32_t j = 0; j < kBatch; ++j) {
        const uint32_t k = k0 + j;
        if (k < n_valid)
          x[j] = *reinterpret_cast<const Vec *>(values + (first + s_pos[k]) * dim +
                                                 static_cast<size_t>(col) * V);
      }
#pragma unroll
      for (uint32_t j = 0; j < kBatch; ++j) {
        const uint32_t k = k0 + j;
        if (k < n_valid) {
          vadd<V>(acc, x[j]);
          if (k + 1 == n_valid || s_id[k + 1] != s_id[k]) {  // end of the id's run
            vstore<V>(partial + (first + s_slot[k]) * dim + static_cast<size_t>(col) * V, acc);
#pragma unroll
            for (int v = 0; v < V; ++v) acc[v] = 0.0f;
          }
        }
      }
    }
  }
}

// Slot of row r in chunk c, or -1: from the slot table (an entry is trusted
// only when the chunk's distinct-id list holds r there, so the table needs
// no clearing), or by binary search of that list.
__device__ __forceinline__ int find_slot(uint32_t r, uint32_t c, const uint32_t *uid,
                                         const uint32_t *ucount, const uint32_t *slots,
                                         uint32_t chunks) {
  const uint32_t n = ucount[c];
  const uint32_t *u = uid + static_cast<uint64_t>(c) * kChunk;
  if (slots) {
    const uint32_t e = slots[static_cast<size_t>(r) * chunks + c];
    return e < n && u[e] == r ? static_cast<int>(e) : -1;
  }
  uint32_t lo = 0, hi = n;
  while (lo < hi) {
    const uint32_t mid = (lo + hi) >> 1;
    if (u[mid] < r) lo = mid + 1;
    else hi = mid;
  }
  return lo < n && u[lo] == r ? static_cast<int>(lo) : -1;
}

// Phase 2: CTA (r, slice) writes dst[r, slice] = base[r, slice] + the chunk
// partials of row r, slice = 256 column groups of V.  Per round of 256
// chunks, the chunks holding r are listed in chunk order (ballots), and the
// list is cut into G contiguous parts, one per group of threads (G = 256 /
// columns groups of the slice); a group folds its part in order with kBatch
// loads in flight, and the G group sums are added in group order at the end:
// the summation order depends only on the ids (deterministic).
template <int V>
__global__ void __launch_bounds__(kThreads2)
row_combine_kernel(const float *__restrict__ partial, const uint32_t *__restrict__ uid,
                   const uint32_t *__restrict__ ucount, const uint32_t *__restrict__ slots,
                   uint32_t n_chunks, uint32_t dim, const float *base, float *dst) {
  pdl_enter();
  using Vec = typename VecOf<V>::T;
  __shared__ uint32_t list[kThreads2];
  __shared__ uint32_t warp_cnt[kThreads2 / 32];
  __shared__ float gsum[kThreads2 * V];
  const uint32_t t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const uint32_t r = blockIdx.x;
  const uint32_t cols = dim / V;
  const uint32_t col0 = blockIdx.y * kThreads2;
  const uint32_t width = min(kThreads2, cols - col0);  // column groups of this slice
  const uint32_t G = kThreads2 / width;                // thread groups
  const uint32_t g = t / width, cl = t % width;
  const bool active = g < G;
  float acc[V];
#pragma unroll
  for (int v = 0; v < V; ++v) acc[v] = 0.0f;
  for (uint32_t round = 0; round < n_chunks; round += kThreads2) {
    const uint32_t c = round + t;
    const int u = c < n_chunks ? find_slot(r, c, uid, ucount, slots, n_chunks) : -1;
    const uint32_t fb = __ballot_sync(0xffffffffu, u >= 0);
    if (lane == 0) warp_cnt[warp] = __popc(fb);
    __syncthreads();
    uint32_t before = 0, m = 0;
    for (uint32_t w = 0; w < kThreads2 / 32; ++w) {
      before += w < warp ? warp_cnt[w] : 0u;
      m += warp_cnt[w];
    }
    if (u >= 0)
      list[before + __popc(fb & ((1u << lane) - 1u))] =
          static_cast<uint32_t>(c) * kChunk + static_cast<uint32_t>(u);
    __syncthreads();
    if (active) {
      const uint32_t per = (m + G - 1) / G, k_begin = g * per, k_end = min(m, k_begin + per);
      for (uint32_t k0 = k_begin; k0 < k_end; k0 += kBatch) {
        Vec x[kBatch];
#pragma unroll
        for (uint32_t j = 0; j < kBatch; ++j)
          if (k0 + j < k_end)
            x[j] = *reinterpret_cast<const Vec *>(partial + static_cast<size_t>(list[k0 + j]) * dim +
                                                   static_cast<size_t>(col0 + cl) * V);
#pragma unroll
        for (uint32_t j = 0; j < kBatch; ++j)
          if (k0 + j < k_end) vadd<V>(acc, x[j]);
      }
    }
    __syncthreads();  // the list is rewritten next round
  }
  if (active) {
#pragma unroll
    for (int v = 0; v < V; ++v) gsum[t * V + v] = acc[v];
  }
  __syncthreads();
  if (g != 0) return;
  float s[V];
#pragma unroll
  for (int v = 0; v < V; ++v) s[v] = gsum[cl * V + v];
  for (uint32_t h = 1; h < G; ++h)
#pragma unroll
    for (int v = 0; v < V; ++v) s[v] += gsum[(h * width + cl) * V + v];
  const size_t o = static_cast<size_t>(r) * dim + static_cast<size_t>(col0 + cl) * V;
  if (base) {
    const Vec b = *reinterpret_cast<const Vec *>(base + o);
    float bb[V];
    if constexpr (V == 4) {
      bb[0] = b.x; bb[1] = b.y; bb[2] = b.z; bb[3] = b.w;
    } else {
      bb[0] = b;
    }
#pragma unroll
    for (int v = 0; v < V; ++v) s[v] = bb[v] + s[v];
  }
  vstore<V>(dst + o, s);
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

// Workspace layout: partial rows (chunks x kChunk x dim floats), the
// distinct ids per slot, one count per chunk, then (when it fits
// kMaxSlotTable) the slot table of n_rows x chunks words.
struct ScatterLayout {
  size_t partial_bytes, uid_bytes, count_bytes, table_offset, table_bytes, total;
};

ScatterLayout scatter_layout(uint32_t n_ids, uint32_t n_rows, uint32_t dim) {
  ScatterLayout l{};
  const size_t chunks = scatter_chunks(n_ids), slots = chunks * kChunk;
  l.partial_bytes = slots * dim * sizeof(float);
  l.uid_bytes = slots * sizeof(uint32_t);
  l.count_bytes = chunks * sizeof(uint32_t);
  l.table_offset = (l.partial_bytes + l.uid_bytes + l.count_bytes + 15) & ~size_t(15);
  const size_t table = static_cast<size_t>(n_rows) * chunks * sizeof(uint32_t);
  l.table_bytes = table <= kMaxSlotTable ? table : 0;
  l.total = l.table_offset + l.table_bytes;
  return l;
}
}  // namespace

size_t tl_embedding_scatter_workspace_size(uint32_t n_ids, uint32_t n_rows, uint32_t dim) {
  return n_ids ? scatter_layout(n_ids, n_rows, dim).total : 0;
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
  const ScatterLayout l = scatter_layout(n_ids, n_rows, dim);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  float *partial = reinterpret_cast<float *>(ws);
  uint32_t *uid = reinterpret_cast<uint32_t *>(ws + l.partial_bytes);
  uint32_t *ucount = reinterpret_cast<uint32_t *>(ws + l.partial_bytes + l.uid_bytes);
  uint32_t *table = l.table_bytes ? reinterpret_cast<uint32_t *>(ws + l.table_offset) : nullptr;
  const bool vec = dim % 4 == 0 && aligned16(values) && aligned16(dst) &&
                   (!base || aligned16(base)) && aligned16(workspace);
  if (chunks) {
    if (vec)
      launch_pdl(chunk_sum_kernel<4>, chunks, kThreads1, 0, s, values, ids, n_ids, dim, n_rows,
                 partial, uid, ucount, table, chunks, status);
    else
      launch_pdl(chunk_sum_kernel<1>, chunks, kThreads1, 0, s, values, ids, n_ids, dim, n_rows,
                 partial, uid, ucount, table, chunks, status);
    const int rc = launch_status("tl_embedding_scatter_add chunks");
    if (rc) return rc;
  }
  const uint32_t cols = vec ? dim / 4 : dim;
  const dim3 grid(n_rows, (cols + kThreads2 - 1) / kThreads2);
  if (vec)
    launch_pdl(row_combine_kernel<4>, grid, kThreads2, 0, s, partial, uid, ucount,
               static_cast<const uint32_t *>(table), chunks, dim, base, dst);
  else
    launch_pdl(row_combine_kernel<1>, grid, kThreads2, 0, s, partial, uid, ucount,
               static_cast<const uint32_t *>(table), chunks, dim, base, dst);
  return launch_status("tl_embedding_scatter_add rows");
}

}  // extern "C"

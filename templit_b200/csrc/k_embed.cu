// Embedding gather and deterministic scatter-add
// (Runtime::embedding_lookup / scatter_add_rows / scatter_index,
// src/my_metal/runtime.cpp:920-1030; math.metal:778-820).
//
// The reference scatters with one float atomic per element, so its result
// depends on arrival order.  Here the scatter is a stable counting sort of
// the ids (one CTA: histogram, scan, stable placement through warp match
// masks) followed by a gather-sum per destination row in input order, which
// makes every run bit-identical.  Ids outside the table never touch memory:
// they raise TL_FLAG_INDEX_RANGE in the device status word instead.
#include "tl_common.cuh"

namespace tl {
namespace {

template <int V>
__global__ void __launch_bounds__(256)
gather_kernel(const float *__restrict__ w, uint32_t n_rows, uint32_t dim,
              const uint32_t *__restrict__ ids, uint32_t n_ids, float *out,
              uint32_t *status) {
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

constexpr int kSortThreads = 1024;

// Stable counting sort of ids into order[] (positions grouped by id, input
// order inside a group) and offsets[r]..offsets[r+1] bounds of group r.
// One CTA; counts/offsets live in `offsets` (n_rows + 1 words).
__global__ void __launch_bounds__(kSortThreads)
bucket_kernel(const uint32_t *__restrict__ ids, uint32_t n_ids, uint32_t n_rows,
              uint32_t *offsets, uint32_t *order, uint32_t *status) {
  // 1. histogram
  for (uint32_t r = threadIdx.x; r <= n_rows; r += blockDim.x) offsets[r] = 0;
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < n_ids; i += blockDim.x) {
    const uint32_t id = ids[i];
    if (id < n_rows) atomicAdd(&offsets[id + 1], 1u);
    else raise_flag(status, TL_FLAG_INDEX_RANGE);
  }
  __syncthreads();
  // 2. inclusive scan of offsets[1..n_rows] -> exclusive starts
  __shared__ uint32_t carry;
  __shared__ uint32_t warp_tot[kSortThreads / 32];
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (uint32_t base = 1; base <= n_rows; base += blockDim.x) {
    const uint32_t r = base + threadIdx.x;
    uint32_t v = r <= n_rows ? offsets[r] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= static_cast<uint32_t>(o)) v += u;
    }
    if (lane == 31) warp_tot[warp] = v;
    __syncthreads();
    if (warp == 0) {
      uint32_t w = lane < blockDim.x / 32 ? warp_tot[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t u = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= static_cast<uint32_t>(o)) w += u;
      }
      warp_tot[lane] = w;  // inclusive warp prefix
    }
    __syncthreads();
    const uint32_t add = carry + (warp ? warp_tot[warp - 1] : 0);
    if (r <= n_rows) offsets[r] = v + add;
    __syncthreads();
    if (threadIdx.x == 0) carry += warp_tot[blockDim.x / 32 - 1];
    __syncthreads();
  }
  // 3. stable placement: chunks of blockDim ids in order; inside a chunk the
  //    warps take turns so earlier positions claim earlier slots.
  for (uint32_t base = 0; base < n_ids; base += blockDim.x) {
    const uint32_t i = base + threadIdx.x;
    const uint32_t id = i < n_ids ? ids[i] : 0xffffffffu;
    const bool valid = i < n_ids && id < n_rows;
    const uint32_t key = valid ? id : 0xffffffffu;
    const uint32_t peers = __match_any_sync(0xffffffffu, key);
    const uint32_t rank = __popc(peers & ((1u << lane) - 1u));
    const bool leader = rank == 0;
    const uint32_t group = __popc(peers);
    for (uint32_t w = 0; w < blockDim.x / 32; ++w) {
      if (warp == w && valid) {
        // offsets[id] is the running insert cursor of bucket id
        uint32_t start = 0;
        if (leader) start = atomicAdd(&offsets[id], group);
        const int src = __ffs(peers) - 1;
        start = __shfl_sync(peers, start, src);
        order[start + rank] = i;
      }
      __syncthreads();
    }
  }
  // offsets[r] now holds the end of bucket r (the insert cursor ran through it)
}

// After bucket_kernel offsets[r] = end of bucket r (the cursor ran to the end)
// so bucket r spans [r ? offsets[r-1] : 0, offsets[r]).
template <int V>
__global__ void __launch_bounds__(256)
segment_sum_kernel(const float *__restrict__ values, const uint32_t *__restrict__ order,
                   const uint32_t *__restrict__ ends, uint32_t dim, uint32_t n_rows,
                   const float *base, float *dst) {
  const uint32_t per_row = dim / V;
  const uint64_t total = static_cast<uint64_t>(n_rows) * per_row;
  const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  for (uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       t < total; t += stride) {
    const uint32_t r = static_cast<uint32_t>(t / per_row);
    const uint32_t c = static_cast<uint32_t>(t % per_row) * V;
    const uint32_t b = r ? ends[r - 1] : 0u, e = ends[r];
    const size_t o = static_cast<size_t>(r) * dim + c;
    if constexpr (V == 4) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (uint32_t k = b; k < e; ++k) {
        const float4 v = *reinterpret_cast<const float4 *>(values + static_cast<size_t>(order[k]) * dim + c);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      if (base) {
        const float4 bv = *reinterpret_cast<const float4 *>(base + o);
        acc.x = bv.x + acc.x;
        acc.y = bv.y + acc.y;
        acc.z = bv.z + acc.z;
        acc.w = bv.w + acc.w;
      }
      *reinterpret_cast<float4 *>(dst + o) = acc;
    } else {
      float acc = 0.0f;
      for (uint32_t k = b; k < e; ++k) acc += values[static_cast<size_t>(order[k]) * dim + c];
      dst[o] = base ? base[o] + acc : acc;
    }
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
    gather_kernel<4><<<grid_for(total / 4, 256), 256, 0, s>>>(weights, n_rows, dim, ids, n_ids, out, status);
  else
    gather_kernel<1><<<grid_for(total, 256), 256, 0, s>>>(weights, n_rows, dim, ids, n_ids, out, status);
  return launch_status("tl_embedding_gather");
}

size_t tl_embedding_scatter_workspace_size(uint32_t n_ids, uint32_t n_rows) {
  return (static_cast<size_t>(n_rows) + 1 + n_ids) * sizeof(uint32_t);
}

int tl_embedding_scatter_add(const float *values, const uint32_t *ids,
                             uint32_t n_ids, uint32_t dim, const float *base,
                             float *dst, uint32_t n_rows, void *workspace,
                             size_t workspace_bytes, void *stream) {
  if (n_rows == 0 || dim == 0) return TL_OK;
  if (!dst || (n_ids && (!values || !ids)))
    return fail(TL_ERR_INVALID, "tl_embedding_scatter_add: null pointer");
  if (!workspace || workspace_bytes < tl_embedding_scatter_workspace_size(n_ids, n_rows))
    return fail(TL_ERR_INVALID, "tl_embedding_scatter_add: workspace too small");
  uint32_t *status = device_status_ptr();
  if (!status) return fail(TL_ERR_CUDA, "tl_embedding_scatter_add: no status word");
  cudaStream_t s = as_stream(stream);
  uint32_t *offsets = static_cast<uint32_t *>(workspace);
  uint32_t *order = offsets + n_rows + 1;
  bucket_kernel<<<1, kSortThreads, 0, s>>>(ids, n_ids, n_rows, offsets, order, status);
  int rc = launch_status("tl_embedding_scatter_add bucket");
  if (rc) return rc;
  // the placement cursor ends each bucket at its end: bucket r = [ends[r-1], ends[r])
  const uint64_t total = static_cast<uint64_t>(n_rows) * dim;
  const bool vec = dim % 4 == 0 && aligned16(values) && aligned16(dst) && (!base || aligned16(base));
  if (vec)
    segment_sum_kernel<4><<<grid_for(total / 4, 256), 256, 0, s>>>(values, order, offsets, dim, n_rows, base, dst);
  else
    segment_sum_kernel<1><<<grid_for(total, 256), 256, 0, s>>>(values, order, offsets, dim, n_rows, base, dst);
  return launch_status("tl_embedding_scatter_add sum");
}

}  // extern "C"

// Optimiser kernels: gradient squared norm, clipping, AdamW, and the fused
// multi-tensor clip + AdamW pass that replaces the whole
// `Compiled::step(max_norm)` program (include/passes/compile.h:236-258).
//
// Reference semantics (include/my_metal/math.metal:955-1043):
//   sqnorm += sum(g^2)                        (atomic per threadgroup)
//   g'  = g * min(1, c * rsqrt(max(sqnorm, 1e-12)))
//   m   = b1*m + (1-b1)*g';   v = b2*v + (1-b2)*g'*g'
//   p'  = p*decay - lr*(m/(1-b1^t)) / (sqrt(v/(1-b2^t)) + eps)
// The norm here is deterministic: per-CTA partial sums in a workspace,
// combined in CTA order (by a single-CTA pass, or in the multi-tensor
// kernel by its last CTA).
#include "tl_common.cuh"

namespace tl {
namespace {

constexpr int kNormThreads = 256;

__device__ __forceinline__ float block_sum(float v) {
  __shared__ float part[kNormThreads / 32];
  v = warp_sum(v);
  const int w = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (lane == 0) part[w] = v;
  __syncthreads();
  float r = 0.0f;
  if (w == 0) {
    r = lane < static_cast<int>(blockDim.x / 32) ? part[lane] : 0.0f;
    r = warp_sum(r);
  }
  __syncthreads();
  return r;  // valid in thread 0
}

__global__ void __launch_bounds__(kNormThreads)
sqnorm_partial_kernel(const float *__restrict__ g, size_t n, float *partial,
                      float *sqnorm) {
  pdl_enter();
  float acc = 0.0f;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t t0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (aligned16(g)) {
    const size_t n4 = n / 4;
    for (size_t i = t0; i < n4; i += stride) {
      const float4 v = reinterpret_cast<const float4 *>(g)[i];
      acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    for (size_t i = n4 * 4 + t0; i < n; i += stride) acc += g[i] * g[i];
  } else {
    for (size_t i = t0; i < n; i += stride) acc += g[i] * g[i];
  }
  const float total = block_sum(acc);
  if (threadIdx.x == 0) {
    if (partial) partial[blockIdx.x] = total;
    else *sqnorm += total;  // single CTA: accumulate directly
  }
}

__global__ void __launch_bounds__(kNormThreads)
sqnorm_combine_kernel(const float *__restrict__ partial, uint32_t count,
                      float *sqnorm) {
  pdl_enter();
  float acc = 0.0f;
  // fixed assignment of partials to threads, then a fixed-shape tree
  for (uint32_t i = threadIdx.x; i < count; i += blockDim.x) acc += partial[i];
  const float total = block_sum(acc);
  if (threadIdx.x == 0) *sqnorm += total;
}

__device__ __forceinline__ float clip_scale(float n2, float max_norm) {
  return fminf(1.0f, max_norm * rsqrtf(fmaxf(n2, 1e-12f)));
}

__global__ void __launch_bounds__(256)
clip_kernel(const float *__restrict__ g, const float *__restrict__ sqnorm,
            float max_norm, float *out, size_t n) {
  pdl_enter();
  const float sc = clip_scale(*sqnorm, max_norm);
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride)
    out[i] = g[i] * sc;
}

struct AdamScalars {
  float b1, b2, decay, lr, c1, c2;
};

__device__ __forceinline__ AdamScalars load_adam(const float *beta1, const float *beta2,
                                                 const float *decay, const float *lr,
                                                 uint32_t step) {
  AdamScalars a;
  a.b1 = *beta1;
  a.b2 = *beta2;
  a.decay = *decay;
  a.lr = *lr;
  a.c1 = 1.0f - powf(a.b1, static_cast<float>(step));
  a.c2 = 1.0f - powf(a.b2, static_cast<float>(step));
  return a;
}

__device__ __forceinline__ float adam_update(const AdamScalars &a, float p, float g,
                                             float &m, float &v, float eps) {
  m = a.b1 * m + (1.0f - a.b1) * g;
  v = a.b2 * v + (1.0f - a.b2) * g * g;
  return p * a.decay - a.lr * (m / a.c1) / (sqrtf(v / a.c2) + eps);
}

__global__ void __launch_bounds__(256)
adamw_kernel(const float *param, const float *__restrict__ grad, float *out,
             float *m1, float *m2, const float *beta1, const float *beta2,
             const float *decay, const float *lr, float eps, uint32_t step,
             size_t n) {
  pdl_enter();
  const AdamScalars a = load_adam(beta1, beta2, decay, lr, step);
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    float m = m1[i], v = m2[i];
    const float r = adam_update(a, param[i], grad[i], m, v, eps);
    m1[i] = m;
    m2[i] = v;
    out[i] = r;
  }
}

// ---- multi-tensor: work is split into TL_OPT_CHUNK-element chunks per slot
__device__ __forceinline__ uint32_t find_slot(const tl_param_slot *slots,
                                              uint32_t n_slots, uint32_t chunk) {
  uint32_t lo = 0, hi = n_slots;  // last slot with chunk0 <= chunk
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) / 2;
    if (slots[mid].chunk0 <= chunk) lo = mid;
    else hi = mid;
  }
  return lo;
}

// Arrival counter of multi_sqnorm_kernel's CTAs (self-resetting: the last
// CTA of a launch wraps it back to 0).
static __device__ unsigned int g_norm_ticket;

// sqnorm[0] += sum over all slots of grad^2.  CTA b sums the chunks b, b +
// grid, ... (a full, aligned chunk as 8 float4 loads per thread in flight),
// writes its partial, and the last CTA to arrive adds the partials in CTA
// order with a fixed-shape tree: deterministic, one launch.
__global__ void __launch_bounds__(kNormThreads)
multi_sqnorm_kernel(const tl_param_slot *__restrict__ slots, uint32_t n_slots,
                    uint32_t n_chunks, float *partial, float *sqnorm) {
  pdl_enter();
  __shared__ bool last;
  constexpr uint32_t kPer = TL_OPT_CHUNK / (kNormThreads * 4);  // float4 per thread
  float acc = 0.0f;
  for (uint32_t c = blockIdx.x; c < n_chunks; c += gridDim.x) {
    const tl_param_slot &sl = slots[find_slot(slots, n_slots, c)];
    const uint64_t begin = static_cast<uint64_t>(c - sl.chunk0) * TL_OPT_CHUNK;
    const uint64_t end = min(sl.count, begin + TL_OPT_CHUNK);
    const float *g = sl.grad;
    if (aligned16(g) && (begin % 4) == 0 && end - begin == TL_OPT_CHUNK) {
      float4 v[kPer];
#pragma unroll
      for (uint32_t j = 0; j < kPer; ++j)
        v[j] = *reinterpret_cast<const float4 *>(g + begin + (j * kNormThreads + threadIdx.x) * 4);
#pragma unroll
      for (uint32_t j = 0; j < kPer; ++j)
        acc += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    } else if (aligned16(g) && (begin % 4) == 0) {
      const uint64_t e4 = begin + ((end - begin) / 4) * 4;
      for (uint64_t i = begin + threadIdx.x * 4; i < e4; i += blockDim.x * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(g + i);
        acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
      for (uint64_t i = e4 + threadIdx.x; i < end; i += blockDim.x) acc += g[i] * g[i];
    } else {
      for (uint64_t i = begin + threadIdx.x; i < end; i += blockDim.x) acc += g[i] * g[i];
    }
  }
  const float total = block_sum(acc);
  if (threadIdx.x == 0) {
    partial[blockIdx.x] = total;
    last = ticket_acq_rel(&g_norm_ticket, gridDim.x - 1) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  float a = 0.0f;
  for (uint32_t i = threadIdx.x; i < gridDim.x; i += blockDim.x) a += __ldcg(partial + i);
  const float all = block_sum(a);
  if (threadIdx.x == 0) *sqnorm += all;
}

__global__ void __launch_bounds__(256)
multi_clip_adamw_kernel(const tl_param_slot *__restrict__ slots, uint32_t n_slots,
                        uint32_t n_chunks, const float *__restrict__ sqnorm,
                        float max_norm, const float *beta1, const float *beta2,
                        const float *decay, const float *lr, float eps) {
  pdl_enter();
  const bool clip = max_norm > 0.0f;
  const float sc = clip ? clip_scale(*sqnorm, max_norm) : 1.0f;
  const float b1 = *beta1, b2 = *beta2, dc = *decay, lrv = *lr;
  for (uint32_t c = blockIdx.x; c < n_chunks; c += gridDim.x) {
    const tl_param_slot &sl = slots[find_slot(slots, n_slots, c)];
    AdamScalars a;
    a.b1 = b1;
    a.b2 = b2;
    a.decay = dc;
    a.lr = lrv;
    a.c1 = 1.0f - powf(b1, static_cast<float>(sl.step));
    a.c2 = 1.0f - powf(b2, static_cast<float>(sl.step));
    const uint64_t begin = static_cast<uint64_t>(c - sl.chunk0) * TL_OPT_CHUNK;
    const uint64_t end = min(sl.count, begin + TL_OPT_CHUNK);
    const bool vec = aligned16(sl.param) && aligned16(sl.out) && aligned16(sl.grad) &&
                     aligned16(sl.m1) && aligned16(sl.m2) && (begin % 4) == 0;
    uint64_t i0 = begin;
    if (vec) {
      const uint64_t e4 = begin + ((end - begin) / 4) * 4;
      for (uint64_t i = begin + threadIdx.x * 4; i < e4; i += blockDim.x * 4) {
        float4 g = *reinterpret_cast<const float4 *>(sl.grad + i);
        if (clip) {
          g.x *= sc;
          g.y *= sc;
          g.z *= sc;
          g.w *= sc;
          *reinterpret_cast<float4 *>(sl.grad + i) = g;
        }
        const float4 p = *reinterpret_cast<const float4 *>(sl.param + i);
        float4 m = *reinterpret_cast<const float4 *>(sl.m1 + i);
        float4 v = *reinterpret_cast<const float4 *>(sl.m2 + i);
        float4 r;
        r.x = adam_update(a, p.x, g.x, m.x, v.x, eps);
        r.y = adam_update(a, p.y, g.y, m.y, v.y, eps);
        r.z = adam_update(a, p.z, g.z, m.z, v.z, eps);
        r.w = adam_update(a, p.w, g.w, m.w, v.w, eps);
        *reinterpret_cast<float4 *>(sl.m1 + i) = m;
        *reinterpret_cast<float4 *>(sl.m2 + i) = v;
        *reinterpret_cast<float4 *>(sl.out + i) = r;
      }
      i0 = e4;
    }
    for (uint64_t i = i0 + threadIdx.x; i < end; i += blockDim.x) {
      float g = sl.grad[i];
      if (clip) {
        g *= sc;
        sl.grad[i] = g;
      }
      float m = sl.m1[i], v = sl.m2[i];
      const float r = adam_update(a, sl.param[i], g, m, v, eps);
      sl.m1[i] = m;
      sl.m2[i] = v;
      sl.out[i] = r;
    }
  }
}

uint32_t norm_blocks(size_t n) { return grid_for((n + 3) / 4, kNormThreads, 4); }

// Gradients <-> one flat buffer in the slots' chunk layout (slot i's
// element e at flat[chunk0 * TL_OPT_CHUNK + e]): CTA b moves chunks b,
// b + grid, ... (float4 when the gradient is 16-byte aligned).
__global__ void __launch_bounds__(256)
multi_grad_flat_kernel(const tl_param_slot *__restrict__ slots, uint32_t n_slots,
                       uint32_t n_chunks, float *flat, int unpack) {
  pdl_enter();
  for (uint32_t c = blockIdx.x; c < n_chunks; c += gridDim.x) {
    const tl_param_slot &sl = slots[find_slot(slots, n_slots, c)];
    const uint64_t begin = static_cast<uint64_t>(c - sl.chunk0) * TL_OPT_CHUNK;
    const uint64_t end = min(sl.count, begin + TL_OPT_CHUNK);
    float *g = sl.grad;
    float *f = flat + static_cast<uint64_t>(sl.chunk0) * TL_OPT_CHUNK;
    if (aligned16(g)) {  // begin is a multiple of TL_OPT_CHUNK: f + i is aligned too
      const uint64_t vend = begin + ((end - begin) & ~static_cast<uint64_t>(3));
      for (uint64_t i = begin + 4 * threadIdx.x; i < vend; i += 4 * blockDim.x) {
        if (unpack)
          *reinterpret_cast<float4 *>(g + i) = __ldcs(reinterpret_cast<const float4 *>(f + i));
        else
          *reinterpret_cast<float4 *>(f + i) = *reinterpret_cast<const float4 *>(g + i);
      }
      const uint64_t i = vend + threadIdx.x;  // the last 0 - 3 elements
      if (i < end) {
        if (unpack) g[i] = f[i];
        else f[i] = g[i];
      }
    } else {
      for (uint64_t i = begin + threadIdx.x; i < end; i += blockDim.x) {
        if (unpack) g[i] = f[i];
        else f[i] = g[i];
      }
    }
  }
}

uint32_t multi_blocks(uint32_t n_chunks) {
  return n_chunks < static_cast<uint32_t>(kNumSMs * 4) ? n_chunks : kNumSMs * 4;
}

}  // namespace
}  // namespace tl

using namespace tl;

extern "C" {

size_t tl_grad_sqnorm_workspace_size(size_t count) {
  const uint32_t b = norm_blocks(count);
  return b > 1 ? b * sizeof(float) : 0;
}

int tl_grad_sqnorm_accumulate(const float *grad, size_t count, float *sqnorm,
                              void *workspace, size_t workspace_bytes, void *stream) {
  if (!sqnorm) return fail(TL_ERR_INVALID, "tl_grad_sqnorm_accumulate: null sqnorm");
  if (count == 0) return TL_OK;
  if (!grad) return fail(TL_ERR_INVALID, "tl_grad_sqnorm_accumulate: null gradient");
  const uint32_t blocks = norm_blocks(count);
  cudaStream_t s = as_stream(stream);
  if (blocks == 1) {
    launch_pdl(sqnorm_partial_kernel, 1, kNormThreads, 0, s, grad, count, nullptr, sqnorm);
    return launch_status("tl_grad_sqnorm_accumulate");
  }
  if (!workspace || workspace_bytes < blocks * sizeof(float))
    return fail(TL_ERR_INVALID, "tl_grad_sqnorm_accumulate: workspace too small");
  float *partial = static_cast<float *>(workspace);
  launch_pdl(sqnorm_partial_kernel, blocks, kNormThreads, 0, s, grad, count, partial, sqnorm);
  int rc = launch_status("tl_grad_sqnorm_accumulate partial");
  if (rc) return rc;
  launch_pdl(sqnorm_combine_kernel, 1, kNormThreads, 0, s, partial, blocks, sqnorm);
  return launch_status("tl_grad_sqnorm_accumulate combine");
}

int tl_clip_gradient(const float *grad, const float *sqnorm, float max_norm,
                     float *out, size_t count, void *stream) {
  if (!(max_norm > 0.0f) || !std::isfinite(max_norm))
    return fail(TL_ERR_INVALID, "maximum gradient norm must be finite and positive");
  if (count == 0) return TL_OK;
  if (!grad || !sqnorm || !out) return fail(TL_ERR_INVALID, "tl_clip_gradient: null pointer");
  launch_pdl(clip_kernel, grid_for(count, 256), 256, 0, as_stream(stream), grad, sqnorm, max_norm,
                                                                   out, count);
  return launch_status("tl_clip_gradient");
}

int tl_adamw(const float *param, const float *grad, float *out, float *m1, float *m2,
             const float *beta1, const float *beta2, const float *decay,
             const float *lr, float epsilon, uint32_t step, size_t count,
             void *stream) {
  if (step == 0) return fail(TL_ERR_INVALID, "AdamW step must be greater than zero");
  if (count == 0) return TL_OK;
  if (!param || !grad || !out || !m1 || !m2 || !beta1 || !beta2 || !decay || !lr)
    return fail(TL_ERR_INVALID, "tl_adamw: null pointer");
  launch_pdl(adamw_kernel, grid_for(count, 256), 256, 0, as_stream(stream), 
      param, grad, out, m1, m2, beta1, beta2, decay, lr, epsilon, step, count);
  return launch_status("tl_adamw");
}

size_t tl_multi_clip_adamw_workspace_size(uint32_t n_chunks) {
  return static_cast<size_t>(multi_blocks(n_chunks)) * sizeof(float);
}

int tl_multi_grad_flat(const tl_param_slot *slots, uint32_t n_slots, uint32_t n_chunks,
                       float *flat, int unpack, void *stream) {
  if (n_slots == 0 || n_chunks == 0) return TL_OK;
  if (!slots || !flat) return fail(TL_ERR_INVALID, "tl_multi_grad_flat: null pointer");
  if (!aligned16(flat)) return fail(TL_ERR_INVALID, "tl_multi_grad_flat: flat not 16-byte aligned");
  launch_pdl(multi_grad_flat_kernel, multi_blocks(n_chunks), 256, 0, as_stream(stream), slots,
             n_slots, n_chunks, flat, unpack ? 1 : 0);
  return launch_status("tl_multi_grad_flat");
}

int tl_multi_clip_adamw(const tl_param_slot *slots, uint32_t n_slots, uint32_t n_chunks,
                        float *sqnorm, float max_norm, const float *beta1,
                        const float *beta2, const float *decay, const float *lr,
                        float epsilon, void *workspace, size_t workspace_bytes,
                        void *stream) {
  if (n_slots == 0 || n_chunks == 0) return TL_OK;
  if (!slots || !beta1 || !beta2 || !decay || !lr)
    return fail(TL_ERR_INVALID, "tl_multi_clip_adamw: null pointer");
  const bool clip = max_norm > 0.0f;
  if (clip && (!std::isfinite(max_norm) || !sqnorm))
    return fail(TL_ERR_INVALID, "tl_multi_clip_adamw: bad clipping arguments");
  const uint32_t blocks = multi_blocks(n_chunks);
  cudaStream_t s = as_stream(stream);
  if (clip) {
    if (!workspace || workspace_bytes < blocks * sizeof(float))
      return fail(TL_ERR_INVALID, "tl_multi_clip_adamw: workspace too small");
    float *partial = static_cast<float *>(workspace);
    launch_pdl(multi_sqnorm_kernel, blocks, kNormThreads, 0, s, slots, n_slots, n_chunks, partial,
               sqnorm);
    const int rc = launch_status("tl_multi_clip_adamw norm");
    if (rc) return rc;
  }
  launch_pdl(multi_clip_adamw_kernel, blocks, 256, 0, s, slots, n_slots, n_chunks, sqnorm, max_norm,
                                                 beta1, beta2, decay, lr, epsilon);
  return launch_status("tl_multi_clip_adamw update");
}

}  // extern "C"

// Row operators over the last dimension: softmax (+ backward), RMS, RMSNorm
// (+ backward) and softmax cross-entropy (+ backward).
//
// The reference runs these one thread per row with three serial passes
// (include/my_metal/math.metal:857-953) and composes RMS/RMSNorm and their
// derivatives from five to seven separate dispatches
// (src/my_metal/runtime.cpp:1031-1072; include/passes/execute.h:291-356).
// Here one warp owns a row: a first pass over the row keeps a per-lane online
// (max, sum-of-exp) or sum-of-squares in registers and merges it across the
// warp with shuffles, a second pass writes the result (the re-read is served
// from L1/L2).  Rows are 128-bit vectorised when the row length allows.
#include "tl_common.cuh"

#include <initializer_list>

namespace tl {
namespace {

constexpr int kWarpsPerBlock = 8;

// Adds one term to a running (max, sum of exp(x - max)).  A -inf term (a
// masked score) contributes nothing, also while the running max is still
// -inf; a NaN term poisons the sum as it does in the reference kernel.
__device__ __forceinline__ void online_add(float &m, float &s, float x) {
  if (x > m) {
    s = s * expf(m - x) + 1.0f;
    m = x;
  } else if (x != -INFINITY) {
    s += expf(x - m);
  }
}

__device__ __forceinline__ void warp_online(float &m, float &s) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
}

// Per-lane (max, sum exp) over a row, merged across the warp.
__device__ __forceinline__ void row_logsumexp(const float *xr, uint32_t cols,
                                              bool vec, uint32_t lane, float &m,
                                              float &s) {
  m = -INFINITY;
  s = 0.0f;
  if (vec) {
    for (uint32_t c = lane * 4; c < cols; c += 128) {
      const float4 v = *reinterpret_cast<const float4 *>(xr + c);
      online_add(m, s, v.x);
      online_add(m, s, v.y);
      online_add(m, s, v.z);
      online_add(m, s, v.w);
    }
  } else {
    for (uint32_t c = lane; c < cols; c += 32) online_add(m, s, xr[c]);
  }
  warp_online(m, s);
}

__device__ __forceinline__ float row_dot(const float *a, const float *b,
                                         uint32_t cols, bool vec, uint32_t lane) {
  float acc = 0.0f;
  if (vec) {
    for (uint32_t c = lane * 4; c < cols; c += 128) {
      const float4 u = *reinterpret_cast<const float4 *>(a + c);
      const float4 w = *reinterpret_cast<const float4 *>(b + c);
      acc += u.x * w.x + u.y * w.y + u.z * w.z + u.w * w.w;
    }
  } else {
    for (uint32_t c = lane; c < cols; c += 32) acc += a[c] * b[c];
  }
  return warp_sum(acc);
}

#define ROW_LOOP                                                             \
  const uint32_t lane = threadIdx.x & 31;                                    \
  const uint32_t warps = gridDim.x * kWarpsPerBlock;                         \
  for (uint32_t row = blockIdx.x * kWarpsPerBlock + threadIdx.x / 32;        \
       row < rows; row += warps)

__global__ void __launch_bounds__(256)
softmax_kernel(const float *__restrict__ x, float *out, uint32_t rows,
               uint32_t cols, bool vec) {
  pdl_enter();
  ROW_LOOP {
    const float *xr = x + static_cast<size_t>(row) * cols;
    float *yr = out + static_cast<size_t>(row) * cols;
    float m, s;
    row_logsumexp(xr, cols, vec, lane, m, s);
    if (vec) {
      for (uint32_t c = lane * 4; c < cols; c += 128) {
        float4 v = *reinterpret_cast<const float4 *>(xr + c);
        v.x = expf(v.x - m) / s;
        v.y = expf(v.y - m) / s;
        v.z = expf(v.z - m) / s;
        v.w = expf(v.w - m) / s;
        *reinterpret_cast<float4 *>(yr + c) = v;
      }
    } else {
      for (uint32_t c = lane; c < cols; c += 32) yr[c] = expf(xr[c] - m) / s;
    }
  }
}

// out = softmax(x / divisor[0] + mask[row % mask_rows, :]): the attention
// score chain of nn::MultiHeadAttention (divide by sqrt(head size), add the
// causal mask, soft_max; include/nn/multi_head.h) in one pass.  Each element
// is transformed exactly as the separate divide and add kernels would, in
// the same per-lane order, so the result is bit-identical to the chain.
__device__ __forceinline__ float score(float x, const float *dv, const float *mr, uint32_t c) {
  if (dv) x = x / *dv;
  if (mr) x = x + mr[c];
  return x;
}

__global__ void __launch_bounds__(256)
softmax_scaled_masked_kernel(const float *__restrict__ x, const float *__restrict__ divisor,
                             const float *__restrict__ mask, uint32_t mask_rows, float *out,
                             uint32_t rows, uint32_t cols, bool vec) {
  pdl_enter();
  ROW_LOOP {
    const float *xr = x + static_cast<size_t>(row) * cols;
    const float *mr = mask ? mask + static_cast<size_t>(row % mask_rows) * cols : nullptr;
    float *yr = out + static_cast<size_t>(row) * cols;
    float m = -INFINITY, s = 0.0f;
    if (vec) {
      for (uint32_t c = lane * 4; c < cols; c += 128) {
        const float4 v = *reinterpret_cast<const float4 *>(xr + c);
        online_add(m, s, score(v.x, divisor, mr, c));
        online_add(m, s, score(v.y, divisor, mr, c + 1));
        online_add(m, s, score(v.z, divisor, mr, c + 2));
        online_add(m, s, score(v.w, divisor, mr, c + 3));
      }
    } else {
      for (uint32_t c = lane; c < cols; c += 32) online_add(m, s, score(xr[c], divisor, mr, c));
    }
    warp_online(m, s);
    if (vec) {
      for (uint32_t c = lane * 4; c < cols; c += 128) {
        float4 v = *reinterpret_cast<const float4 *>(xr + c);
        v.x = expf(score(v.x, divisor, mr, c) - m) / s;
        v.y = expf(score(v.y, divisor, mr, c + 1) - m) / s;
        v.z = expf(score(v.z, divisor, mr, c + 2) - m) / s;
        v.w = expf(score(v.w, divisor, mr, c + 3) - m) / s;
        *reinterpret_cast<float4 *>(yr + c) = v;
      }
    } else {
      for (uint32_t c = lane; c < cols; c += 32) yr[c] = expf(score(xr[c], divisor, mr, c) - m) / s;
    }
  }
}

// dx = y * (g - sum(g*y)) (then / divisor[0] when given: the derivative of
// the score division that precedes the softmax, folded in)
__device__ __forceinline__ float div_opt(float v, const float *d) { return d ? v / *d : v; }

__global__ void __launch_bounds__(256)
softmax_backward_kernel(const float *__restrict__ g, const float *__restrict__ y,
                        const float *__restrict__ divisor, float *dx, uint32_t rows,
                        uint32_t cols, bool vec) {
  pdl_enter();
  ROW_LOOP {
    const size_t off = static_cast<size_t>(row) * cols;
    const float dot = row_dot(g + off, y + off, cols, vec, lane);
    if (vec) {
      for (uint32_t c = lane * 4; c < cols; c += 128) {
        const float4 gv = *reinterpret_cast<const float4 *>(g + off + c);
        const float4 yv = *reinterpret_cast<const float4 *>(y + off + c);
        float4 r;
        r.x = div_opt(yv.x * (gv.x - dot), divisor);
        r.y = div_opt(yv.y * (gv.y - dot), divisor);
        r.z = div_opt(yv.z * (gv.z - dot), divisor);
        r.w = div_opt(yv.w * (gv.w - dot), divisor);
        *reinterpret_cast<float4 *>(dx + off + c) = r;
      }
    } else {
      for (uint32_t c = lane; c < cols; c += 32)
        dx[off + c] = div_opt(y[off + c] * (g[off + c] - dot), divisor);
    }
  }
}

__device__ __forceinline__ float row_rms(const float *xr, uint32_t cols, bool vec,
                                         uint32_t lane) {
  const float ss = row_dot(xr, xr, cols, vec, lane);
  return sqrtf(ss / static_cast<float>(cols) + 1e-6f);
}

__global__ void __launch_bounds__(256)
rms_kernel(const float *__restrict__ x, float *rms, uint32_t rows, uint32_t cols,
           bool vec) {
  pdl_enter();
  ROW_LOOP {
    const float r = row_rms(x + static_cast<size_t>(row) * cols, cols, vec, lane);
    if (lane == 0) rms[row] = r;
  }
}

__global__ void __launch_bounds__(256)
rmsnorm_kernel(const float *__restrict__ x, float *out, float *rms_out,
               uint32_t rows, uint32_t cols, bool vec) {
  pdl_enter();
  ROW_LOOP {
    const float *xr = x + static_cast<size_t>(row) * cols;
    float *yr = out + static_cast<size_t>(row) * cols;
    const float r = row_rms(xr, cols, vec, lane);
    if (rms_out && lane == 0) rms_out[row] = r;
    if (vec) {
      for (uint32_t c = lane * 4; c < cols; c += 128) {
        float4 v = *reinterpret_cast<const float4 *>(xr + c);
        v.x /= r;
        v.y /= r;
        v.z /= r;
        v.w /= r;
        *reinterpret_cast<float4 *>(yr + c) = v;
      }
    } else {
      for (uint32_t c = lane; c < cols; c += 32) yr[c] = xr[c] / r;
    }
  }
}

// dx = (g - y * (sum(g*y)/D)) / rms(x), plus addend when given (the
// residual-stream gradient the executor adds next, folded in).  addend may
// alias dx: each element is read before it is written by the same thread.
__global__ void __launch_bounds__(256)
rmsnorm_backward_kernel(const float *__restrict__ g, const float *__restrict__ x,
                        const float *__restrict__ y, const float *addend, float *dx,
                        uint32_t rows, uint32_t cols, bool vec) {
  pdl_enter();
  ROW_LOOP {
    const size_t off = static_cast<size_t>(row) * cols;
    const float r = row_rms(x + off, cols, vec, lane);
    const float mean = row_dot(g + off, y + off, cols, vec, lane) / static_cast<float>(cols);
    if (vec) {
      for (uint32_t c = lane * 4; c < cols; c += 128) {
        const float4 gv = *reinterpret_cast<const float4 *>(g + off + c);
        const float4 yv = *reinterpret_cast<const float4 *>(y + off + c);
        float4 o;
        o.x = (gv.x - yv.x * mean) / r;
        o.y = (gv.y - yv.y * mean) / r;
        o.z = (gv.z - yv.z * mean) / r;
        o.w = (gv.w - yv.w * mean) / r;
        if (addend) {
          const float4 a = *reinterpret_cast<const float4 *>(addend + off + c);
          o = make_float4(a.x + o.x, a.y + o.y, a.z + o.z, a.w + o.w);
        }
        *reinterpret_cast<float4 *>(dx + off + c) = o;
      }
    } else {
      for (uint32_t c = lane; c < cols; c += 32) {
        const float o = (g[off + c] - y[off + c] * mean) / r;
        dx[off + c] = addend ? addend[off + c] + o : o;
      }
    }
  }
}

__global__ void __launch_bounds__(256)
xent_kernel(const float *__restrict__ z, const uint32_t *__restrict__ t,
            float *loss, uint32_t rows, uint32_t vocab, bool vec) {
  pdl_enter();
  ROW_LOOP {
    const uint32_t target = t[row];
    if (target >= vocab) {
      if (lane == 0) loss[row] = INFINITY;
      continue;
    }
    const float *zr = z + static_cast<size_t>(row) * vocab;
    float m, s;
    row_logsumexp(zr, vocab, vec, lane, m, s);
    if (lane == 0) loss[row] = m + logf(s) - zr[target];
  }
}

__global__ void __launch_bounds__(256)
xent_backward_kernel(const float *__restrict__ z, const uint32_t *__restrict__ t,
                     const float *__restrict__ scale, float *dz, uint32_t rows,
                     uint32_t vocab, bool vec) {
  pdl_enter();
  ROW_LOOP {
    const uint32_t target = t[row];
    const float *zr = z + static_cast<size_t>(row) * vocab;
    float *dr = dz + static_cast<size_t>(row) * vocab;
    if (target >= vocab) {
      for (uint32_t c = lane; c < vocab; c += 32) dr[c] = INFINITY;
      continue;
    }
    float m, s;
    row_logsumexp(zr, vocab, vec, lane, m, s);
    const bool scaled = scale != nullptr;
    const float k = scaled ? scale[row] : 1.0f;
    if (vec) {
      for (uint32_t c = lane * 4; c < vocab; c += 128) {
        float4 v = *reinterpret_cast<const float4 *>(zr + c);
        float p[4] = {expf(v.x - m) / s, expf(v.y - m) / s, expf(v.z - m) / s,
                      expf(v.w - m) / s};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (c + j == target) p[j] -= 1.0f;
          if (scaled) p[j] = k * p[j];
        }
        *reinterpret_cast<float4 *>(dr + c) = make_float4(p[0], p[1], p[2], p[3]);
      }
    } else {
      for (uint32_t c = lane; c < vocab; c += 32) {
        float p = expf(zr[c] - m) / s;
        if (c == target) p -= 1.0f;
        dr[c] = scaled ? k * p : p;
      }
    }
  }
}

// Register-resident cross-entropy (vocab <= 128 * NV, 128-bit rows): the
// warp loads the whole row of logits at once (NV float4 per lane in
// flight), then the row maximum, the sum of exp(z - max) and the loss
// max + log(sum) - z[target] (math.metal:884-911) from registers: one pass
// over memory instead of a latency-bound online pass.
template <int NV>
__device__ __forceinline__ void load_row_regs(const float *zr, uint32_t cols, uint32_t lane,
                                              float4 (&v)[NV], float &m, float &s) {
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const uint32_t c = (i * 32 + lane) * 4;
    v[i] = c < cols ? *reinterpret_cast<const float4 *>(zr + c)
                    : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
  }
  m = -INFINITY;
#pragma unroll
  for (int i = 0; i < NV; ++i) m = fmaxf(m, fmaxf(fmaxf(v[i].x, v[i].y), fmaxf(v[i].z, v[i].w)));
  m = warp_max(m);
  s = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const uint32_t c = (i * 32 + lane) * 4;
    if (c < cols) s += (expf(v[i].x - m) + expf(v[i].y - m)) + (expf(v[i].z - m) + expf(v[i].w - m));
  }
  s = warp_sum(s);
}

// z[target] from the lane holding it (register select, then a shuffle).
template <int NV>
__device__ __forceinline__ float target_logit(const float4 (&v)[NV], uint32_t target,
                                              uint32_t lane) {
  const uint32_t it = target >> 7, comp = target & 3u;
  float z = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (static_cast<uint32_t>(i) == it)
      z = comp == 0 ? v[i].x : comp == 1 ? v[i].y : comp == 2 ? v[i].z : v[i].w;
  }
  (void)lane;
  return __shfl_sync(0xffffffffu, z, (target >> 2) & 31u);
}

template <int NV>
__global__ void __launch_bounds__(256)
xent_regs_kernel(const float *__restrict__ z, const uint32_t *__restrict__ t, float *loss,
                 uint32_t rows, uint32_t vocab) {
  pdl_enter();
  ROW_LOOP {
    const uint32_t target = t[row];
    if (target >= vocab) {
      if (lane == 0) loss[row] = INFINITY;
      continue;
    }
    float4 v[NV];
    float m, s;
    load_row_regs<NV>(z + static_cast<size_t>(row) * vocab, vocab, lane, v, m, s);
    const float zt = target_logit<NV>(v, target, lane);
    if (lane == 0) loss[row] = m + logf(s) - zt;
  }
}

// dz = (softmax(z) - onehot(target)) (* row_scale): math.metal:912-953 (and
// the executor's hadamard by the root gradient) from the registers.
template <int NV>
__global__ void __launch_bounds__(256, 2)
xent_backward_regs_kernel(const float *__restrict__ z, const uint32_t *__restrict__ t,
                          const float *__restrict__ scale, float *dz, uint32_t rows,
                          uint32_t vocab) {
  pdl_enter();
  ROW_LOOP {
    const uint32_t target = t[row];
    float *dr = dz + static_cast<size_t>(row) * vocab;
    if (target >= vocab) {
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const uint32_t c = (i * 32 + lane) * 4;
        if (c < vocab)
          *reinterpret_cast<float4 *>(dr + c) = make_float4(INFINITY, INFINITY, INFINITY, INFINITY);
      }
      continue;
    }
    float4 v[NV];
    float m, s;
    load_row_regs<NV>(z + static_cast<size_t>(row) * vocab, vocab, lane, v, m, s);
    const bool scaled = scale != nullptr;
    const float k = scaled ? scale[row] : 1.0f;
    const float inv_s = 1.0f / s;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint32_t c = (i * 32 + lane) * 4;
      if (c >= vocab) continue;
      float p[4] = {expf(v[i].x - m) * inv_s, expf(v[i].y - m) * inv_s,
                    expf(v[i].z - m) * inv_s, expf(v[i].w - m) * inv_s};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (c + j == target) p[j] -= 1.0f;
        if (scaled) p[j] = k * p[j];
      }
      *reinterpret_cast<float4 *>(dr + c) = make_float4(p[0], p[1], p[2], p[3]);
    }
  }
}

// ---- register-resident rows (cols <= 128 * NV, 128-bit rows) ----------
// One warp per row keeps the whole row in registers (NV float4 per lane,
// lane l holding columns 4l + 128i): one pass over memory.  The backward
// and RMSNorm kernels keep the looping kernels' per-lane order of
// operations (bit-identical results); the softmax is the three-pass form.
// Register-resident softmax: the row's maximum, then the sum of
// exp(x - max), then exp(x - max) / sum - the reference kernel's three
// passes (math.metal:857-882) over registers, without the online
// rescaling's data-dependent branches (half of a causal score row is -inf).
template <int NV>
__global__ void __launch_bounds__(256)
softmax_regs_kernel(const float *__restrict__ x, const float *__restrict__ divisor,
                    const float *__restrict__ mask, uint32_t mask_rows, float *out,
                    uint32_t rows, uint32_t cols) {
  pdl_enter();
  ROW_LOOP {
    const float *xr = x + static_cast<size_t>(row) * cols;
    const float *mr = mask ? mask + static_cast<size_t>(row % mask_rows) * cols : nullptr;
    float4 v[NV];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint32_t c = (i * 32 + lane) * 4;
      if (c < cols) {
        v[i] = *reinterpret_cast<const float4 *>(xr + c);
        v[i].x = score(v[i].x, divisor, mr, c);
        v[i].y = score(v[i].y, divisor, mr, c + 1);
        v[i].z = score(v[i].z, divisor, mr, c + 2);
        v[i].w = score(v[i].w, divisor, mr, c + 3);
        m = fmaxf(m, fmaxf(fmaxf(v[i].x, v[i].y), fmaxf(v[i].z, v[i].w)));
      }
    }
    m = warp_max(m);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint32_t c = (i * 32 + lane) * 4;
      if (c < cols) {
        v[i] = make_float4(expf(v[i].x - m), expf(v[i].y - m), expf(v[i].z - m),
                           expf(v[i].w - m));
        s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
      }
    }
    s = warp_sum(s);
    float *yr = out + static_cast<size_t>(row) * cols;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint32_t c = (i * 32 + lane) * 4;
      if (c < cols)
        *reinterpret_cast<float4 *>(yr + c) =
            make_float4(v[i].x / s, v[i].y / s, v[i].z / s, v[i].w / s);
    }
  }
}

template <int NV>
__global__ void __launch_bounds__(256)
softmax_backward_regs_kernel(const float *__restrict__ g, const float *__restrict__ y,
                             const float *__restrict__ divisor, float *dx, uint32_t rows,
                             uint32_t cols) {
  pdl_enter();
  ROW_LOOP {
    const size_t off = static_cast<size_t>(row) * cols;
    float4 gv[NV], yv[NV];
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint32_t c = (i * 32 + lane) * 4;
      if (c < cols) {
        gv[i] = *reinterpret_cast<const float4 *>(g + off + c);
        yv[i] = *reinterpret_cast<const float4 *>(y + off + c);
        acc += gv[i].x * yv[i].x + gv[i].y * yv[i].y + gv[i].z * yv[i].z + gv[i].w * yv[i].w;
      }
    }
    const float dot = warp_sum(acc);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint32_t c = (i * 32 + lane) * 4;
      if (c < cols)
        *reinterpret_cast<float4 *>(dx + off + c) =
            make_float4(div_opt(yv[i].x * (gv[i].x - dot), divisor),
                        div_opt(yv[i].y * (gv[i].y - dot), divisor),
                        div_opt(yv[i].z * (gv[i].z - dot), divisor),
                        div_opt(yv[i].w * (gv[i].w - dot), divisor));
    }
  }
}

template <int NV>
__global__ void __launch_bounds__(256)
rmsnorm_regs_kernel(const float *__restrict__ x, float *out, float *rms_out, uint32_t rows,
                    uint32_t cols) {
  pdl_enter();
  ROW_LOOP {
    const float *xr = x + static_cast<size_t>(row) * cols;
    float4 v[NV];
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint32_t c = (i * 32 + lane) * 4;
      if (c < cols) {
        v[i] = *reinterpret_cast<const float4 *>(xr + c);
        acc += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
      }
    }
    const float r = sqrtf(warp_sum(acc) / static_cast<float>(cols) + 1e-6f);
    if (rms_out && lane == 0) rms_out[row] = r;
    float *yr = out + static_cast<size_t>(row) * cols;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint32_t c = (i * 32 + lane) * 4;
      if (c < cols)
        *reinterpret_cast<float4 *>(yr + c) =
            make_float4(v[i].x / r, v[i].y / r, v[i].z / r, v[i].w / r);
    }
  }
}

template <int NV>
__global__ void __launch_bounds__(256)
rmsnorm_backward_regs_kernel(const float *__restrict__ g, const float *__restrict__ x,
                             const float *__restrict__ y, const float *addend, float *dx,
                             uint32_t rows, uint32_t cols) {
  pdl_enter();
  ROW_LOOP {
    const size_t off = static_cast<size_t>(row) * cols;
    float4 gv[NV], yv[NV], av[NV];
    float ss = 0.0f, gy = 0.0f;
    // the addend is loaded with the row's other inputs, before the two
    // warp reductions, so its latency is not paid after them
    if (addend) {
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const uint32_t c = (i * 32 + lane) * 4;
        if (c < cols) av[i] = *reinterpret_cast<const float4 *>(addend + off + c);
      }
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint32_t c = (i * 32 + lane) * 4;
      if (c < cols) {
        const float4 xv = *reinterpret_cast<const float4 *>(x + off + c);
        ss += xv.x * xv.x + xv.y * xv.y + xv.z * xv.z + xv.w * xv.w;
        gv[i] = *reinterpret_cast<const float4 *>(g + off + c);
        yv[i] = *reinterpret_cast<const float4 *>(y + off + c);
        gy += gv[i].x * yv[i].x + gv[i].y * yv[i].y + gv[i].z * yv[i].z + gv[i].w * yv[i].w;
      }
    }
    const float r = sqrtf(warp_sum(ss) / static_cast<float>(cols) + 1e-6f);
    const float mean = warp_sum(gy) / static_cast<float>(cols);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint32_t c = (i * 32 + lane) * 4;
      if (c < cols) {
        float4 o = make_float4((gv[i].x - yv[i].x * mean) / r, (gv[i].y - yv[i].y * mean) / r,
                               (gv[i].z - yv[i].z * mean) / r, (gv[i].w - yv[i].w * mean) / r);
        if (addend) o = make_float4(av[i].x + o.x, av[i].y + o.y, av[i].z + o.z, av[i].w + o.w);
        *reinterpret_cast<float4 *>(dx + off + c) = o;
      }
    }
  }
}

// ---- rows of 64 * NP columns (attention scores: T = 192) ---------------
// Lane l holds columns 2l + 64i (a float2 each), so every lane does the same
// work and loads stay coalesced (256 bytes per warp instruction).  A
// divisor that is a power of two (sqrt of a power-of-four head size) is
// applied as a multiplication, which is exact; the final normalisation
// multiplies by one reciprocal of the row sum.
__device__ __forceinline__ bool pow2f(float d) {
  const uint32_t b = __float_as_uint(d);
  const uint32_t e = (b >> 23) & 0xffu;
  return (b & 0x7fffffu) == 0 && e != 0 && e != 0xffu;
}

template <int NP>
__global__ void __launch_bounds__(256)
softmax_pairs_kernel(const float *__restrict__ x, const float *__restrict__ divisor,
                     const float *__restrict__ mask, uint32_t mask_rows, float *out,
                     uint32_t rows, uint32_t cols) {
  pdl_enter();
  const float dv = divisor ? *divisor : 1.0f;
  const bool exact_scale = divisor && pow2f(dv);
  const float rdv = 1.0f / dv;
  ROW_LOOP {
    const float *xr = x + static_cast<size_t>(row) * cols;
    const float *mr = mask ? mask + static_cast<size_t>(row % mask_rows) * cols : nullptr;
    float2 v[NP];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      const uint32_t c = 2 * lane + 64 * i;
      v[i] = *reinterpret_cast<const float2 *>(xr + c);
      if (divisor) {
        if (exact_scale) v[i] = make_float2(v[i].x * rdv, v[i].y * rdv);
        else v[i] = make_float2(v[i].x / dv, v[i].y / dv);
      }
      if (mr) {
        const float2 k = *reinterpret_cast<const float2 *>(mr + c);
        v[i] = make_float2(v[i].x + k.x, v[i].y + k.y);
      }
      m = fmaxf(m, fmaxf(v[i].x, v[i].y));
    }
    m = warp_max(m);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      v[i] = make_float2(expf(v[i].x - m), expf(v[i].y - m));
      s += v[i].x + v[i].y;
    }
    const float inv = 1.0f / warp_sum(s);
    float *yr = out + static_cast<size_t>(row) * cols;
#pragma unroll
    for (int i = 0; i < NP; ++i)
      *reinterpret_cast<float2 *>(yr + 2 * lane + 64 * i) = make_float2(v[i].x * inv, v[i].y * inv);
  }
}

template <int NP>
__global__ void __launch_bounds__(256)
softmax_backward_pairs_kernel(const float *__restrict__ g, const float *__restrict__ y,
                              const float *__restrict__ divisor, float *dx, uint32_t rows,
                              uint32_t cols) {
  pdl_enter();
  const float dv = divisor ? *divisor : 1.0f;
  const bool exact_scale = divisor && pow2f(dv);
  const float rdv = 1.0f / dv;
  ROW_LOOP {
    const size_t off = static_cast<size_t>(row) * cols;
    float2 gv[NP], yv[NP];
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      const uint32_t c = 2 * lane + 64 * i;
      gv[i] = *reinterpret_cast<const float2 *>(g + off + c);
      yv[i] = *reinterpret_cast<const float2 *>(y + off + c);
      acc += gv[i].x * yv[i].x + gv[i].y * yv[i].y;
    }
    const float dot = warp_sum(acc);
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      float2 r = make_float2(yv[i].x * (gv[i].x - dot), yv[i].y * (gv[i].y - dot));
      if (divisor) {
        if (exact_scale) r = make_float2(r.x * rdv, r.y * rdv);
        else r = make_float2(r.x / dv, r.y / dv);
      }
      *reinterpret_cast<float2 *>(dx + off + 2 * lane + 64 * i) = r;
    }
  }
}

// float2 pairs per lane for rows of exactly 64 * NP columns (0: other rows)
int pairs_for(uint32_t cols, std::initializer_list<const void *> ptrs) {
  if (cols % 64 || cols > 512) return 0;
  for (const void *p : ptrs)
    if (p && (reinterpret_cast<uintptr_t>(p) & 7u)) return 0;
  return static_cast<int>(cols / 64);
}

#define TL_PAIRS_DISPATCH(NPVAR, LAUNCH) \
  switch (NPVAR) {                       \
    case 1: LAUNCH(1); break;            \
    case 2: LAUNCH(2); break;            \
    case 3: LAUNCH(3); break;            \
    case 4: LAUNCH(4); break;            \
    case 5: LAUNCH(5); break;            \
    case 6: LAUNCH(6); break;            \
    case 7: LAUNCH(7); break;            \
    default: LAUNCH(8); break;           \
  }

// Float4s per lane that hold a row of `cols` (0: too long, use the loops).
int regs_for(uint32_t cols) {
  const uint32_t nv = (cols + 127) / 128;
  if (nv <= 1) return 1;
  if (nv <= 2) return 2;
  if (nv <= 3) return 3;
  if (nv <= 4) return 4;
  if (nv <= 6) return 6;
  if (nv <= 8) return 8;
  return 0;
}

#define TL_ROWS_DISPATCH(NVVAR, LAUNCH) \
  switch (NVVAR) {                      \
    case 1: LAUNCH(1); break;           \
    case 2: LAUNCH(2); break;           \
    case 3: LAUNCH(3); break;           \
    case 4: LAUNCH(4); break;           \
    case 6: LAUNCH(6); break;           \
    default: LAUNCH(8); break;          \
  }

// float4 registers per lane of the register-resident cross-entropy (0: the
// online kernels for longer rows)
int xent_regs_for(uint32_t vocab) {
  if (vocab <= 512) return 4;
  if (vocab <= 1024) return 8;
  if (vocab <= 2048) return 16;
  return 0;
}

unsigned row_grid(uint32_t rows) {
  return grid_for(rows, kWarpsPerBlock, 16);
}

bool row_vec(uint32_t cols, std::initializer_list<const void *> ptrs) {
  if (cols % 4) return false;
  for (const void *p : ptrs)
    if (p && !aligned16(p)) return false;
  return true;
}

}  // namespace
}  // namespace tl

using namespace tl;

extern "C" {

int tl_softmax_rows(const float *x, float *out, uint32_t rows, uint32_t cols,
                    void *stream) {
  if (cols == 0) return fail(TL_ERR_INVALID, "softmax requires a non-empty final dimension");
  if (rows == 0) return TL_OK;
  if (!x || !out) return fail(TL_ERR_INVALID, "tl_softmax_rows: null pointer");
  const int np = pairs_for(cols, {x, out});
  const int nv = row_vec(cols, {x, out}) ? regs_for(cols) : 0;
  if (np) {
#define L(NP) launch_pdl(softmax_pairs_kernel<NP>, row_grid(rows), 256, 0, as_stream(stream),  \
    x, nullptr, nullptr, 0, out, rows, cols)
    TL_PAIRS_DISPATCH(np, L)
#undef L
  } else if (nv) {
#define L(NV) launch_pdl(softmax_regs_kernel<NV>, row_grid(rows), 256, 0, as_stream(stream),  \
    x, nullptr, nullptr, 0, out, rows, cols)
    TL_ROWS_DISPATCH(nv, L)
#undef L
  } else {
    launch_pdl(softmax_kernel, row_grid(rows), 256, 0, as_stream(stream), x, out, rows, cols,
                                                                  row_vec(cols, {x, out}));
  }
  return launch_status("tl_softmax_rows");
}

int tl_softmax_scaled_masked_rows(const float *x, const float *divisor, const float *mask,
                                  uint32_t mask_rows, float *out, uint32_t rows,
                                  uint32_t cols, void *stream) {
  if (cols == 0) return fail(TL_ERR_INVALID, "softmax requires a non-empty final dimension");
  if (rows == 0) return TL_OK;
  if (!x || !out) return fail(TL_ERR_INVALID, "tl_softmax_scaled_masked_rows: null pointer");
  if (mask && mask_rows == 0)
    return fail(TL_ERR_INVALID, "tl_softmax_scaled_masked_rows: mask without rows");
  const int np = pairs_for(cols, {x, out, mask});
  const int nv = row_vec(cols, {x, out, mask}) ? regs_for(cols) : 0;
  if (np) {
#define L(NP) launch_pdl(softmax_pairs_kernel<NP>, row_grid(rows), 256, 0, as_stream(stream),  \
    x, divisor, mask, mask_rows, out, rows, cols)
    TL_PAIRS_DISPATCH(np, L)
#undef L
  } else if (nv) {
#define L(NV) launch_pdl(softmax_regs_kernel<NV>, row_grid(rows), 256, 0, as_stream(stream),  \
    x, divisor, mask, mask_rows, out, rows, cols)
    TL_ROWS_DISPATCH(nv, L)
#undef L
  } else {
    launch_pdl(softmax_scaled_masked_kernel, row_grid(rows), 256, 0, as_stream(stream), 
        x, divisor, mask, mask_rows, out, rows, cols, row_vec(cols, {x, out, mask}));
  }
  return launch_status("tl_softmax_scaled_masked_rows");
}

int tl_softmax_backward_rows(const float *grad, const float *y, const float *divisor,
                             float *dx, uint32_t rows, uint32_t cols, void *stream) {
  if (rows == 0 || cols == 0) return TL_OK;
  if (!grad || !y || !dx) return fail(TL_ERR_INVALID, "tl_softmax_backward_rows: null pointer");
  const int np = pairs_for(cols, {grad, y, dx});
  const int nv = row_vec(cols, {grad, y, dx}) ? regs_for(cols) : 0;
  if (np) {
#define L(NP) launch_pdl(softmax_backward_pairs_kernel<NP>, row_grid(rows), 256, 0, as_stream(stream),  \
    grad, y, divisor, dx, rows, cols)
    TL_PAIRS_DISPATCH(np, L)
#undef L
  } else if (nv) {
#define L(NV) launch_pdl(softmax_backward_regs_kernel<NV>, row_grid(rows), 256, 0, as_stream(stream),  \
    grad, y, divisor, dx, rows, cols)
    TL_ROWS_DISPATCH(nv, L)
#undef L
  } else {
    launch_pdl(softmax_backward_kernel, row_grid(rows), 256, 0, as_stream(stream), 
        grad, y, divisor, dx, rows, cols, row_vec(cols, {grad, y, dx}));
  }
  return launch_status("tl_softmax_backward_rows");
}

int tl_rms_rows(const float *x, float *rms, uint32_t rows, uint32_t cols,
                void *stream) {
  if (rows == 0) return TL_OK;
  if (cols == 0) return fail(TL_ERR_INVALID, "tl_rms_rows: empty rows");
  if (!x || !rms) return fail(TL_ERR_INVALID, "tl_rms_rows: null pointer");
  launch_pdl(rms_kernel, row_grid(rows), 256, 0, as_stream(stream), x, rms, rows, cols,
                                                            row_vec(cols, {x}));
  return launch_status("tl_rms_rows");
}

int tl_rmsnorm_rows(const float *x, float *out, float *rms_out, uint32_t rows,
                    uint32_t cols, void *stream) {
  if (rows == 0) return TL_OK;
  if (cols == 0) return fail(TL_ERR_INVALID, "tl_rmsnorm_rows: empty rows");
  if (!x || !out) return fail(TL_ERR_INVALID, "tl_rmsnorm_rows: null pointer");
  const int nv = row_vec(cols, {x, out}) ? regs_for(cols) : 0;
  if (nv) {
#define L(NV) launch_pdl(rmsnorm_regs_kernel<NV>, row_grid(rows), 256, 0, as_stream(stream),  \
    x, out, rms_out, rows, cols)
    TL_ROWS_DISPATCH(nv, L)
#undef L
  } else {
    launch_pdl(rmsnorm_kernel, row_grid(rows), 256, 0, as_stream(stream), 
        x, out, rms_out, rows, cols, row_vec(cols, {x, out}));
  }
  return launch_status("tl_rmsnorm_rows");
}

int tl_rmsnorm_backward_rows(const float *grad, const float *x, const float *y,
                             const float *addend, float *dx, uint32_t rows, uint32_t cols,
                             void *stream) {
  if (rows == 0) return TL_OK;
  if (cols == 0) return fail(TL_ERR_INVALID, "tl_rmsnorm_backward_rows: empty rows");
  if (!grad || !x || !y || !dx)
    return fail(TL_ERR_INVALID, "tl_rmsnorm_backward_rows: null pointer");
  const int nv = row_vec(cols, {grad, x, y, dx, addend}) ? regs_for(cols) : 0;
  if (nv) {
#define L(NV) launch_pdl(rmsnorm_backward_regs_kernel<NV>, row_grid(rows), 256, 0, as_stream(stream),  \
    grad, x, y, addend, dx, rows, cols)
    TL_ROWS_DISPATCH(nv, L)
#undef L
  } else {
    launch_pdl(rmsnorm_backward_kernel, row_grid(rows), 256, 0, as_stream(stream), 
        grad, x, y, addend, dx, rows, cols, row_vec(cols, {grad, x, y, dx, addend}));
  }
  return launch_status("tl_rmsnorm_backward_rows");
}

int tl_xent_rows(const float *logits, const uint32_t *targets, float *loss,
                 uint32_t rows, uint32_t vocab, void *stream) {
  if (vocab == 0)
    return fail(TL_ERR_INVALID, "cross_entropy requires logits with a non-empty final dimension");
  if (rows == 0) return TL_OK;
  if (!logits || !targets || !loss) return fail(TL_ERR_INVALID, "tl_xent_rows: null pointer");
  const int nv = row_vec(vocab, {logits}) ? xent_regs_for(vocab) : 0;
  if (nv == 4)
    launch_pdl(xent_regs_kernel<4>, row_grid(rows), 256, 0, as_stream(stream), logits, targets,
               loss, rows, vocab);
  else if (nv == 8)
    launch_pdl(xent_regs_kernel<8>, row_grid(rows), 256, 0, as_stream(stream), logits, targets,
               loss, rows, vocab);
  else if (nv == 16)
    launch_pdl(xent_regs_kernel<16>, row_grid(rows), 256, 0, as_stream(stream), logits, targets,
               loss, rows, vocab);
  else
    launch_pdl(xent_kernel, row_grid(rows), 256, 0, as_stream(stream),
               logits, targets, loss, rows, vocab, row_vec(vocab, {logits}));
  return launch_status("tl_xent_rows");
}

int tl_xent_backward_rows(const float *logits, const uint32_t *targets,
                          const float *row_scale, float *dlogits, uint32_t rows,
                          uint32_t vocab, void *stream) {
  if (vocab == 0)
    return fail(TL_ERR_INVALID,
                "cross_entropy_derivative requires logits with a non-empty final dimension");
  if (rows == 0) return TL_OK;
  if (!logits || !targets || !dlogits)
    return fail(TL_ERR_INVALID, "tl_xent_backward_rows: null pointer");
  const int nv = row_vec(vocab, {logits, dlogits}) ? xent_regs_for(vocab) : 0;
  if (nv == 4)
    launch_pdl(xent_backward_regs_kernel<4>, row_grid(rows), 256, 0, as_stream(stream), logits,
               targets, row_scale, dlogits, rows, vocab);
  else if (nv == 8)
    launch_pdl(xent_backward_regs_kernel<8>, row_grid(rows), 256, 0, as_stream(stream), logits,
               targets, row_scale, dlogits, rows, vocab);
  else if (nv == 16)
    launch_pdl(xent_backward_regs_kernel<16>, row_grid(rows), 256, 0, as_stream(stream), logits,
               targets, row_scale, dlogits, rows, vocab);
  else
    launch_pdl(xent_backward_kernel, row_grid(rows), 256, 0, as_stream(stream),
               logits, targets, row_scale, dlogits, rows, vocab, row_vec(vocab, {logits, dlogits}));
  return launch_status("tl_xent_backward_rows");
}

}  // extern "C"

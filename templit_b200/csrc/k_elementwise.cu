// Elementwise kernels: broadcast binary ops, scalar ops, unary ops, fused
// GELU backward, copy and fill.  All are HBM-bound; every kernel moves 128-bit
// vectors where the innermost dimension allows and runs a grid-stride loop
// over a grid of 8 CTAs per SM.
//
// Broadcast semantics follow the reference Metal runtime: operand strides
// are aligned to the output shape from the right and a size-1 dimension
// broadcasts (src/my_metal/runtime.cpp:18-39, math.metal:401-510).  Unlike
// the Metal kernel, which decodes every element through all dimensions,
// the host coalesces adjacent dimensions first, so the common shapes
// (same-shape, bias row, per-row scalar) decode through one or two dims.
#include "tl_common.cuh"

#include <cmath>

namespace tl {
namespace {

struct NdParams {
  int rank;
  uint32_t ostride[TL_MAX_RANK];  // contiguous output strides (elements)
  uint32_t sa[TL_MAX_RANK];       // operand a strides (0 = broadcast)
  uint32_t sb[TL_MAX_RANK];       // operand b strides
};

template <int OP>
__device__ __forceinline__ float apply_binary(float x, float y) {
  if constexpr (OP == TL_ADD) return x + y;
  if constexpr (OP == TL_SUB) return x - y;
  if constexpr (OP == TL_MUL) return x * y;
  return x / y;
}

template <int OP, int VEC>
__global__ void __launch_bounds__(256)
binary_kernel(const float *__restrict__ a, const float *__restrict__ b,
              float *out, NdParams p, uint32_t n_vec) {
  pdl_enter();
  const int r = p.rank;
  for (uint32_t v = blockIdx.x * blockDim.x + threadIdx.x; v < n_vec;
       v += gridDim.x * blockDim.x) {
    uint32_t rem = v * VEC, oa = 0, ob = 0;
#pragma unroll 1
    for (int d = 0; d < r - 1; ++d) {
      const uint32_t c = rem / p.ostride[d];
      rem -= c * p.ostride[d];
      oa += c * p.sa[d];
      ob += c * p.sb[d];
    }
    oa += rem * p.sa[r - 1];
    ob += rem * p.sb[r - 1];
    if constexpr (VEC == 4) {
      float4 x, y;
      if (p.sa[r - 1]) x = *reinterpret_cast<const float4 *>(a + oa);
      else x = make_float4(a[oa], a[oa], a[oa], a[oa]);
      if (p.sb[r - 1]) y = *reinterpret_cast<const float4 *>(b + ob);
      else y = make_float4(b[ob], b[ob], b[ob], b[ob]);
      float4 z;
      z.x = apply_binary<OP>(x.x, y.x);
      z.y = apply_binary<OP>(x.y, y.y);
      z.z = apply_binary<OP>(x.z, y.z);
      z.w = apply_binary<OP>(x.w, y.w);
      *reinterpret_cast<float4 *>(out + v * 4) = z;
    } else {
      out[v] = apply_binary<OP>(a[oa], b[ob]);
    }
  }
}

template <int OP>
__device__ __forceinline__ float apply_scalar(float x, float s) {
  if constexpr (OP == TL_SCALAR_ADD) return x + s;
  if constexpr (OP == TL_SCALAR_DIV) return x / s;
  return powf(x, s);
}

template <int OP>
__device__ __forceinline__ float apply_unary(float x) {
  if constexpr (OP == TL_SIGMOID) return 1.0f / (1.0f + expf(-x));
  if constexpr (OP == TL_SQRT) return sqrtf(x);
  if constexpr (OP == TL_EXP) return expf(x);
  if constexpr (OP == TL_GELU) return gelu_f(x);
  return gelu_deriv_f(x);
}

// Generic vector map: out[i] = F(x[i]) (and y[i] when binary).
template <typename F>
__global__ void __launch_bounds__(256)
map1_kernel(const float *__restrict__ x, float *out, size_t n, F f) {
  pdl_enter();
  const size_t n4 = n / 4;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t t0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (size_t i = t0; i < n4; i += stride) {
    float4 v = reinterpret_cast<const float4 *>(x)[i];
    v.x = f(v.x);
    v.y = f(v.y);
    v.z = f(v.z);
    v.w = f(v.w);
    reinterpret_cast<float4 *>(out)[i] = v;
  }
  for (size_t i = n4 * 4 + t0; i < n; i += stride) out[i] = f(x[i]);
}

template <typename F>
__global__ void __launch_bounds__(256)
map1_scalar_kernel(const float *__restrict__ x, float *out, size_t n, F f) {
  pdl_enter();
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < n; i += stride)
    out[i] = f(x[i]);
}

template <typename F>
__global__ void __launch_bounds__(256)
map2_kernel(const float *__restrict__ x, const float *__restrict__ y,
            float *out, size_t n, F f) {
  pdl_enter();
  const size_t n4 = n / 4;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t t0 = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (size_t i = t0; i < n4; i += stride) {
    float4 u = reinterpret_cast<const float4 *>(x)[i];
    const float4 w = reinterpret_cast<const float4 *>(y)[i];
    u.x = f(u.x, w.x);
    u.y = f(u.y, w.y);
    u.z = f(u.z, w.z);
    u.w = f(u.w, w.w);
    reinterpret_cast<float4 *>(out)[i] = u;
  }
  for (size_t i = n4 * 4 + t0; i < n; i += stride) out[i] = f(x[i], y[i]);
}

template <typename F>
__global__ void __launch_bounds__(256)
map2_scalar_kernel(const float *__restrict__ x, const float *__restrict__ y,
                   float *out, size_t n, F f) {
  pdl_enter();
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < n; i += stride)
    out[i] = f(x[i], y[i]);
}

template <typename F>
int launch_map1(const float *x, float *out, size_t n, cudaStream_t s, F f,
                const char *what) {
  if (n == 0) return TL_OK;
  if (aligned16(x) && aligned16(out))
    launch_pdl(map1_kernel<F>, grid_for((n + 3) / 4, 256), 256, 0, s, x, out, n, f);
  else
    launch_pdl(map1_scalar_kernel<F>, grid_for(n, 256), 256, 0, s, x, out, n, f);
  return launch_status(what);
}

template <typename F>
int launch_map2(const float *x, const float *y, float *out, size_t n,
                cudaStream_t s, F f, const char *what) {
  if (n == 0) return TL_OK;
  if (aligned16(x) && aligned16(y) && aligned16(out))
    launch_pdl(map2_kernel<F>, grid_for((n + 3) / 4, 256), 256, 0, s, x, y, out, n, f);
  else
    launch_pdl(map2_scalar_kernel<F>, grid_for(n, 256), 256, 0, s, x, y, out, n, f);
  return launch_status(what);
}

template <int OP> struct ScalarFn {
  float s;
  __device__ float operator()(float x) const { return apply_scalar<OP>(x, s); }
};
template <int OP> struct UnaryFn {
  __device__ float operator()(float x) const { return apply_unary<OP>(x); }
};
struct GeluBackwardFn {
  __device__ float operator()(float x, float g) const { return gelu_deriv_f(x) * g; }
};

__global__ void fill_u32_kernel(uint32_t *dst, uint32_t v, size_t n) {
  pdl_enter();
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < n; i += stride)
    dst[i] = v;
}

// Computes the broadcast strides of an operand against the output shape and
// coalesces dimensions.  Returns TL_OK or an error status.
int plan_broadcast(const uint32_t *a_shape, int a_rank, const uint32_t *b_shape,
                   int b_rank, const uint32_t *out_shape, int out_rank,
                   NdParams &p, size_t &numel) {
  if (out_rank < 1 || out_rank > TL_MAX_RANK || a_rank < 0 || b_rank < 0 ||
      a_rank > out_rank || b_rank > out_rank)
    return fail(TL_ERR_INVALID, "binary op: operand rank exceeds output rank");
  uint32_t shape[TL_MAX_RANK], sa[TL_MAX_RANK], sb[TL_MAX_RANK];
  numel = 1;
  for (int i = 0; i < out_rank; ++i) {
    shape[i] = out_shape[i];
    numel *= out_shape[i];
  }
  auto strides_of = [&](const uint32_t *s, int r, uint32_t *out) -> bool {
    uint32_t dense[TL_MAX_RANK];
    uint64_t st = 1;
    for (int i = r; i-- > 0;) {
      dense[i] = static_cast<uint32_t>(st);
      st *= s[i];
    }
    const int off = out_rank - r;
    for (int i = 0; i < out_rank; ++i) out[i] = 0;
    for (int i = 0; i < r; ++i) {
      if (s[i] == shape[off + i]) out[off + i] = dense[i];
      else if (s[i] == 1) out[off + i] = 0;
      else return false;
    }
    return true;
  };
  if (!strides_of(a_shape, a_rank, sa) || !strides_of(b_shape, b_rank, sb))
    return fail(TL_ERR_INVALID, "invalid broadcast");
  // Drop unit dims, then merge neighbours that stay linear in every operand.
  int r = 0;
  uint32_t cs[TL_MAX_RANK], ca[TL_MAX_RANK], cb[TL_MAX_RANK];
  for (int i = 0; i < out_rank; ++i) {
    if (shape[i] == 1) continue;
    if (r > 0 && ca[r - 1] == sa[i] * shape[i] && cb[r - 1] == sb[i] * shape[i]) {
      cs[r - 1] *= shape[i];
      ca[r - 1] = sa[i];
      cb[r - 1] = sb[i];
      continue;
    }
    cs[r] = shape[i];
    ca[r] = sa[i];
    cb[r] = sb[i];
    ++r;
  }
  if (r == 0) {
    cs[0] = 1;
    ca[0] = 0;
    cb[0] = 0;
    r = 1;
  }
  p.rank = r;
  uint32_t st = 1;
  for (int i = r; i-- > 0;) {
    p.ostride[i] = st;
    st *= cs[i];
    p.sa[i] = ca[i];
    p.sb[i] = cb[i];
  }
  return TL_OK;
}

template <int OP>
void launch_binary(const float *a, const float *b, float *out, const NdParams &p,
                   uint32_t inner, size_t n, cudaStream_t s) {
  const int r = p.rank;
  const bool vec = inner % 4 == 0 && p.sa[r - 1] <= 1 && p.sb[r - 1] <= 1 &&
                   aligned16(out) && (p.sa[r - 1] == 0 || aligned16(a)) &&
                   (p.sb[r - 1] == 0 || aligned16(b));
  if (vec) {
    const uint32_t nv = static_cast<uint32_t>(n / 4);
    launch_pdl(binary_kernel<OP, 4>, grid_for(nv, 256), 256, 0, s, a, b, out, p, nv);
  } else {
    launch_pdl(binary_kernel<OP, 1>, grid_for(n, 256), 256, 0, s, 
        a, b, out, p, static_cast<uint32_t>(n));
  }
}

}  // namespace
}  // namespace tl

using namespace tl;

extern "C" {

int tl_binary(int op, const float *a, const uint32_t *a_shape, int a_rank,
              const float *b, const uint32_t *b_shape, int b_rank, float *out,
              const uint32_t *out_shape, int out_rank, void *stream) {
  if (op < TL_ADD || op > TL_DIV) return fail(TL_ERR_INVALID, "tl_binary: unknown op");
  NdParams p{};
  size_t n = 0;
  int rc = plan_broadcast(a_shape, a_rank, b_shape, b_rank, out_shape, out_rank, p, n);
  if (rc) return rc;
  if (n == 0) return TL_OK;
  if (!a || !b || !out) return fail(TL_ERR_INVALID, "tl_binary: null pointer");
  if (n > 0xffffffffull) return fail(TL_ERR_RANGE, "tl_binary: more than 2^32-1 elements");
  // the innermost coalesced extent decides whether 4-wide vectors stay in one row
  uint32_t inner = p.rank == 1 ? static_cast<uint32_t>(n) : p.ostride[p.rank - 2];
  cudaStream_t s = as_stream(stream);
  switch (op) {
    case TL_ADD: launch_binary<TL_ADD>(a, b, out, p, inner, n, s); break;
    case TL_SUB: launch_binary<TL_SUB>(a, b, out, p, inner, n, s); break;
    case TL_MUL: launch_binary<TL_MUL>(a, b, out, p, inner, n, s); break;
    default: launch_binary<TL_DIV>(a, b, out, p, inner, n, s); break;
  }
  return launch_status("tl_binary");
}

int tl_scalar(int op, const float *x, float sc, float *out, size_t count,
              void *stream) {
  if (count && (!x || !out)) return fail(TL_ERR_INVALID, "tl_scalar: null pointer");
  cudaStream_t s = as_stream(stream);
  switch (op) {
    case TL_SCALAR_ADD: return launch_map1(x, out, count, s, ScalarFn<TL_SCALAR_ADD>{sc}, "tl_scalar add");
    case TL_SCALAR_DIV: return launch_map1(x, out, count, s, ScalarFn<TL_SCALAR_DIV>{sc}, "tl_scalar div");
    case TL_SCALAR_POW: return launch_map1(x, out, count, s, ScalarFn<TL_SCALAR_POW>{sc}, "tl_scalar pow");
    default: return fail(TL_ERR_INVALID, "tl_scalar: unknown op");
  }
}

int tl_unary(int op, const float *x, float *out, size_t count, void *stream) {
  if (count && (!x || !out)) return fail(TL_ERR_INVALID, "tl_unary: null pointer");
  cudaStream_t s = as_stream(stream);
  switch (op) {
    case TL_SIGMOID: return launch_map1(x, out, count, s, UnaryFn<TL_SIGMOID>{}, "tl_unary sigmoid");
    case TL_SQRT: return launch_map1(x, out, count, s, UnaryFn<TL_SQRT>{}, "tl_unary sqrt");
    case TL_EXP: return launch_map1(x, out, count, s, UnaryFn<TL_EXP>{}, "tl_unary exp");
    case TL_GELU: return launch_map1(x, out, count, s, UnaryFn<TL_GELU>{}, "tl_unary gelu");
    case TL_GELU_DERIVATIVE:
      return launch_map1(x, out, count, s, UnaryFn<TL_GELU_DERIVATIVE>{}, "tl_unary gelu'");
    default: return fail(TL_ERR_INVALID, "tl_unary: unknown op");
  }
}

int tl_gelu_backward(const float *x, const float *grad, float *out, size_t count,
                     void *stream) {
  if (count && (!x || !grad || !out))
    return fail(TL_ERR_INVALID, "tl_gelu_backward: null pointer");
  return launch_map2(x, grad, out, count, as_stream(stream), GeluBackwardFn{},
                     "tl_gelu_backward");
}

int tl_copy(const float *x, float *out, size_t count, void *stream) {
  if (count == 0 || x == out) return TL_OK;
  if (!x || !out) return fail(TL_ERR_INVALID, "tl_copy: null pointer");
  return check_cuda(cudaMemcpyAsync(out, x, count * sizeof(float),
                                    cudaMemcpyDeviceToDevice, as_stream(stream)),
                    "tl_copy");
}

int tl_fill_u32(void *dst, uint32_t pattern, size_t count, void *stream) {
  if (count == 0) return TL_OK;
  if (!dst) return fail(TL_ERR_INVALID, "tl_fill_u32: null pointer");
  cudaStream_t s = as_stream(stream);
  if (pattern == 0)
    return check_cuda(cudaMemsetAsync(dst, 0, count * 4, s), "tl_fill_u32 memset");
  launch_pdl(fill_u32_kernel, grid_for(count, 256), 256, 0, s, static_cast<uint32_t *>(dst),
                                                       pattern, count);
  return launch_status("tl_fill_u32");
}

}  // extern "C"

// Shared helpers for the TempLit B200 kernel library: status reporting,
// launch geometry and small device utilities.
#pragma once

#include "templit_cuda.h"

#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>
#include <string>
#include <utility>

namespace tl {

// 148 SMs on B200 (2 dies x 74); grids of memory-bound kernels are sized in
// multiples of this so every SM gets the same number of resident CTAs.
constexpr int kNumSMs = 148;

// Records `msg` as the thread's last error and returns `code`.
int fail(int code, const std::string &msg);
// Converts a CUDA error into a status (TL_OK when e == cudaSuccess).
int check_cuda(cudaError_t e, const char *what);
// Status after a launch: cudaGetLastError.
int launch_status(const char *what);

inline cudaStream_t as_stream(void *s) { return static_cast<cudaStream_t>(s); }

// Programmatic dependent launch: every kernel of the library is launched
// with programmatic stream serialisation and waits for the previous
// kernel's completion and memory (griddepcontrol.wait) before it touches
// global memory, so its launch is staged while the previous kernel still
// runs.  TL_PDL=0 in the environment turns it off.
bool pdl_enabled();

__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args &&...args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // failures are reported by launch_status (cudaGetLastError)
  (void)cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// launch_pdl for a kernel whose CTAs run in clusters of `cluster` along x
// (grid.x a multiple of it).
template <typename... KArgs, typename... Args>
inline void launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t s, unsigned cluster, Args &&...args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  (void)cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Grid for a grid-stride loop over `work` items with `threads` per CTA,
// capped at `per_sm` CTAs per SM.
inline unsigned grid_for(size_t work, int threads, int per_sm = 8) {
  size_t blocks = (work + threads - 1) / threads;
  size_t cap = static_cast<size_t>(kNumSMs) * per_sm;
  if (blocks > cap) blocks = cap;
  if (blocks == 0) blocks = 1;
  return static_cast<unsigned>(blocks);
}

__host__ __device__ inline bool aligned16(const void *p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Device address of this device's status word (tl_device_status); kernels
// that can meet bad data take it as an argument and raise flags there
// instead of faulting.
uint32_t *device_status_ptr();

// Arrival ticket of a "last CTA folds the partials" reduction: atomicInc
// (wraps to 0 after `limit`) with acquire-release semantics at GPU scope.
// Called by one thread after a __syncthreads() that follows the CTA's
// partial stores, the release covers those stores (release is cumulative);
// in the CTA that draws the last ticket, a __syncthreads() after the call
// orders every thread's reads of the partials after the acquire.  No
// per-thread memory fence is needed on either side.
__device__ __forceinline__ unsigned ticket_acq_rel(unsigned *p, unsigned limit) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.inc.u32 %0, [%1], %2;"
               : "=r"(old)
               : "l"(p), "r"(limit)
               : "memory");
  return old;
}

__device__ __forceinline__ void raise_flag(uint32_t *status, uint32_t flag) {
  atomicOr(status, flag);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Online (max, sum-of-exp) pair merge used by softmax / cross-entropy rows.
__device__ __forceinline__ void online_merge(float &m, float &s, float m2,
                                             float s2) {
  float mn = fmaxf(m, m2);
  if (mn == -INFINITY) {  // both empty: keep (-inf, 0)
    m = mn;
    return;
  }
  s = s * expf(m - mn) + s2 * expf(m2 - mn);
  m = mn;
}

// 2^x and 1/x by the SFU (PTX ex2.approx / rcp.approx, subnormals flushed).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// GELU, tanh approximation, with the constants of the reference kernels
// (include/my_metal/math.metal:821-855): 0.5 x (1 + tanh u), u = a (x +
// b x^3), a = sqrt(2 / 3.14159265), b = 0.044715.  Evaluated through the
// identity 0.5 (1 + tanh u) = 1 / (1 + e^{-2u}) = s: GELU = x s and
// GELU' = s + 0.5 x (1 - tanh^2 u) u' = s (1 + 2 a x e s (1 + 3 b x^2)),
// with e = e^{-2u} = 2^{-2u log2(e)} (so 1 - s = e s exactly, without the
// cancellation of 1 - s).  The exponent is clamped to +-126: beyond it s is
// 0 or 1 to float precision.  About 1e-6 relative to the exact formula
// (the SFU's 2^x and 1/x are within a few ulp; the exponent's rounding
// grows with |u|).
constexpr float kGeluA = 0.7978845612587234f;       // sqrt(2 / 3.14159265)
constexpr float kGeluB = 0.044715f;
constexpr float kGeluNeg2ALog2e = -2.302208199459653f;  // -2 a log2(e)

__device__ __forceinline__ float gelu_exp_term(float x, float x2) {
  const float z = kGeluNeg2ALog2e * fmaf(kGeluB * x2, x, x);
  return ex2_approx(fminf(fmaxf(z, -126.0f), 126.0f));
}

__device__ __forceinline__ float gelu_f(float x) {
  const float e = gelu_exp_term(x, x * x);
  return x * rcp_approx(1.0f + e);
}

__device__ __forceinline__ float gelu_deriv_f(float x) {
  const float x2 = x * x;
  const float e = gelu_exp_term(x, x2);
  const float s = rcp_approx(1.0f + e);
  const float q = fmaf(3.0f * kGeluB, x2, 1.0f);
  return fmaf(s, (2.0f * kGeluA) * x * (e * s) * q, s);
}

}  // namespace tl

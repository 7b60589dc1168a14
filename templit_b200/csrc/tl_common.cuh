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

// GELU, tanh approximation, with the constants of the reference kernels
// (include/my_metal/math.metal:821-855).
__device__ __forceinline__ float gelu_f(float x) {
  const float k = sqrtf(2.0f / 3.14159265f);
  return 0.5f * x * (1.0f + tanhf(k * (x + 0.044715f * x * x * x)));
}

__device__ __forceinline__ float gelu_deriv_f(float x) {
  const float a = 0.7978845608f;
  const float b = 0.044715f;
  const float x2 = x * x;
  const float t = tanhf(a * (x + b * x2 * x));
  return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * a * (1.0f + 3.0f * b * x2);
}

}  // namespace tl

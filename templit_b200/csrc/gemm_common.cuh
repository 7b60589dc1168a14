// Shared GEMM argument block, batch decoding and epilogue for the tensor-core
// (tcgen05) and CUDA-core GEMM kernels behind tl_gemm.
#pragma once

#include "tl_common.cuh"

namespace tl {

struct GemmArgs {
  const float *a;
  const float *b;
  float *c;
  const float *bias;
  float *gelu_out;
  const float *addend;  // C's layout; C itself when accumulating (beta = 1)
  const float *gelu_grad_x;  // C's layout: C = GELU'(x) * product
  uint32_t c_heads, c_head_rows;  // head-split store (tl_gemm_desc), 0: none
  int split_tf32;  // TL_GEMM_3XTF32: big and small tf32 halves of each operand
  uint32_t m, n, k;
  uint64_t lda, ldb, ldc;  // row strides of the stored matrices (elements)
  int trans_a, trans_b;
  float beta;
  uint32_t batch_rank;
  uint32_t batch_shape[TL_GEMM_MAX_BATCH_RANK];
  uint64_t sa[TL_GEMM_MAX_BATCH_RANK];
  uint64_t sb[TL_GEMM_MAX_BATCH_RANK];
  uint64_t sc[TL_GEMM_MAX_BATCH_RANK];
  uint64_t batch_count;
  uint64_t batch_base;  // first batch index of this launch
  // grouped products (tl_gemm_desc.group_mode): groups == 1 when none
  int group_mode;
  uint32_t groups;
  const float *ag[TL_GEMM_MAX_GROUPS];
  const float *bg[TL_GEMM_MAX_GROUPS];
  float *cg[TL_GEMM_MAX_GROUPS];
  const float *biasg[TL_GEMM_MAX_GROUPS];
};

// Element offsets of batch `z` (relative to batch_base) in A, B and C.
__device__ __forceinline__ void batch_offsets(const GemmArgs &g, uint64_t z,
                                              uint64_t &oa, uint64_t &ob,
                                              uint64_t &oc) {
  uint64_t b = g.batch_base + z;
  oa = ob = oc = 0;
  for (int d = static_cast<int>(g.batch_rank) - 1; d >= 0; --d) {
    const uint64_t c = b % g.batch_shape[d];
    b /= g.batch_shape[d];
    oa += c * g.sa[d];
    ob += c * g.sb[d];
    oc += c * g.sc[d];
  }
}

// Final value of C[idx] (idx relative to the batch's C base, column n):
// v = A*B (+ bias[n]) then addend + v (or GELU'(x) * v for a folded GELU
// backward, in the order of the reference's hadamard) - the reference adds the bias after
// the product (EXPR_LINEAR: mult then add, include/passes/execute.h:241-252)
// and gradient accumulation adds the new term to the old (context.h:74-89).
// `bias`: g.bias, or a group's bias of a grouped product.
__device__ __forceinline__ void epilogue_store(const GemmArgs &g, float *Cb, const float *bias,
                                               uint64_t oc, size_t idx, uint32_t n, float v) {
  if (bias) v = v + bias[n];
  if (g.addend) v = g.addend[oc + idx] + v;
  if (g.gelu_grad_x) v = gelu_deriv_f(g.gelu_grad_x[oc + idx]) * v;
  Cb[idx] = v;
  if (g.gelu_out) g.gelu_out[oc + idx] = gelu_f(v);
}
__device__ __forceinline__ void epilogue_store(const GemmArgs &g, float *Cb,
                                               uint64_t oc, size_t idx,
                                               uint32_t n, float v) {
  epilogue_store(g, Cb, g.bias, oc, idx, n, v);
}

int launch_sgemm(const GemmArgs &g, cudaStream_t s);
// Returns TL_ERR_UNSUPPORTED when the operands do not meet the tensor-core
// path's alignment rules; the caller then falls back to launch_sgemm.
// `workspace` holds split-K slices when the plan splits K (see
// tc_gemm_workspace); with less room the product runs unsplit.
int launch_tc_gemm(const GemmArgs &g, void *workspace, size_t workspace_bytes, cudaStream_t s);
size_t tc_gemm_workspace(const GemmArgs &g);
// The tensor-core path's operand rules (TMA: 16-byte aligned bases, row and
// batch strides; at most three walked batch dims per operand).
bool tc_gemm_supported(const GemmArgs &g);

}  // namespace tl

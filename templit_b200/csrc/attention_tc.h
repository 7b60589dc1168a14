// Fused tensor-core attention kernels (k_attention_tc.cu) behind
// tl_attention_fwd / tl_attention_bwd.
#pragma once

#include "tl_common.cuh"

namespace tl {

constexpr uint32_t kMaxFusedKeys = 192;  // longest sequence of the fused kernels

// Shape and element strides of the head-strided q, k, v, o (and gradients).
struct FusedAttnShape {
  uint32_t B, T, H, D;
  uint64_t sb, sh, ld;
};

// True when the fused kernels take this shape: D == 64, T <= 192, T % 4 == 0,
// strides and pointers 16-byte aligned.
bool fused_attention_supported(const FusedAttnShape &sh, const void *const *ptrs, int n);

int launch_attention_fwd_tc(const float *q, const float *k, const float *v, const float *divisor,
                            const float *mask, float *p, float *o, const FusedAttnShape &sh,
                            cudaStream_t s);

// dq, dk, dv from the forward's p; ds ([B, H, T, T]) receives dS.
int launch_attention_bwd_tc(const float *q, const float *k, const float *v, const float *p,
                            const float *divisor, const float *d_o, float *dq, float *dk,
                            float *dv, float *ds, const FusedAttnShape &sh, cudaStream_t s);

}  // namespace tl

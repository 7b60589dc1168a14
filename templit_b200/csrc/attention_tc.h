// Fused tensor-core attention kernels (k_attention_tc.cu) behind
// tl_attention_fwd / tl_attention_bwd and the runtime's fused attention ops.
#pragma once

#include "tl_common.cuh"

namespace tl {

constexpr uint32_t kMaxFusedKeys = 192;  // longest sequence of the fused kernels
constexpr uint32_t kFusedHeadDim = 64;   // head width of the fused kernels

// One [T, D] block per (batch, head) of a strided tensor: element (b, h, t, d)
// at p + b * sb + h * sh + t * ld + d, or, when `trans`, the block is stored
// transposed ([D, T]: element (t, d) at t + d * ld).
struct HeadView {
  const float *p;
  uint64_t sb, sh, ld;
  bool trans;
};

struct AttnDims {
  uint32_t B, T, H;
};

// True when the fused kernels take these operands: T <= 192 with T % 4 == 0,
// 16-byte aligned pointers and strides, and only K stored transposed
// (`k_may_trans` marks which views may be).
bool fused_attention_fits(const AttnDims &d, const HeadView *views, const bool *may_trans,
                          int n);

// P = softmax(Q K^T / divisor + mask) ([B, H, T, T], dense), O = P V.
// mask_flag (optional device word): first set to whether the mask is the
// causal one, which the kernel then applies arithmetically.
int launch_attention_fwd_tc(const AttnDims &d, const HeadView &q, const HeadView &k,
                            const HeadView &v, const float *divisor, const float *mask, float *p,
                            const HeadView &o, uint32_t *mask_flag, cudaStream_t s,
                            bool mask_checked = false);
// dS = P * (dP - rowsum(dP * P)) / divisor with dP = dO V^T (written to ds,
// dense [B, H, T, T]); dQ = dS K.
int launch_attention_bwd_q_tc(const AttnDims &d, const HeadView &d_o, const HeadView &v,
                              const HeadView &k, const float *p, const float *divisor, float *ds,
                              const HeadView &dq, cudaStream_t s);
// dK = dS^T Q (when dk.p) and dV = P^T dO (when dv.p), one launch.
int launch_attention_bwd_kv_tc(const AttnDims &d, const float *ds, const HeadView &q,
                               const HeadView &dk, const float *p, const HeadView &d_o,
                               const HeadView &dv, cudaStream_t s);

// ---- flash attention (k_flash_attn.cu): any T, D == 64, no T x T tensor
// True when the flash kernels take these operands (16-byte aligned pointers
// and strides; only K may be stored transposed).
bool flash_attention_fits(const AttnDims &d, const HeadView *views, int n);
// O = softmax(Q K^T / divisor + mask) V and the row log-sum-exp lse
// ([B, H, T], natural log).  mask_flag (optional device word): nonzero when
// the mask is the causal one, applied by position without reading it.
int launch_flash_fwd(const AttnDims &d, const HeadView &q, const HeadView &k, const HeadView &v,
                     const float *divisor, const float *mask, const uint32_t *mask_flag,
                     const HeadView &o, float *lse, cudaStream_t s);
// dQ, dK, dV from Q, K, V, O, dO and lse; delta ([B, H, T]) is scratch.
int launch_flash_bwd(const AttnDims &d, const HeadView &q, const HeadView &k, const HeadView &v,
                     const HeadView &o, const HeadView &d_o, const float *divisor,
                     const float *mask, const uint32_t *mask_flag, const float *lse,
                     float *delta, const HeadView &dq, const HeadView &dk, const HeadView &dv,
                     cudaStream_t s);
// P = exp(Q K^T / divisor + mask - lse), dense [B, H, T, T].
int launch_flash_probs(const AttnDims &d, const HeadView &q, const HeadView &k,
                       const float *divisor, const float *mask, const uint32_t *mask_flag,
                       const float *lse, float *p, cudaStream_t s);
// *flag = 1 when mask ([T, T]) is the causal mask, else 0.
int launch_mask_check(const float *mask, uint32_t T, uint32_t *flag, cudaStream_t s);

}  // namespace tl

// Multi-head attention core of nn::MultiHeadAttention (include/nn/
// multi_head.h:45-52) as library calls: the score and value products run on
// the tensor-core GEMM with every head addressed in place (batch dims
// (B, H) with their own strides, rows with a row stride, so [B, T, H, D]
// projections need no head split), the softmax with its divide and mask in
// one row pass, and the backward's softmax derivative (SFTMX_DERIVATIVE,
// include/passes/execute.h:291-308) with the divide folded in.  Scores, their
// gradient and the softmax gradient live in the caller's workspace.
#include "attention_tc.h"
#include "tl_common.cuh"

#include <cstring>

namespace tl {
namespace {

// One batched product over (B, H) with per-operand strides.
struct Operand {
  const float *p;
  uint64_t sb, sh, ld;  // batch strides and row stride (elements)
};

int product(const Operand &a, bool ta, const Operand &b, bool tb, float *c, uint64_t csb,
            uint64_t csh, uint64_t ldc, uint32_t m, uint32_t n, uint32_t k, uint32_t B,
            uint32_t H, int precision, cudaStream_t s) {
  tl_gemm_desc d;
  std::memset(&d, 0, sizeof(d));
  d.a = a.p;
  d.b = b.p;
  d.c = c;
  d.m = m;
  d.n = n;
  d.k = k;
  d.trans_a = ta;
  d.trans_b = tb;
  d.precision = precision;
  d.batch_rank = 2;
  d.batch_shape[0] = B;
  d.batch_shape[1] = H;
  d.a_batch_stride[0] = a.sb;
  d.a_batch_stride[1] = a.sh;
  d.b_batch_stride[0] = b.sb;
  d.b_batch_stride[1] = b.sh;
  d.c_batch_stride[0] = csb;
  d.c_batch_stride[1] = csh;
  d.lda = a.ld;
  d.ldb = b.ld;
  d.ldc = ldc;
  return tl_gemm(&d, s);
}

size_t scores_bytes(uint32_t B, uint32_t T, uint32_t H) {
  return static_cast<size_t>(B) * H * T * T * sizeof(float);
}

// Strides of one [.., T, D] head block of q, k, v, o and their gradients.
struct HeadLayout {
  uint64_t sb, sh, ld;
};

int check_args(const void *const *ptrs, int n, uint32_t B, uint32_t T, uint32_t H, uint32_t D,
               int layout, int precision, size_t ws_bytes, size_t need, const char *what,
               HeadLayout &hl) {
  for (int i = 0; i < n; ++i)
    if (!ptrs[i]) return fail(TL_ERR_INVALID, std::string(what) + ": null pointer");
  if (!B || !T || !H || !D) return fail(TL_ERR_INVALID, std::string(what) + ": empty shape");
  if (precision != TL_GEMM_TF32 && precision != TL_GEMM_FP32)
    return fail(TL_ERR_INVALID, std::string(what) + ": unknown precision");
  if (static_cast<uint64_t>(B) * H * T > UINT32_MAX)
    return fail(TL_ERR_INVALID, std::string(what) + ": too many score rows");
  if (ws_bytes < need) return fail(TL_ERR_INVALID, std::string(what) + ": workspace too small");
  const uint64_t td = static_cast<uint64_t>(T) * D;
  if (layout == TL_ATTN_BTHD)
    hl = {td * H, D, static_cast<uint64_t>(H) * D};
  else if (layout == TL_ATTN_BHTD)
    hl = {td * H, td, D};
  else
    return fail(TL_ERR_INVALID, std::string(what) + ": unknown layout");
  return TL_OK;
}

}  // namespace
}  // namespace tl

using namespace tl;

extern "C" {

size_t tl_attention_workspace_size(uint32_t B, uint32_t T, uint32_t H, uint32_t D) {
  (void)D;
  return 2 * scores_bytes(B, T, H);
}

int tl_attention_fwd(const float *q, const float *k, const float *v, const float *divisor,
                     const float *mask, float *p, float *o, uint32_t B, uint32_t T, uint32_t H,
                     uint32_t D, int32_t layout, int32_t precision, void *workspace,
                     size_t workspace_bytes, void *stream) {
  const void *ptrs[] = {q, k, v, divisor, p, o, workspace};
  HeadLayout hl;
  int rc = check_args(ptrs, 7, B, T, H, D, layout, precision, workspace_bytes,
                      scores_bytes(B, T, H), "tl_attention_fwd", hl);
  if (rc) return rc;
  cudaStream_t s = as_stream(stream);
  const uint64_t hs = hl.sb, hh = hl.sh, ld = hl.ld;
  if (precision == TL_GEMM_TF32 && D == kFusedHeadDim && aligned16(p) &&
      (!mask || aligned16(mask))) {
    const AttnDims dims{B, T, H};
    auto view = [&](const float *x) { return HeadView{x, hs, hh, ld, false}; };
    const HeadView views[] = {view(q), view(k), view(v), view(o)};
    const bool may_trans[] = {false, false, false, false};
    if (fused_attention_fits(dims, views, may_trans, 4)) {
      uint32_t *flag = aligned16(workspace) ? static_cast<uint32_t *>(workspace) : nullptr;
      rc = launch_attention_fwd_tc(dims, views[0], views[1], views[2], divisor, mask, p, views[3],
                                   flag, s);
      if (rc != TL_ERR_UNSUPPORTED) return rc;
    }
  }
  const uint64_t ts = static_cast<uint64_t>(T) * T;
  float *scores = static_cast<float *>(workspace);
  // S = Q K^T per (b, h)
  rc = product({q, hs, hh, ld}, false, {k, hs, hh, ld}, true, scores, H * ts, ts, T, T, T, D, B,
               H, precision, s);
  if (rc) return rc;
  // P = softmax(S / divisor + mask)
  rc = tl_softmax_scaled_masked_rows(scores, divisor, mask, mask ? T : 0, p,
                                     static_cast<uint32_t>(static_cast<uint64_t>(B) * H * T), T,
                                     stream);
  if (rc) return rc;
  // O = P V, written into [B, T, H, D]
  return product({p, H * ts, ts, T}, false, {v, hs, hh, ld}, false, o, hs, hh, ld, T, D, T, B, H,
                 precision, s);
}

int tl_attention_bwd(const float *q, const float *k, const float *v, const float *p,
                     const float *divisor, const float *d_o, float *dq, float *dk, float *dv,
                     uint32_t B, uint32_t T, uint32_t H, uint32_t D, int32_t layout,
                     int32_t precision, void *workspace, size_t workspace_bytes, void *stream) {
  const void *ptrs[] = {q, k, v, p, divisor, d_o, dq, dk, dv, workspace};
  HeadLayout hl;
  int rc = check_args(ptrs, 10, B, T, H, D, layout, precision, workspace_bytes,
                      2 * scores_bytes(B, T, H), "tl_attention_bwd", hl);
  if (rc) return rc;
  cudaStream_t s = as_stream(stream);
  const uint64_t hs = hl.sb, hh = hl.sh, ld = hl.ld;
  if (precision == TL_GEMM_TF32 && D == kFusedHeadDim && aligned16(p) && aligned16(workspace)) {
    const AttnDims dims{B, T, H};
    auto view = [&](const float *x) { return HeadView{x, hs, hh, ld, false}; };
    const HeadView views[] = {view(q), view(k), view(v), view(d_o), view(dq), view(dk), view(dv)};
    const bool may_trans[7] = {};
    if (fused_attention_fits(dims, views, may_trans, 7)) {
      float *ds = static_cast<float *>(workspace);
      rc = launch_attention_bwd_q_tc(dims, views[3], views[2], views[1], p, divisor, ds, views[4],
                                     s);
      if (rc == TL_OK)
        rc = launch_attention_bwd_kv_tc(dims, ds, views[0], views[5], p, views[3], views[6], s);
      if (rc != TL_ERR_UNSUPPORTED) return rc;
    }
  }
  const uint64_t ts = static_cast<uint64_t>(T) * T;
  float *dp = static_cast<float *>(workspace);
  float *ds = dp + static_cast<size_t>(B) * H * ts;
  // dP = dO V^T
  rc = product({d_o, hs, hh, ld}, false, {v, hs, hh, ld}, true, dp, H * ts, ts, T, T, T, D, B, H,
               precision, s);
  if (rc) return rc;
  // dS = P (dP - rowsum(dP P)) / divisor
  rc = tl_softmax_backward_rows(dp, p, divisor, ds,
                                static_cast<uint32_t>(static_cast<uint64_t>(B) * H * T), T,
                                stream);
  if (rc) return rc;
  // dQ = dS K;  dK = dS^T Q;  dV = P^T dO   (all into [B, T, H, D])
  rc = product({ds, H * ts, ts, T}, false, {k, hs, hh, ld}, false, dq, hs, hh, ld, T, D, T, B, H,
               precision, s);
  if (rc) return rc;
  rc = product({ds, H * ts, ts, T}, true, {q, hs, hh, ld}, false, dk, hs, hh, ld, T, D, T, B, H,
               precision, s);
  if (rc) return rc;
  return product({p, H * ts, ts, T}, true, {d_o, hs, hh, ld}, false, dv, hs, hh, ld, T, D, T, B, H,
                 precision, s);
}

namespace {

tl::HeadView hv(const tl_attn_view &v) {
  return tl::HeadView{v.p, v.batch_stride, v.head_stride, v.row_stride, v.transposed != 0};
}

bool fused_fits(const tl_attn_desc &d) {
  if (d.D != tl::kFusedHeadDim) return false;
  const tl::AttnDims dims{d.B, d.T, d.H};
  switch (d.pass) {
    case TL_ATTN_FORWARD: {
      if (!d.divisor || !d.p || !d.q.p || !d.k.p || !d.v.p || !d.o.p || !tl::aligned16(d.p) ||
          (d.mask && !tl::aligned16(d.mask)))
        return false;
      const tl::HeadView v[] = {hv(d.q), hv(d.k), hv(d.v), hv(d.o)};
      const bool t[] = {false, true, false, false};
      return tl::fused_attention_fits(dims, v, t, 4);
    }
    case TL_ATTN_BACKWARD_Q: {
      if (!d.divisor || !d.p || !d.ds || !d.d_o.p || !d.v.p || !d.k.p || !d.dq.p ||
          !tl::aligned16(d.p) || !tl::aligned16(d.ds))
        return false;
      const tl::HeadView v[] = {hv(d.d_o), hv(d.v), hv(d.k), hv(d.dq)};
      const bool t[] = {false, false, true, false};
      return tl::fused_attention_fits(dims, v, t, 4);
    }
    case TL_ATTN_PRODUCT_TN: {
      if (!d.ds || !d.q.p || !d.dk.p || !tl::aligned16(d.ds)) return false;
      const tl::HeadView v[] = {hv(d.q), hv(d.dk)};
      const bool t[] = {false, false};
      return tl::fused_attention_fits(dims, v, t, 2);
    }
    default:
      return false;
  }
}

}  // namespace

int tl_attention_fused_supported(const tl_attn_desc *d) { return d && fused_fits(*d) ? 1 : 0; }

int tl_attention_fused(const tl_attn_desc *d, void *stream) {
  if (!d) return fail(TL_ERR_INVALID, "tl_attention_fused: null descriptor");
  if (!fused_fits(*d)) return fail(TL_ERR_UNSUPPORTED, "tl_attention_fused: shape not supported");
  const tl::AttnDims dims{d->B, d->T, d->H};
  cudaStream_t s = as_stream(stream);
  switch (d->pass) {
    case TL_ATTN_FORWARD: {
      // a flag the caller has checked already, else the workspace's word
      uint32_t *flag = d->mask_flag ? const_cast<uint32_t *>(d->mask_flag)
                       : d->workspace && d->workspace_bytes >= 16 && tl::aligned16(d->workspace)
                           ? static_cast<uint32_t *>(d->workspace)
                           : nullptr;
      return tl::launch_attention_fwd_tc(dims, hv(d->q), hv(d->k), hv(d->v), d->divisor, d->mask,
                                         d->p, hv(d->o), flag, s, d->mask_flag != nullptr);
    }
    case TL_ATTN_BACKWARD_Q:
      return tl::launch_attention_bwd_q_tc(dims, hv(d->d_o), hv(d->v), hv(d->k), d->p,
                                           d->divisor, d->ds, hv(d->dq), s);
    default: {
      const tl::HeadView none{nullptr, 0, 0, 0, false};
      return tl::launch_attention_bwd_kv_tc(dims, d->ds, hv(d->q), hv(d->dk), nullptr, none,
                                            none, s);
    }
  }
}

}  // extern "C"

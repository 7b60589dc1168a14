// The recorded program of a runtime window: one Op per runtime call (or
// per Storage data movement inside the window), executed in order on the
// backend stream at submit().  Internal to the runtime.
#pragma once

#include "internal.h"

#include <array>
#include <cstdint>
#include <string>
#include <vector>

namespace cuda::internal {

constexpr int kMaxRank = TL_MAX_RANK;

// A dense tensor argument: device address, allocation id and shape.
struct TRef {
  void *p = nullptr;
  uint64_t id = 0;
  uint8_t rank = 0;
  uint32_t shape[kMaxRank] = {};

  uint64_t numel() const {
    if (rank == 0) return 0;
    uint64_t n = 1;
    for (int i = 0; i < rank; ++i) n *= shape[i];
    return n;
  }
  uint32_t last() const { return rank ? shape[rank - 1] : 0; }
  float *f() const { return static_cast<float *>(p); }
  uint32_t *u() const { return static_cast<uint32_t *>(p); }
  bool same_shape(const TRef &o) const {
    if (rank != o.rank) return false;
    for (int i = 0; i < rank; ++i)
      if (shape[i] != o.shape[i]) return false;
    return true;
  }
};

enum class Kind : uint8_t {
  // one per runtime call
  Binary,      // code = tl_binary_op; t0 a, t1 b, t2 out
  Scalar,      // code = tl_scalar_op; t0 x, t1 out, f0 scalar
  Unary,       // code = tl_unary_op; t0 x, t1 out
  Copy,        // t0 src, t1 dst (same element count)
  Reduce,      // code = tl_reduce_op; t0 x, t1 out
  Argmax,      // t0 x, t1 out index
  Transpose,   // t0 x, t1 out, i0 dim_a, i1 dim_b
  Softmax,     // t0 x, t1 out (+ t2 divisor [1], t3 mask [r, cols] added per row r % rows)
  Rms,         // t0 x, t1 rms
  RmsNorm,     // t0 x, t1 out
  Xent,        // t0 logits, t1 targets, t2 loss
  XentBwd,     // t0 logits, t1 targets, t2 dlogits, t3 row scale (optional)
  Gather,      // t0 weights, t1 ids, t2 out
  Scatter,     // t0 values, t1 ids, t2 base (optional), t3 dst
  SqNorm,      // t0 gradient, t1 sqnorm
  Clip,        // t0 gradient, t1 sqnorm, t2 out, f0 max_norm
  AdamW,       // t0 param, t1 grad, t2 out, t3 m1, t4 m2, t5 b1, t6 b2, t7 decay, t8 lr; f0 eps, u0 step
  Gemm,        // gemm descriptor; t0 a, t1 b, t2 c (+ t3 bias, t4 gelu out, t5 addend,
               //   t6 GELU-backward input)
  // Storage data movement inside the window
  HostWrite,   // t0 dst (rank 1 byte view), u64 offset, host payload
  Fill,        // t0 dst, u0 pattern, n elements
  DevCopy,     // t0 dst, t1 src, n bytes
  Release,     // t0: allocation id (and address) released here, n bytes (no launch)
  // produced by the optimiser
  GeluBwd,     // t0 x, t1 grad, t2 out
  SoftmaxBwd,  // t0 grad, t1 y, t2 out (+ t3 divisor [1])
  RmsNormBwd,  // t0 grad, t1 x, t2 y, t3 out (+ t4 addend)
  MultiAdamW,  // slots in `multi`; t0 sqnorm (optional); f0 max_norm; f1 eps; t5..t8 scalars
  AllReduce,   // NCCL sum of the gradients in `multi`
  // fused attention (tl_attention_fused with `attn`), code = tl_attn_pass:
  //   forward       t0 q, t1 k, t2 v, t3 divisor, t4 mask (optional), t5 p, t6 o
  //   backward Q    t0 dO, t1 v, t2 k, t3 p, t4 divisor, t5 ds, t6 dq
  //   product TN    t0 ds (or p), t1 q (or dO), t2 dk (or dv)
  Attention,
  // flash attention (tl_flash_attention_*, `flash` holds the descriptor):
  //   FlashFwd    t0 q, t1 k, t2 v, t3 divisor, t4 mask (optional), t5 P, t6 o:
  //               writes o and P's log-sum-exp (a runtime buffer), not P;
  //               P becomes a virtual tensor (FlashRecord) until something
  //               other than FlashBwd reads it
  //   FlashBwd    t0 q, t1 k, t2 v, t3 o, t4 dO, t5 divisor, t6 P (virtual),
  //               t7 dk, t8 dv; group_refs: [0] dq, [1] mask (optional)
  //   FlashProbs  t0 q, t1 k, t2 divisor, t3 mask (optional), t4 P: writes
  //               P from the log-sum-exp (a virtual P is read by another op)
  FlashFwd,
  FlashBwd,
  FlashProbs,
};

const char *kind_name(Kind k);

struct MultiSlot {
  TRef param, out, grad, m1, m2;
  uint32_t step;
};

struct Op {
  Kind kind;
  int32_t code = 0;
  std::array<TRef, 9> t{};
  float f0 = 0.0f, f1 = 0.0f;
  int32_t i0 = 0, i1 = 0;
  uint32_t u0 = 0;
  uint64_t n = 0;          // element / byte counts for data movement
  size_t workspace = 0;    // device scratch bytes this op needs
  tl_gemm_desc gemm{};
  tl_attn_desc attn{};             // Attention
  tl_flash_desc flash{};           // FlashFwd, FlashBwd, FlashProbs
  std::vector<uint8_t> host;       // HostWrite payload
  std::vector<MultiSlot> multi;    // MultiAdamW / AllReduce
  // grouped GEMM operands beyond group 0 (gemm.group_mode): N groups
  // (B, C, bias) per group, K groups (A, B) per group, from group 1 on
  std::vector<TRef> group_refs;
  bool dead = false;               // folded away by the optimiser
  uint32_t src = UINT32_MAX;       // index in the recorded program (optimiser cache)
};

}  // namespace cuda::internal

// Program optimiser: pattern rewrites over a recorded window.
//
// The typed executor (include/passes/execute.h, JTPuffer/TempLit) emits one
// runtime call per expression node, so fusable work reaches the runtime as
// short op sequences.  Because the runtime records a whole window before it
// launches anything, it can see those sequences and replace them with one
// kernel, provided every value another op (or the host, after wait()) can
// still observe comes out identical.  An intermediate is only skipped when
// its storage is released inside the window (an executor-local temporary:
// the transposed operand and product of a mult derivative, the reduced
// tensors of the softmax / RMSNorm derivative rules) and no op reads it in
// between.  Buffers are identified by allocation id, never by address, so
// memory reused after a release is never confused with the value released.
#include "optimize.h"

#include <algorithm>
#include <string>
#include <unordered_map>
#include <unordered_set>

namespace cuda::internal {

Access access(const Op &op) {
  Access a;
  const auto &t = op.t;
  switch (op.kind) {
    case Kind::Binary: a.read(t[0]); a.read(t[1]); a.write(t[2]); break;
    case Kind::Reduce:  // + grouped reductions' (input, output) pairs
      a.read(t[0]); a.write(t[1]);
      for (size_t k = 0; k + 1 < op.group_refs.size(); k += 2) {
        a.read(op.group_refs[k]);
        a.write(op.group_refs[k + 1]);
      }
      break;
    case Kind::Scalar: case Kind::Unary: case Kind::Copy: case Kind::Argmax:
    case Kind::Transpose: case Kind::Rms: case Kind::RmsNorm:
      a.read(t[0]); a.write(t[1]); break;
    case Kind::Softmax: a.read(t[0]); a.read(t[2]); a.read(t[3]); a.write(t[1]); break;
    case Kind::Xent: a.read(t[0]); a.read(t[1]); a.write(t[2]); break;
    case Kind::XentBwd: a.read(t[0]); a.read(t[1]); a.read(t[3]); a.write(t[2]); break;
    case Kind::Gather: a.read(t[0]); a.read(t[1]); a.write(t[2]); break;
    case Kind::Scatter: a.read(t[0]); a.read(t[1]); a.read(t[2]); a.write(t[3]); break;
    case Kind::SqNorm: a.read(t[0]); a.read(t[1]); a.write(t[1]); break;
    case Kind::Clip: a.read(t[0]); a.read(t[1]); a.write(t[2]); break;
    case Kind::AdamW:
      for (int i : {0, 1, 3, 4, 5, 6, 7, 8}) a.read(t[i]);
      a.write(t[2]); a.write(t[3]); a.write(t[4]); break;
    case Kind::Gemm:
      a.read(t[0]); a.read(t[1]); a.read(t[3]); a.read(t[5]); a.read(t[6]);
      if (op.gemm.beta != 0.0f) a.read(t[2]);
      a.write(t[2]); a.write(t[4]);
      if (op.gemm.group_mode == TL_GEMM_GROUP_N) {
        for (size_t i = 0; i + 2 < op.group_refs.size(); i += 3) {
          a.read(op.group_refs[i]);
          a.write(op.group_refs[i + 1]);
          a.read(op.group_refs[i + 2]);
        }
      } else if (op.gemm.group_mode == TL_GEMM_GROUP_K) {
        for (const TRef &r : op.group_refs) a.read(r);
      }
      break;
    case Kind::HostWrite: case Kind::Fill: a.write(t[0]); break;
    case Kind::DevCopy: a.read(t[1]); a.write(t[0]); break;
    case Kind::GeluBwd: a.read(t[0]); a.read(t[1]); a.write(t[2]); break;
    case Kind::SoftmaxBwd: a.read(t[0]); a.read(t[1]); a.read(t[3]); a.write(t[2]); break;
    case Kind::RmsNormBwd:
      a.read(t[0]); a.read(t[1]); a.read(t[2]); a.read(t[4]); a.write(t[3]); break;
    case Kind::Attention:
      if (op.code == TL_ATTN_PRODUCT_TN) {
        a.read(t[0]); a.read(t[1]); a.write(t[2]);
      } else {
        for (int i = 0; i < 5; ++i) a.read(t[i]);
        a.write(t[5]); a.write(t[6]);
      }
      break;
    case Kind::FlashFwd:  // P (t5) is defined here, though not stored
      for (int i = 0; i < 5; ++i) a.read(t[i]);
      a.write(t[5]); a.write(t[6]); break;
    case Kind::FlashBwd:
      for (int i = 0; i < 7; ++i) a.read(t[i]);
      if (op.group_refs.size() > 1) a.read(op.group_refs[1]);
      a.write(t[7]); a.write(t[8]);
      if (!op.group_refs.empty()) a.write(op.group_refs[0]);
      break;
    case Kind::FlashProbs:
      for (int i = 0; i < 4; ++i) a.read(t[i]);
      a.write(t[4]); break;
    default: break;  // Release, MultiAdamW, AllReduce: handled by their passes
  }
  return a;
}

bool full_write(const Op &op) {
  switch (op.kind) {
    case Kind::HostWrite: return op.n == 0 && op.host.size() >= op.t[0].numel();
    case Kind::Fill: return op.n * 4 >= op.t[0].numel();
    case Kind::DevCopy: return op.n >= op.t[0].numel();
    case Kind::SqNorm: return false;  // accumulates
    default: return true;
  }
}

namespace {

constexpr size_t kNone = static_cast<size_t>(-1);
constexpr uint32_t kFusedHeadDimHost = 64;  // head width of tl_attention_fused
constexpr uint32_t kFusedMaxKeysHost = 192;  // longest sequence of tl_attention_fused

// Window liveness of the program being optimised (null: none known).
thread_local const Liveness *g_live = nullptr;

bool reads(const Access &a, uint64_t id) {
  for (int i = 0; i < a.nr; ++i)
    if (a.r[i] == id) return true;
  return false;
}
bool writes(const Access &a, uint64_t id) {
  for (int i = 0; i < a.nw; ++i)
    if (a.w[i] == id) return true;
  return false;
}

// Next live op after i (skipping dead ops and releases), or kNone.
size_t next_op(const std::vector<Op> &p, size_t i) {
  for (size_t j = i + 1; j < p.size(); ++j)
    if (!p[j].dead && p[j].kind != Kind::Release) return j;
  return kNone;
}

// True when the value in allocation `id` is never read after op `after`
// (exclusive) before the allocation is released inside the program, except
// by the ops listed in `allowed`.  A write that fully replaces the value
// also ends its life.
bool dead_after(const std::vector<Op> &p, size_t after, uint64_t id,
                std::initializer_list<size_t> allowed = {}) {
  for (size_t j = after + 1; j < p.size(); ++j) {
    const Op &op = p[j];
    if (op.dead) continue;
    if (op.kind == Kind::Release) {
      if (op.t[0].id == id) return true;
      continue;
    }
    if (op.kind == Kind::MultiAdamW || op.kind == Kind::AllReduce) {
      for (const auto &s : op.multi)
        if (s.grad.id == id || s.param.id == id || s.m1.id == id || s.m2.id == id) return false;
      continue;
    }
    bool ok = false;
    for (size_t k : allowed)
      if (k == j) ok = true;
    const Access a = access(op);
    if (reads(a, id) && !ok) return false;
    if (writes(a, id) && !reads(a, id) && full_write(op)) return true;
  }
  // alive at the end of the program: observable unless window-local
  return g_live && g_live->window_local(id);
}

bool is_last_two(const Op &tr) {
  const int r = tr.t[0].rank;
  return r >= 2 && tr.i0 == r - 2 && tr.i1 == r - 1;
}

bool same(const TRef &a, const TRef &b) { return a.p && a.id == b.id; }

// ------------------------------------------------------------------- GEMM
// transpose(X -> T); mult(T, G -> P); sum_to_shape(P -> D) with T, P released:
// the weight gradient of EXPR_MULT_RHS_DERIVATIVE (execute.h:210-232) as
// one TN product D = X^T G with K = every batch row.  X and G must be dense
// batched operands of the same batch shape.
uint64_t fuse_weight_gradient(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t i = 0; i < p.size(); ++i) {
    Op &tr = p[i];
    if (tr.dead || tr.kind != Kind::Transpose || !is_last_two(tr)) continue;
    const size_t j = next_op(p, i);
    if (j == kNone) continue;
    Op &mm = p[j];
    if (mm.kind != Kind::Gemm || !same(mm.t[0], tr.t[1]) || mm.gemm.trans_a || mm.gemm.trans_b ||
        mm.gemm.bias || mm.gemm.gelu_out || mm.gemm.beta != 0.0f || mm.gemm.batch_rank == 0)
      continue;
    const size_t k = next_op(p, j);
    if (k == kNone) continue;
    Op &rd = p[k];
    if (rd.kind != Kind::Reduce || rd.code != TL_REDUCE_SUM || !same(rd.t[0], mm.t[2])) continue;
    const tl_gemm_desc &g = mm.gemm;
    // output must be exactly one [M, N] matrix (all batch dims summed)
    if (rd.t[1].numel() != uint64_t(g.m) * g.n || rd.t[1].last() != g.n) continue;
    // dense, unbroadcast batch operands
    uint64_t batch = 1;
    bool dense = true;
    for (int d = static_cast<int>(g.batch_rank) - 1; d >= 0; --d) {
      const uint64_t want_a = uint64_t(g.m) * g.k * batch, want_b = uint64_t(g.k) * g.n * batch;
      if (g.a_batch_stride[d] != want_a || g.b_batch_stride[d] != want_b) dense = false;
      batch *= g.batch_shape[d];
    }
    if (!dense || uint64_t(g.k) * batch > 0x7fffffffull) continue;
    if (!dead_after(p, j, mm.t[0].id) || !dead_after(p, k, mm.t[2].id)) continue;
    Op fused = mm;
    fused.t[0] = tr.t[0];                 // X, stored [batch*K, M]
    fused.t[2] = rd.t[1];                 // D
    fused.gemm.a = static_cast<const float *>(tr.t[0].p);
    fused.gemm.c = rd.t[1].f();
    fused.gemm.trans_a = 1;
    fused.gemm.k = static_cast<uint32_t>(g.k * batch);
    fused.gemm.batch_rank = 0;
    fused.workspace = 0;
    tr.dead = true;
    mm.dead = true;
    rd = std::move(fused);
    folded += 2;
  }
  return folded;
}

// transpose(W -> T); mult(.., T ..) with T released after the mult: the
// operand is read in its stored order instead (EXPR_MULT_LHS/RHS_DERIVATIVE,
// execute.h:187-232, and expression transposes feeding a product).
uint64_t fold_transposes(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t i = 0; i < p.size(); ++i) {
    Op &tr = p[i];
    if (tr.dead || tr.kind != Kind::Transpose || !is_last_two(tr)) continue;
    const size_t j = next_op(p, i);
    if (j == kNone) continue;
    Op &mm = p[j];
    if (mm.kind != Kind::Gemm) continue;
    tl_gemm_desc &g = mm.gemm;
    const bool as_b = same(mm.t[1], tr.t[1]) && !same(mm.t[0], tr.t[1]) && !g.trans_b;
    const bool as_a = same(mm.t[0], tr.t[1]) && !same(mm.t[1], tr.t[1]) && !g.trans_a &&
                      mm.i1 == 0;  // a flattened product's rows are not the source's rows
    if (!as_a && !as_b) continue;
    if (!dead_after(p, j, tr.t[1].id)) continue;
    if (as_b) {
      mm.t[1] = tr.t[0];
      g.b = static_cast<const float *>(tr.t[0].p);
      g.trans_b = 1;
    } else {
      mm.t[0] = tr.t[0];
      g.a = static_cast<const float *>(tr.t[0].p);
      g.trans_a = 1;
    }
    tr.dead = true;
    ++folded;
  }
  return folded;
}

// mult(X, W -> C); add(C, bias[1,N] -> C) [; GELU(C -> H)]: EXPR_LINEAR
// (execute.h:241-252) and the FFN activation as one GEMM epilogue.
uint64_t fuse_gemm_epilogues(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t i = 0; i < p.size(); ++i) {
    Op &mm = p[i];
    if (mm.dead || mm.kind != Kind::Gemm || mm.gemm.beta != 0.0f) continue;
    size_t j = next_op(p, i);
    if (j == kNone) continue;
    Op &ad = p[j];
    if (!mm.gemm.bias && ad.kind == Kind::Binary && ad.code == TL_ADD && same(ad.t[0], mm.t[2]) &&
        same(ad.t[2], mm.t[2]) && ad.t[2].same_shape(mm.t[2]) && ad.t[1].last() == mm.gemm.n &&
        ad.t[1].numel() == mm.gemm.n && !same(ad.t[1], mm.t[2])) {
      mm.t[3] = ad.t[1];
      mm.gemm.bias = ad.t[1].f();
      ad.dead = true;
      ++folded;
      j = next_op(p, i);
      if (j == kNone) continue;
    }
    Op &ge = p[j];
    if (!mm.gemm.gelu_out && ge.kind == Kind::Unary && ge.code == TL_GELU &&
        same(ge.t[0], mm.t[2]) && ge.t[1].numel() == mm.t[2].numel() && !same(ge.t[1], mm.t[2]) &&
        mm.gemm.batch_rank == 0) {
      mm.t[4] = ge.t[1];
      mm.gemm.gelu_out = ge.t[1].f();
      ge.dead = true;
      ++folded;
    }
  }
  return folded;
}

// --------------------------------------------------------- derivative rules
// SFTMX_DERIVATIVE (execute.h:291-308):
//   hadamard(g, y -> d); sum(d -> r); sub(g, r -> d); hadamard(y, d -> d)
uint64_t fuse_softmax_backward(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t i = 0; i < p.size(); ++i) {
    Op &h1 = p[i];
    if (h1.dead || h1.kind != Kind::Binary || h1.code != TL_MUL) continue;
    const TRef g = h1.t[0], y = h1.t[1], d = h1.t[2];
    if (!g.same_shape(y) || !g.same_shape(d) || same(d, g) || same(d, y)) continue;
    const size_t j = next_op(p, i);
    if (j == kNone) continue;
    Op &sm = p[j];
    if (sm.kind != Kind::Reduce || sm.code != TL_REDUCE_SUM || !same(sm.t[0], d) ||
        sm.t[1].rank != d.rank || sm.t[1].last() != 1 ||
        sm.t[1].numel() * d.last() != d.numel())
      continue;
    const TRef r = sm.t[1];
    const size_t k = next_op(p, j);
    if (k == kNone) continue;
    Op &sb = p[k];
    if (sb.kind != Kind::Binary || sb.code != TL_SUB || !same(sb.t[0], g) || !same(sb.t[1], r) ||
        !same(sb.t[2], d))
      continue;
    const size_t l = next_op(p, k);
    if (l == kNone) continue;
    Op &h2 = p[l];
    if (h2.kind != Kind::Binary || h2.code != TL_MUL || !same(h2.t[0], y) || !same(h2.t[1], d) ||
        !same(h2.t[2], d))
      continue;
    if (!dead_after(p, l, r.id)) continue;
    Op fused;
    fused.kind = Kind::SoftmaxBwd;
    fused.t[0] = g;
    fused.t[1] = y;
    fused.t[2] = d;
    h1.dead = sm.dead = sb.dead = true;
    h2 = std::move(fused);
    folded += 3;
  }
  return folded;
}

// RMSN_DERIVATIVE (execute.h:330-356):
//   RMS(x -> s); hadamard(g, y -> d); sum(d -> m); divide(m, D -> m);
//   hadamard(y, m -> d); sub(g, d -> d); divide(d, s -> d)
uint64_t fuse_rmsnorm_backward(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t i = 0; i < p.size(); ++i) {
    Op &rm = p[i];
    if (rm.dead || rm.kind != Kind::Rms) continue;
    const TRef x = rm.t[0], s = rm.t[1];
    size_t idx[6];
    size_t c = i;
    bool ok = true;
    for (int n = 0; n < 6 && ok; ++n) {
      c = next_op(p, c);
      ok = c != kNone;
      idx[n] = c;
    }
    if (!ok) continue;
    Op &h1 = p[idx[0]], &sm = p[idx[1]], &dv = p[idx[2]], &h2 = p[idx[3]], &sb = p[idx[4]],
       &dd = p[idx[5]];
    if (h1.kind != Kind::Binary || h1.code != TL_MUL) continue;
    const TRef g = h1.t[0], y = h1.t[1], d = h1.t[2];
    if (!g.same_shape(x) || !y.same_shape(x) || !d.same_shape(x) || same(d, g) || same(d, y) ||
        same(d, x))
      continue;
    if (sm.kind != Kind::Reduce || sm.code != TL_REDUCE_SUM || !same(sm.t[0], d)) continue;
    const TRef m = sm.t[1];
    if (m.numel() * x.last() != x.numel() || m.last() != 1) continue;
    if (dv.kind != Kind::Scalar || dv.code != TL_SCALAR_DIV || !same(dv.t[0], m) ||
        !same(dv.t[1], m) || dv.f0 != static_cast<float>(x.last()))
      continue;
    if (h2.kind != Kind::Binary || h2.code != TL_MUL || !same(h2.t[0], y) || !same(h2.t[1], m) ||
        !same(h2.t[2], d))
      continue;
    if (sb.kind != Kind::Binary || sb.code != TL_SUB || !same(sb.t[0], g) || !same(sb.t[1], d) ||
        !same(sb.t[2], d))
      continue;
    if (dd.kind != Kind::Binary || dd.code != TL_DIV || !same(dd.t[0], d) || !same(dd.t[1], s) ||
        !same(dd.t[2], d))
      continue;
    if (!dead_after(p, idx[5], s.id) || !dead_after(p, idx[5], m.id)) continue;
    Op fused;
    fused.kind = Kind::RmsNormBwd;
    fused.t[0] = g;
    fused.t[1] = x;
    fused.t[2] = y;
    fused.t[3] = d;
    rm.dead = h1.dead = sm.dead = dv.dead = h2.dead = sb.dead = true;
    dd = std::move(fused);
    folded += 6;
  }
  return folded;
}

// cross_entropy_derivative(z, t -> D); hadamard(root[..,1], D -> out) with D
// released: the loss root gradient applied per row inside the kernel.
// GELU_derivative(x -> T); hadamard(T, g -> out) (or (g, T)) with T
// released: the GELU chain rule in one pass.
// True when no live op strictly between i and j writes or releases `id`.
bool unchanged_between(const std::vector<Op> &p, size_t i, size_t j, uint64_t id) {
  for (size_t k = i + 1; k < j; ++k) {
    const Op &op = p[k];
    if (op.dead) continue;
    if (op.kind == Kind::Release) {
      if (op.t[0].id == id) return false;
      continue;
    }
    if (op.kind == Kind::MultiAdamW || op.kind == Kind::AllReduce) return false;
    if (writes(access(op), id)) return false;
  }
  return true;
}

// First live op after i that reads `id` (kNone if none).
size_t first_reader(const std::vector<Op> &p, size_t i, uint64_t id) {
  for (size_t j = i + 1; j < p.size(); ++j) {
    const Op &op = p[j];
    if (op.dead || op.kind == Kind::Release) continue;
    if (op.kind == Kind::MultiAdamW || op.kind == Kind::AllReduce) return kNone;
    if (reads(access(op), id)) return j;
  }
  return kNone;
}

uint64_t fuse_pointwise_backward(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t i = 0; i < p.size(); ++i) {
    Op &a = p[i];
    if (a.dead) continue;
    const bool xent = a.kind == Kind::XentBwd && !a.t[3].p;
    const bool gelu = a.kind == Kind::Unary && a.code == TL_GELU_DERIVATIVE;
    if (!xent && !gelu) continue;
    const TRef tmp = xent ? a.t[2] : a.t[1];
    // the product may come later in the program: the fused op then runs at
    // the product's position, so its other inputs must still hold the
    // values they had at op i
    const size_t j = first_reader(p, i, tmp.id);
    if (j == kNone) continue;
    Op &h = p[j];
    if (h.kind != Kind::Binary || h.code != TL_MUL || !h.t[2].same_shape(tmp)) continue;
    const bool left = same(h.t[1], tmp) && !same(h.t[0], tmp);
    const bool right = same(h.t[0], tmp) && !same(h.t[1], tmp);
    if (!left && !right) continue;
    const TRef other = left ? h.t[0] : h.t[1];
    if (!dead_after(p, j, tmp.id)) continue;
    if (!unchanged_between(p, i, j, a.t[0].id)) continue;
    if (xent && !unchanged_between(p, i, j, a.t[1].id)) continue;
    Op fused;
    if (xent) {
      // root gradient [..., 1] against logits [..., V]
      if (other.rank != tmp.rank || other.last() != 1 ||
          other.numel() * tmp.last() != tmp.numel())
        continue;
      fused = a;
      fused.t[3] = other;
      fused.t[2] = h.t[2];
    } else {
      if (!other.same_shape(tmp)) continue;
      fused.kind = Kind::GeluBwd;
      fused.t[0] = a.t[0];
      fused.t[1] = other;
      fused.t[2] = h.t[2];
    }
    h = std::move(fused);
    a.dead = true;
    ++folded;
  }
  return folded;
}

// Latest live op before j that writes `id` (kNone if none, or if the
// allocation is released or an optimiser op intervenes first).
size_t last_writer(const std::vector<Op> &p, size_t j, uint64_t id) {
  for (size_t k = j; k-- > 0;) {
    const Op &op = p[k];
    if (op.dead) continue;
    if (op.kind == Kind::Release) {
      if (op.t[0].id == id) return kNone;
      continue;
    }
    if (op.kind == Kind::MultiAdamW || op.kind == Kind::AllReduce) return kNone;
    if (writes(access(op), id)) return k;
  }
  return kNone;
}

// True when no live op strictly between i and j reads, writes or releases id.
bool untouched_between(const std::vector<Op> &p, size_t i, size_t j, uint64_t id) {
  for (size_t k = i + 1; k < j; ++k) {
    const Op &op = p[k];
    if (op.dead) continue;
    if (op.kind == Kind::Release) {
      if (op.t[0].id == id) return false;
      continue;
    }
    if (op.kind == Kind::MultiAdamW || op.kind == Kind::AllReduce) return false;
    const Access a = access(op);
    if (reads(a, id) || writes(a, id)) return false;
  }
  return true;
}

bool is_scalar_tensor(const TRef &t) { return t.p && t.numel() == 1; }

// mult(...) -> P; add(A, P) -> O (either operand order) with the add the only
// reader of P: the product is written to O with A added in the epilogue
// (C = A + (A*B + bias), the add's own arithmetic).  The executor emits this
// for every residual connection (the attention / FFN output added to the
// stream) and for every gradient that sums contributions of several paths.
uint64_t fuse_gemm_accumulate(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t j = 0; j < p.size(); ++j) {
    Op &h = p[j];
    if (h.dead || h.kind != Kind::Binary || h.code != TL_ADD) continue;
    const TRef O = h.t[2];
    for (int side = 0; side < 2; ++side) {
      const TRef P = h.t[side], A = h.t[1 - side];
      if (!P.p || !A.p || P.id == A.id || P.numel() != O.numel() || A.numel() != O.numel())
        continue;
      const size_t x = last_writer(p, j, P.id);
      if (x == kNone) continue;
      Op &mm = p[x];
      if (mm.kind != Kind::Gemm || mm.gemm.beta != 0.0f || mm.gemm.gelu_out || mm.t[5].p ||
          mm.t[2].id != P.id)
        continue;
      if (first_reader(p, x, P.id) != j || !dead_after(p, j, P.id)) continue;
      if (!unchanged_between(p, x, j, A.id) || !untouched_between(p, x, j, O.id)) continue;
      const Access ma = access(mm);
      if (reads(ma, O.id)) continue;  // the product's operands must not be its output
      mm.t[2].p = O.p;
      mm.t[2].id = O.id;
      mm.gemm.c = O.f();
      if (A.id == O.id) {
        mm.gemm.beta = 1.0f;  // accumulate in place: C = C + product
      } else {
        mm.t[5] = A;
        mm.gemm.addend = A.f();
      }
      h.dead = true;
      ++folded;
      break;
    }
  }
  return folded;
}

// softmax_backward(G, Y) -> T; divide(T, D[1]) -> O: the derivative of the
// score division (divide by sqrt(head size)) folded into the row kernel.
// rmsnorm_backward(G, X, Y) -> T; add(A, T) -> O: the residual-stream
// gradient added in the same pass.  Both run at the second op's position.
uint64_t fuse_row_backward_tails(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t i = 0; i < p.size(); ++i) {
    Op &a = p[i];
    if (a.dead) continue;
    const bool sm = a.kind == Kind::SoftmaxBwd && !a.t[3].p;
    const bool rn = a.kind == Kind::RmsNormBwd && !a.t[4].p;
    if (!sm && !rn) continue;
    const TRef T = sm ? a.t[2] : a.t[3];
    const size_t j = first_reader(p, i, T.id);
    if (j == kNone) continue;
    Op &h = p[j];
    if (h.kind != Kind::Binary || !dead_after(p, j, T.id)) continue;
    const TRef O = h.t[2];
    if (O.numel() != T.numel()) continue;
    bool inputs_ok = true;
    for (int k = 0; k < (sm ? 2 : 3); ++k)
      if (!unchanged_between(p, i, j, a.t[k].id) || a.t[k].id == O.id) inputs_ok = false;
    if (!inputs_ok) continue;
    Op fused = a;
    if (sm) {
      if (h.code != TL_DIV || !same(h.t[0], T) || same(h.t[1], T) || !is_scalar_tensor(h.t[1]))
        continue;
      fused.t[2] = O;
      fused.t[3] = h.t[1];
    } else {
      if (h.code != TL_ADD) continue;
      const bool left = same(h.t[1], T) && !same(h.t[0], T);
      const bool right = same(h.t[0], T) && !same(h.t[1], T);
      if (!left && !right) continue;
      const TRef A = left ? h.t[0] : h.t[1];
      if (A.numel() != T.numel()) continue;
      fused.t[3] = O;
      fused.t[4] = A;
    }
    h = std::move(fused);
    a.dead = true;
    ++folded;
  }
  return folded;
}

// divide(S, D[1]) -> S1; add(S1, M) -> S2 (M broadcast over leading dims);
// softmax(S2) -> P, with S1 and S2 read by nothing else: one softmax pass
// that divides and adds the mask as it reads the scores
// (nn::MultiHeadAttention, include/nn/multi_head.h).  Either step may be
// absent.
bool mask_broadcasts(const TRef &m, const TRef &s) {
  int lead = 0;
  while (lead < m.rank && m.shape[lead] == 1) ++lead;
  const int tail = m.rank - lead;
  if (tail < 1 || tail > s.rank) return false;
  for (int d = 0; d < tail; ++d)
    if (m.shape[lead + d] != s.shape[s.rank - tail + d]) return false;
  return true;
}

uint64_t fuse_score_softmax(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t k = 0; k < p.size(); ++k) {
    Op &sm = p[k];
    if (sm.dead || sm.kind != Kind::Softmax || sm.t[2].p || sm.t[3].p) continue;
    TRef X = sm.t[0];
    TRef D{}, M{};
    std::vector<size_t> gone;
    // optional mask add
    size_t j = last_writer(p, k, X.id);
    if (j != kNone && p[j].kind == Kind::Binary && p[j].code == TL_ADD) {
      const Op &ad = p[j];
      for (int side = 0; side < 2; ++side) {
        const TRef S1 = ad.t[side], m = ad.t[1 - side];
        if (S1.numel() == X.numel() && m.numel() < X.numel() && m.last() == X.last() &&
            mask_broadcasts(m, X) && first_reader(p, j, X.id) == k && dead_after(p, k, X.id) &&
            unchanged_between(p, j, k, m.id)) {
          M = m;
          gone.push_back(j);
          X = S1;
          break;
        }
      }
    }
    // optional division by a one-element tensor
    const size_t end = gone.empty() ? k : gone.back();
    size_t i = last_writer(p, end, X.id);
    if (i != kNone && p[i].kind == Kind::Binary && p[i].code == TL_DIV &&
        is_scalar_tensor(p[i].t[1]) && !same(p[i].t[1], X) && p[i].t[0].numel() == X.numel() &&
        first_reader(p, i, X.id) == end && dead_after(p, end, X.id) &&
        unchanged_between(p, i, k, p[i].t[0].id) && unchanged_between(p, i, k, p[i].t[1].id)) {
      D = p[i].t[1];
      X = p[i].t[0];
      gone.push_back(i);
    }
    if (gone.empty() || X.id == sm.t[1].id) continue;
    if (!unchanged_between(p, gone.back(), k, X.id)) continue;
    sm.t[0] = X;
    sm.t[2] = D;
    sm.t[3] = M;
    for (size_t g : gone) p[g].dead = true;
    folded += gone.size();
  }
  return folded;
}

// ---------------------------------------------- head transposes as strides
// Dense row-major strides of a shape.
void dense_strides(const TRef &t, uint64_t (&st)[kMaxRank]) {
  uint64_t acc = 1;
  for (int d = t.rank; d-- > 0;) {
    st[d] = acc;
    acc *= t.shape[d];
  }
}

// Strides, in X's memory, of the dims of Y = transpose(X, a, b).
void transposed_view(const Op &tr, uint64_t (&st)[kMaxRank]) {
  uint64_t xs[kMaxRank];
  dense_strides(tr.t[0], xs);
  for (int d = 0; d < tr.t[0].rank; ++d) st[d] = xs[d];
  std::swap(st[tr.i0], st[tr.i1]);
}

// Re-expresses the product's flattened batch over the `lead` leading dims
// of shape `dims`: operand X walks them with strides xs (from its view),
// the other operands densely (their flattened stride split over the dims).
// False unless the product's batch is exactly those dims, flattened densely
// for this operand (stride `mat`).
bool expand_batch(tl_gemm_desc &g, int which, const uint32_t *dims, int lead,
                  const uint64_t *xs, uint64_t mat) {
  if (lead > TL_GEMM_MAX_BATCH_RANK) return false;
  uint64_t *out[3] = {g.a_batch_stride, g.b_batch_stride, g.c_batch_stride};
  uint64_t count = 1;
  for (int d = 0; d < lead; ++d) count *= dims[d];
  if (g.batch_rank == static_cast<uint32_t>(lead) && lead > 1) {
    // already walked per dim (an earlier fold): this operand must be dense
    uint64_t inner = mat;
    for (int d = lead; d-- > 0;) {
      if (g.batch_shape[d] != dims[d] || out[which][d] != inner) return false;
      inner *= dims[d];
    }
    for (int d = 0; d < lead; ++d) out[which][d] = xs[d];
    return true;
  }
  uint64_t flat[3] = {0, 0, 0};
  if (g.batch_rank == 0) {
    if (count != 1) return false;
  } else {
    if (g.batch_rank != 1 || g.batch_shape[0] != count) return false;
    for (int o = 0; o < 3; ++o) flat[o] = out[o][0];
    if (flat[which] != mat) return false;
  }
  uint64_t inner = 1;  // product of dims after d
  for (int d = lead; d-- > 0;) {
    g.batch_shape[d] = dims[d];
    for (int o = 0; o < 3; ++o) out[o][d] = o == which ? xs[d] : flat[o] * inner;
    inner *= dims[d];
  }
  g.batch_rank = static_cast<uint32_t>(lead);
  return true;
}

// transpose(X -> Y) swapping dims of a [..., T, H, D]-style tensor, with Y
// read only as a GEMM operand: the GEMMs read X through strides (the batch
// walks the view's leading dims, the row stride is the view's) and the
// transpose goes.  GEMM(...) -> O; transpose(O -> Z): the GEMM writes Z
// through strides.  Attention's head split / merge
// (expr::transpose<1, 2> of nn::MultiHeadAttention, include/nn/multi_head.h)
// in both directions.
uint64_t fold_head_transposes(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t i = 0; i < p.size(); ++i) {
    Op &tr = p[i];
    if (tr.dead || tr.kind != Kind::Transpose) continue;
    const TRef X = tr.t[0], Y = tr.t[1];
    const int r = X.rank;
    if (r < 3 || Y.rank != r) continue;
    uint64_t ys[kMaxRank];
    transposed_view(tr, ys);

    // ---- input side: every reader of Y is a GEMM operand
    std::vector<size_t> readers;
    bool ok = true;
    size_t j = i;
    while (ok) {
      j = first_reader(p, j, Y.id);
      if (j == kNone) break;
      const Op &mm = p[j];
      if (mm.kind != Kind::Gemm || mm.gemm.beta != 0.0f || same(mm.t[2], Y) ||
          same(mm.t[3], Y) || same(mm.t[5], Y) || (same(mm.t[0], Y) && same(mm.t[1], Y)))
        ok = false;
      else
        readers.push_back(j);
    }
    if (ok && !readers.empty() && dead_after(p, readers.back(), Y.id) &&
        unchanged_between(p, i, readers.back(), X.id)) {
      std::vector<Op> trial;
      for (size_t k : readers) {
        Op mm = p[k];
        tl_gemm_desc &g = mm.gemm;
        const int which = same(mm.t[0], Y) ? 0 : 1;
        const bool trans = which == 0 ? g.trans_a : g.trans_b;
        // the operand as stored by the GEMM: [rows][cols] = Y's last two dims
        const uint32_t rows = which == 0 ? (trans ? g.k : g.m) : (trans ? g.n : g.k);
        const uint32_t cols = which == 0 ? (trans ? g.m : g.k) : (trans ? g.k : g.n);
        if (Y.shape[r - 2] != rows || Y.shape[r - 1] != cols || mm.i1 != 0) {
          ok = false;
          break;
        }
        uint64_t ld;
        bool flip;
        if (ys[r - 1] == 1) {
          ld = ys[r - 2];
          flip = false;
        } else if (ys[r - 2] == 1) {
          ld = ys[r - 1];
          flip = true;
        } else {
          ok = false;
          break;
        }
        if (!expand_batch(g, which, Y.shape, r - 2, ys, static_cast<uint64_t>(rows) * cols)) {
          ok = false;
          break;
        }
        if (which == 0) {
          mm.t[0] = X;
          g.a = static_cast<const float *>(X.p);
          g.lda = ld;
          if (flip) g.trans_a = !g.trans_a;
        } else {
          mm.t[1] = X;
          g.b = static_cast<const float *>(X.p);
          g.ldb = ld;
          if (flip) g.trans_b = !g.trans_b;
        }
        trial.push_back(std::move(mm));
      }
      if (ok) {
        for (size_t k = 0; k < readers.size(); ++k) p[readers[k]] = std::move(trial[k]);
        tr.dead = true;
        ++folded;
        continue;
      }
    }

    // ---- output side: a GEMM produced X for this transpose only
    const size_t x = last_writer(p, i, X.id);
    if (x == kNone) continue;
    Op &mm = p[x];
    if (mm.kind != Kind::Gemm || mm.gemm.beta != 0.0f || mm.gemm.gelu_out || mm.t[5].p ||
        mm.t[2].id != X.id || mm.i1 != 0)
      continue;
    if (first_reader(p, x, X.id) != i || !dead_after(p, i, X.id) ||
        !untouched_between(p, x, i, Y.id) || reads(access(mm), Y.id))
      continue;
    tl_gemm_desc g = mm.gemm;
    if (X.shape[r - 2] != g.m || X.shape[r - 1] != g.n || (g.ldc != 0 && g.ldc != g.n)) continue;
    // strides of X's dims inside Y (Y dense)
    uint64_t yd[kMaxRank], xs[kMaxRank];
    dense_strides(Y, yd);
    for (int d = 0; d < r; ++d) xs[d] = yd[d];
    std::swap(xs[tr.i0], xs[tr.i1]);
    uint64_t ldc;
    if (xs[r - 1] == 1) {
      ldc = xs[r - 2];
    } else if (xs[r - 2] == 1 && !g.bias) {
      // C^T = B^T A^T: the product's rows become the stored columns
      std::swap(g.a, g.b);
      std::swap(g.m, g.n);
      std::swap(g.lda, g.ldb);
      const int32_t ta = g.trans_a;
      g.trans_a = !g.trans_b;
      g.trans_b = !ta;
      for (uint32_t d = 0; d < g.batch_rank; ++d) std::swap(g.a_batch_stride[d], g.b_batch_stride[d]);
      std::swap(mm.t[0], mm.t[1]);
      ldc = xs[r - 1];
    } else {
      continue;
    }
    if (!expand_batch(g, 2, X.shape, r - 2, xs, static_cast<uint64_t>(g.m) * g.n)) continue;
    g.ldc = ldc;
    g.c = static_cast<float *>(Y.p);
    mm.gemm = g;
    mm.t[2].p = Y.p;
    mm.t[2].id = Y.id;
    tr.dead = true;
    ++folded;
  }
  return folded;
}

// ------------------------------------------------ GELU backward epilogue
// mult(...) -> G; GELU backward(x, G) -> D (GELU_derivative(x) hadamard G,
// folded by fuse_pointwise_backward) with G read by nothing else: the
// product writes D = GELU'(x) * (its value) in its epilogue (the FFN's
// gradient through the activation, include/nn/decoder_block.h).
uint64_t fuse_gemm_gelu_backward(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t k = 0; k < p.size(); ++k) {
    Op &gb = p[k];
    if (gb.dead || gb.kind != Kind::GeluBwd) continue;
    const TRef X = gb.t[0], G = gb.t[1], D = gb.t[2];
    const size_t j = last_writer(p, k, G.id);
    if (j == kNone) continue;
    Op &mm = p[j];
    const tl_gemm_desc &g = mm.gemm;
    if (mm.kind != Kind::Gemm || !same(mm.t[2], G) || g.beta != 0.0f || g.addend ||
        mm.t[5].p || g.gelu_out || g.gelu_grad_x || g.group_mode != TL_GEMM_GROUP_NONE)
      continue;
    // C dense, X and D the same dense shape
    uint64_t batch = 1;
    for (uint32_t d = 0; d < g.batch_rank; ++d) batch *= g.batch_shape[d];
    const uint64_t mn = static_cast<uint64_t>(g.m) * g.n;
    bool dense = (g.ldc == 0 || g.ldc == g.n) && batch * mn == G.numel() &&
                 X.numel() == G.numel() && D.numel() == G.numel();
    uint64_t inner = mn;
    for (uint32_t d = g.batch_rank; d-- > 0;) {
      dense = dense && g.c_batch_stride[d] == inner;
      inner *= g.batch_shape[d];
    }
    if (!dense || same(X, G) || same(D, G) || reads(access(mm), D.id) ||
        first_reader(p, j, G.id) != k || !dead_after(p, k, G.id) ||
        !unchanged_between(p, j, k, X.id) || !untouched_between(p, j, k, D.id))
      continue;
    mm.gemm.c = D.f();
    mm.gemm.gelu_grad_x = X.f();
    mm.t[2] = D;
    mm.t[6] = X;
    gb.dead = true;
    ++folded;
  }
  return folded;
}

// -------------------------------------------------------- fused attention
// A plain product: no epilogue, no groups, TF32 (the fused kernels' type).
bool plain_product(const Op &op) {
  const tl_gemm_desc &g = op.gemm;
  return !op.dead && op.kind == Kind::Gemm && g.beta == 0.0f && !g.bias && !g.gelu_out &&
         !g.addend && !g.gelu_grad_x && !op.t[5].p && g.group_mode == TL_GEMM_GROUP_NONE &&
         g.precision == TL_GEMM_TF32 && op.i1 == 0;
}

// Operand `which` (0 A, 1 B, 2 C) of a product batched over B x H (one
// flattened dim or the two dims) as per-(batch, head) blocks whose stored
// rows hold `cols` elements when dense.
bool head_view(const tl_gemm_desc &g, int which, uint32_t B, uint32_t H, uint32_t cols,
               bool transposed, tl_attn_view &v) {
  const uint64_t *st = which == 0 ? g.a_batch_stride
                       : which == 1 ? g.b_batch_stride
                                    : g.c_batch_stride;
  const uint64_t ld = which == 0 ? g.lda : which == 1 ? g.ldb : g.ldc;
  v = tl_attn_view{};
  v.p = which == 0 ? g.a : which == 1 ? g.b : g.c;
  v.row_stride = ld ? ld : cols;
  v.transposed = transposed ? 1 : 0;
  if (g.batch_rank == 1 && g.batch_shape[0] == static_cast<uint64_t>(B) * H) {
    v.head_stride = st[0];
    v.batch_stride = st[0] * H;
  } else if (g.batch_rank == 2 && g.batch_shape[0] == B && g.batch_shape[1] == H) {
    v.batch_stride = st[0];
    v.head_stride = st[1];
  } else {
    return false;
  }
  return true;
}

bool dense_scores(const tl_attn_view &v, uint32_t H, uint32_t T) {
  const uint64_t tt = static_cast<uint64_t>(T) * T;
  return v.row_stride == T && v.head_stride == tt && v.batch_stride == tt * H && !v.transposed;
}

// [B, H, T, T] tensor: its B, H, T.
bool score_dims(const TRef &t, uint32_t &B, uint32_t &H, uint32_t &T) {
  if (t.rank != 4 || t.shape[2] != t.shape[3]) return false;
  B = t.shape[0];
  H = t.shape[1];
  T = t.shape[2];
  return true;
}

// The executor's attention composite (include/nn/multi_head.h:45-52 and its
// gradients) on the fused tensor-core kernels:
//   forward   S = Q K^T (product), softmax(S / divisor + mask) -> P, O = P V
//             -> one op at O's product (S never written)
//   backward  dP = dO V^T, softmax derivative(dP, P) / divisor -> dS,
//             dQ = dS K -> one op at dQ's product (dP never written)
//   dK = dS^T Q and dV = P^T dO (square [T, T] left operands) -> the
//             key-side kernel in place of the product
// Each only when the fused kernels take the operands' strides and the
// values read at the fused op's position are those the originals read.
// The runtime's flash-attention state (records of virtual P tensors, LSE
// buffers, per-mask causal words) for the program being optimised; null
// when the caller keeps none.
thread_local FlashState *g_flash = nullptr;

uint64_t fuse_attention(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t k = 0; k < p.size(); ++k) {
    Op &sm = p[k];
    if (sm.dead) continue;
    if (sm.kind == Kind::Softmax && sm.t[2].p) {
      const TRef X = sm.t[0], Y = sm.t[1], div = sm.t[2], mask = sm.t[3];
      uint32_t B, H, T;
      if (!score_dims(Y, B, H, T) || !is_scalar_tensor(div)) continue;
      if (mask.p && mask.numel() != static_cast<uint64_t>(T) * T) continue;
      const size_t i = last_writer(p, k, X.id);
      if (i == kNone || !plain_product(p[i]) || first_reader(p, i, X.id) != k ||
          !dead_after(p, k, X.id))
        continue;
      const size_t j = first_reader(p, k, Y.id);
      if (j == kNone || !plain_product(p[j]) || !same(p[j].t[0], Y) || same(p[j].t[1], Y))
        continue;
      const tl_gemm_desc &g1 = p[i].gemm, &g2 = p[j].gemm;
      if (g1.m != T || g1.n != T || g1.k != kFusedHeadDimHost || g1.trans_a || g2.m != T ||
          g2.k != T || g2.n != kFusedHeadDimHost || g2.trans_a || g2.trans_b)
        continue;
      tl_attn_desc d{};
      d.pass = TL_ATTN_FORWARD;
      d.B = B;
      d.H = H;
      d.T = T;
      d.D = kFusedHeadDimHost;
      tl_attn_view sv, pv;
      if (!head_view(g1, 0, B, H, g1.k, false, d.q) ||
          !head_view(g1, 1, B, H, g1.trans_b ? g1.k : g1.n, !g1.trans_b, d.k) ||
          !head_view(g1, 2, B, H, T, false, sv) || !dense_scores(sv, H, T) ||
          !head_view(g2, 0, B, H, T, false, pv) || !dense_scores(pv, H, T) ||
          !head_view(g2, 1, B, H, g2.n, false, d.v) || !head_view(g2, 2, B, H, g2.n, false, d.o))
        continue;
      d.divisor = div.f();
      d.mask = mask.p ? mask.f() : nullptr;
      d.p = Y.f();
      const TRef Q = p[i].t[0], K = p[i].t[1];
      if (!unchanged_between(p, i, j, Q.id) || !unchanged_between(p, i, j, K.id) ||
          !unchanged_between(p, k, j, div.id) || (mask.p && !unchanged_between(p, k, j, mask.id)) ||
          !untouched_between(p, k, j, Y.id) || tl_attention_fused_supported(&d) != 1)
        continue;
      // the causal check of the mask: one runtime word per mask, checked
      // once per program (assign_mask_checks)
      if (mask.p && g_flash) d.mask_flag = g_flash->mask_word(mask.id);
      Op fused{};
      fused.kind = Kind::Attention;
      fused.code = TL_ATTN_FORWARD;
      fused.attn = d;
      fused.workspace = 256;  // the causal-mask word when the runtime keeps none
      fused.t[0] = Q;
      fused.t[1] = K;
      fused.t[2] = p[j].t[1];
      fused.t[3] = div;
      fused.t[4] = mask;
      fused.t[5] = Y;
      fused.t[6] = p[j].t[2];
      fused.src = p[j].src;
      p[i].dead = true;
      sm.dead = true;
      p[j] = std::move(fused);
      folded += 2;
    } else if (sm.kind == Kind::SoftmaxBwd && sm.t[3].p) {
      const TRef dP = sm.t[0], P = sm.t[1], dS = sm.t[2], div = sm.t[3];
      uint32_t B, H, T;
      if (!score_dims(P, B, H, T) || !dS.same_shape(P) || !is_scalar_tensor(div)) continue;
      const size_t i = last_writer(p, k, dP.id);
      if (i == kNone || !plain_product(p[i]) || first_reader(p, i, dP.id) != k ||
          !dead_after(p, k, dP.id))
        continue;
      const size_t j = first_reader(p, k, dS.id);
      if (j == kNone || !plain_product(p[j]) || !same(p[j].t[0], dS) || same(p[j].t[1], dS))
        continue;
      const tl_gemm_desc &g1 = p[i].gemm, &g2 = p[j].gemm;
      if (g1.m != T || g1.n != T || g1.k != kFusedHeadDimHost || g1.trans_a || !g1.trans_b ||
          g2.m != T || g2.k != T || g2.n != kFusedHeadDimHost || g2.trans_a)
        continue;
      tl_attn_desc d{};
      d.pass = TL_ATTN_BACKWARD_Q;
      d.B = B;
      d.H = H;
      d.T = T;
      d.D = kFusedHeadDimHost;
      tl_attn_view pv, sv;
      if (!head_view(g1, 0, B, H, g1.k, false, d.d_o) ||
          !head_view(g1, 1, B, H, g1.k, false, d.v) || !head_view(g1, 2, B, H, T, false, pv) ||
          !dense_scores(pv, H, T) || !head_view(g2, 0, B, H, T, false, sv) ||
          !dense_scores(sv, H, T) ||
          !head_view(g2, 1, B, H, g2.trans_b ? g2.k : g2.n, g2.trans_b, d.k) ||
          !head_view(g2, 2, B, H, g2.n, false, d.dq))
        continue;
      d.divisor = div.f();
      d.p = P.f();
      d.ds = dS.f();
      const TRef dO = p[i].t[0], V = p[i].t[1];
      if (!unchanged_between(p, i, j, dO.id) || !unchanged_between(p, i, j, V.id) ||
          !unchanged_between(p, k, j, P.id) || !unchanged_between(p, k, j, div.id) ||
          !untouched_between(p, k, j, dS.id) || tl_attention_fused_supported(&d) != 1)
        continue;
      Op fused{};
      fused.kind = Kind::Attention;
      fused.code = TL_ATTN_BACKWARD_Q;
      fused.attn = d;
      fused.t[0] = dO;
      fused.t[1] = V;
      fused.t[2] = p[j].t[1];
      fused.t[3] = P;
      fused.t[4] = div;
      fused.t[5] = dS;
      fused.t[6] = p[j].t[2];
      fused.src = p[j].src;
      p[i].dead = true;
      sm.dead = true;
      p[j] = std::move(fused);
      folded += 2;
    }
  }
  // dK = dS^T Q, dV = P^T dO: square left operand, transposed
  for (Op &op : p) {
    if (!plain_product(op)) continue;
    const tl_gemm_desc &g = op.gemm;
    uint32_t B, H, T;
    if (!g.trans_a || g.trans_b || !score_dims(op.t[0], B, H, T) || g.m != T || g.k != T ||
        g.n != kFusedHeadDimHost)
      continue;
    tl_attn_desc d{};
    d.pass = TL_ATTN_PRODUCT_TN;
    d.B = B;
    d.H = H;
    d.T = T;
    d.D = kFusedHeadDimHost;
    tl_attn_view av;
    if (!head_view(g, 0, B, H, T, false, av) || !dense_scores(av, H, T) ||
        !head_view(g, 1, B, H, g.n, false, d.q) || !head_view(g, 2, B, H, g.n, false, d.dk))
      continue;
    d.ds = op.t[0].f();
    if (tl_attention_fused_supported(&d) != 1) continue;
    Op fused{};
    fused.kind = Kind::Attention;
    fused.code = TL_ATTN_PRODUCT_TN;
    fused.attn = d;
    fused.t[0] = op.t[0];
    fused.t[1] = op.t[1];
    fused.t[2] = op.t[2];
    fused.src = op.src;
    op = std::move(fused);
  }
  return folded;
}

// ---------------------------------------------------------- flash attention
// The attention composite on the flash kernels (any sequence length):
//   forward   S = Q K^T, softmax(S / divisor + mask) -> P, O = P V  ->  one
//             FlashFwd at O's product, writing O and P's row log-sum-exp
//             only; P stays virtual (FlashRecord) for the backward window
//   backward  dP = dO V^T, softmax derivative(dP, P) / divisor -> dS,
//             dQ = dS K, dK = dS^T Q, dV = P^T dO  ->  one FlashBwd at the
//             first of these ops (the gradients are consumed right after
//             each is made, so they are written early, never late), P of a
//             virtual record recomputed from Q, K and the log-sum-exp, dP
//             and dS never written
// resolve_flash then rebuilds a virtual P (FlashProbs) in front of any other
// reader, and before any write or release of its recipe's inputs.


bool no_reuse_between(const std::vector<Op> &p, size_t i, size_t j, const TRef &dst);

bool same_view(const tl_attn_view &a, const tl_attn_view &b) {
  return a.p == b.p && a.batch_stride == b.batch_stride && a.head_stride == b.head_stride &&
         a.row_stride == b.row_stride && a.transposed == b.transposed;
}

const FlashRecord *flash_record(uint64_t p_id) {
  if (!g_flash) return nullptr;
  for (const FlashRecord &r : g_flash->records())
    if (r.p_id == p_id) return &r;
  return nullptr;
}

uint64_t fuse_flash_forward(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t k = 0; k < p.size(); ++k) {
    Op &sm = p[k];
    if (sm.dead || sm.kind != Kind::Softmax || !sm.t[2].p) continue;
    const TRef X = sm.t[0], Y = sm.t[1], div = sm.t[2], mask = sm.t[3];
    uint32_t B, H, T;
    if (!score_dims(Y, B, H, T) || !is_scalar_tensor(div)) continue;
    if (!g_flash->always() && T <= kFusedMaxKeysHost) continue;  // the fused kernels' range
    if (mask.p && mask.numel() != static_cast<uint64_t>(T) * T) continue;
    const size_t i = last_writer(p, k, X.id);
    if (i == kNone || !plain_product(p[i]) || first_reader(p, i, X.id) != k ||
        !dead_after(p, k, X.id))
      continue;
    const size_t j = first_reader(p, k, Y.id);
    if (j == kNone || !plain_product(p[j]) || !same(p[j].t[0], Y) || same(p[j].t[1], Y))
      continue;
    const tl_gemm_desc &g1 = p[i].gemm, &g2 = p[j].gemm;
    if (g1.m != T || g1.n != T || g1.k != kFusedHeadDimHost || g1.trans_a || g2.m != T ||
        g2.k != T || g2.n != kFusedHeadDimHost || g2.trans_a || g2.trans_b)
      continue;
    tl_flash_desc d{};
    d.B = B;
    d.H = H;
    d.T = T;
    d.D = kFusedHeadDimHost;
    tl_attn_view sv, pv;
    if (!head_view(g1, 0, B, H, g1.k, false, d.q) ||
        !head_view(g1, 1, B, H, g1.trans_b ? g1.k : g1.n, !g1.trans_b, d.k) ||
        !head_view(g1, 2, B, H, T, false, sv) || !dense_scores(sv, H, T) ||
        !head_view(g2, 0, B, H, T, false, pv) || !dense_scores(pv, H, T) ||
        !head_view(g2, 1, B, H, g2.n, false, d.v) || !head_view(g2, 2, B, H, g2.n, false, d.o))
      continue;
    const TRef Q = p[i].t[0], K = p[i].t[1];
    if (!unchanged_between(p, i, j, Q.id) || !unchanged_between(p, i, j, K.id) ||
        !unchanged_between(p, k, j, div.id) || (mask.p && !unchanged_between(p, k, j, mask.id)) ||
        !untouched_between(p, k, j, Y.id))
      continue;
    d.divisor = div.f();
    d.mask = mask.p ? mask.f() : nullptr;
    d.mask_flag = mask.p ? g_flash->mask_word(mask.id) : nullptr;
    d.lse = g_flash->lse_buffer(Y.id, static_cast<size_t>(B) * H * T * 4);
    if (tl_flash_attention_supported(&d) != 1 || !d.lse || (mask.p && !d.mask_flag)) continue;
    Op fused{};
    fused.kind = Kind::FlashFwd;
    fused.code = 0;  // bit 0, check the mask first: assign_mask_checks
    fused.flash = d;
    fused.t[0] = Q;
    fused.t[1] = K;
    fused.t[2] = p[j].t[1];
    fused.t[3] = div;
    fused.t[4] = mask;
    fused.t[5] = Y;
    fused.t[6] = p[j].t[2];
    fused.src = p[j].src;
    p[i].dead = true;
    sm.dead = true;
    p[j] = std::move(fused);
    folded += 2;
  }
  return folded;
}

// Readers of `id` after op `after`: their positions (live ops only, up to
// the allocation's release or a full rewrite).
std::vector<size_t> readers_after(const std::vector<Op> &p, size_t after, uint64_t id) {
  std::vector<size_t> out;
  for (size_t j = after + 1; j < p.size(); ++j) {
    const Op &op = p[j];
    if (op.dead) continue;
    if (op.kind == Kind::Release) {
      if (op.t[0].id == id) break;
      continue;
    }
    if (op.kind == Kind::MultiAdamW || op.kind == Kind::AllReduce) continue;
    const Access a = access(op);
    if (reads(a, id)) out.push_back(j);
    if (writes(a, id) && !reads(a, id) && full_write(op)) break;
  }
  return out;
}

uint64_t fuse_flash_backward(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t k = 0; k < p.size(); ++k) {
    Op &sm = p[k];
    if (sm.dead || sm.kind != Kind::SoftmaxBwd || !sm.t[3].p) continue;
    const TRef dP = sm.t[0], P = sm.t[1], dS = sm.t[2], div = sm.t[3];
    const FlashRecord *rec = flash_record(P.id);
    uint32_t B, H, T;
    if (!rec || !rec->o_valid || !score_dims(P, B, H, T) || !dS.same_shape(P) ||
        B != rec->desc.B || H != rec->desc.H || T != rec->desc.T || !same(div, rec->divisor))
      continue;
    // dP = dO V^T, read only by the softmax derivative
    const size_t i = last_writer(p, k, dP.id);
    if (i == kNone || !plain_product(p[i]) || first_reader(p, i, dP.id) != k ||
        !dead_after(p, k, dP.id))
      continue;
    const tl_gemm_desc &g1 = p[i].gemm;
    if (g1.m != T || g1.n != T || g1.k != kFusedHeadDimHost || g1.trans_a || !g1.trans_b)
      continue;
    // dS read by exactly dQ = dS K and dK = dS^T Q, then dead; P^T dO -> dV
    const std::vector<size_t> ds_readers = readers_after(p, k, dS.id);
    if (ds_readers.size() != 2) continue;
    size_t jq = kNone, jk = kNone, jv = kNone;
    for (size_t r : ds_readers) {
      const Op &op = p[r];
      if (!plain_product(op) || !same(op.t[0], dS) || same(op.t[1], dS)) continue;
      const tl_gemm_desc &g = op.gemm;
      if (g.m != T || g.k != T || g.n != kFusedHeadDimHost) continue;
      if (!g.trans_a) jq = r;
      else if (!g.trans_b) jk = r;
    }
    if (jq == kNone || jk == kNone || !dead_after(p, std::max(jq, jk), dS.id)) continue;
    for (size_t r : readers_after(p, k, P.id)) {
      const Op &op = p[r];
      if (plain_product(op) && same(op.t[0], P) && op.gemm.trans_a && !op.gemm.trans_b &&
          op.gemm.m == T && op.gemm.k == T && op.gemm.n == kFusedHeadDimHost &&
          same(op.t[1], p[i].t[0])) {
        jv = r;
        break;
      }
    }
    if (jv == kNone) continue;
    const tl_gemm_desc &gq = p[jq].gemm, &gk = p[jk].gemm, &gv = p[jv].gemm;
    tl_flash_desc d = rec->desc;
    tl_attn_view kq, qk, dov, vv, dov2;
    if (!head_view(g1, 0, B, H, g1.k, false, dov) || !head_view(g1, 1, B, H, g1.k, true, vv) ||
        !head_view(gq, 1, B, H, gq.trans_b ? gq.k : gq.n, gq.trans_b, kq) ||
        !head_view(gq, 2, B, H, gq.n, false, d.dq) ||
        !head_view(gk, 1, B, H, gk.n, false, qk) || !head_view(gk, 2, B, H, gk.n, false, d.dk) ||
        !head_view(gv, 1, B, H, gv.n, false, dov2) || !head_view(gv, 2, B, H, gv.n, false, d.dv))
      continue;
    // the backward's operands are the recipe's tensors, read the same way
    vv.transposed = 0;
    if (!same(p[jq].t[1], rec->k) || !same_view(kq, rec->desc.k) || !same(p[jk].t[1], rec->q) ||
        !same_view(qk, rec->desc.q) || !same(p[i].t[1], rec->v) || !same_view(vv, rec->desc.v) ||
        !same_view(dov, dov2))
      continue;
    d.d_o = dov;
    // the fused op runs at F, the first of the group; its inputs exist there
    // (dO is the dP product's input) and are read-only up to the last one
    const size_t F = std::min({i, k, jq, jk, jv});
    const size_t J = std::max({jq, jk, jv});
    const TRef dO = p[i].t[0], dQ = p[jq].t[2], dK = p[jk].t[2], dV = p[jv].t[2];
    bool ok = true;
    for (const TRef *in : {&rec->q, &rec->k, &rec->v, &rec->divisor, &dO, &P})
      ok = ok && unchanged_between(p, F, J, in->id);
    ok = ok && (!rec->mask.p || unchanged_between(p, F, J, rec->mask.id));
    // O: not written in this program before the backward (from op 0 on)
    ok = ok && unchanged_between(p, kNone, F, rec->o.id);
    // each gradient is written at F instead of at its product: nothing in
    // between may read or write its buffer, or reuse its addresses
    for (size_t r : {jq, jk, jv}) {
      const TRef &out = p[r].t[2];
      ok = ok && untouched_between(p, F, r, out.id) && no_reuse_between(p, F, r, out);
      for (const TRef *in : {&rec->q, &rec->k, &rec->v, &rec->o, &dO, &P})
        ok = ok && out.id != in->id;
    }
    ok = ok && dQ.id != dK.id && dQ.id != dV.id && dK.id != dV.id;
    if (!ok) continue;
    Op fused{};
    fused.kind = Kind::FlashBwd;
    fused.flash = d;
    fused.t[0] = rec->q;
    fused.t[1] = rec->k;
    fused.t[2] = rec->v;
    fused.t[3] = rec->o;
    fused.t[4] = dO;
    fused.t[5] = rec->divisor;
    fused.t[6] = P;
    fused.t[7] = dK;
    fused.t[8] = dV;
    fused.group_refs = {dQ, rec->mask};
    fused.workspace = static_cast<size_t>(B) * H * T * 4;  // delta = rowsum(dO * O)
    fused.src = p[F].src;
    for (size_t r : {i, k, jq, jk, jv})
      if (r != F) p[r].dead = true;
    p[F] = std::move(fused);
    folded += 4;
  }
  return folded;
}

// One op's effect on the virtual-P records.  Returns the records that must
// be rebuilt before the op (it reads P, writes part of it, or changes or
// releases an input of P's recipe); those leave the list.
std::vector<FlashRecord> step_flash_records(const Op &op, std::vector<FlashRecord> &records) {
  std::vector<FlashRecord> rebuild;
  if (op.dead) return rebuild;
  if (op.kind == Kind::Release) {
    const uint64_t id = op.t[0].id;
    for (size_t r = 0; r < records.size();) {
      const FlashRecord &f = records[r];
      if (f.p_id == id) {
        records.erase(records.begin() + static_cast<std::ptrdiff_t>(r));
        continue;
      }
      if (id == f.q.id || id == f.k.id || id == f.divisor.id || (f.mask.p && id == f.mask.id)) {
        rebuild.push_back(f);
        records.erase(records.begin() + static_cast<std::ptrdiff_t>(r));
        continue;
      }
      if (id == f.o.id) records[r].o_valid = false;
      ++r;
    }
    return rebuild;
  }
  const bool opaque = op.kind == Kind::MultiAdamW || op.kind == Kind::AllReduce;
  const Access a = access(op);
  for (size_t r = 0; r < records.size();) {
    FlashRecord &f = records[r];
    bool touches = false;
    if (opaque) {
      for (const auto &m : op.multi)
        for (const TRef *t : {&m.param, &m.out, &m.grad, &m.m1, &m.m2})
          touches = touches || (t->p && (t->id == f.p_id || t->id == f.q.id ||
                                         t->id == f.k.id || t->id == f.divisor.id ||
                                         (f.mask.p && t->id == f.mask.id)));
    }
    const bool fwd_here = op.kind == Kind::FlashFwd && op.t[5].id == f.p_id;
    const bool reads_p = op.kind != Kind::FlashBwd && !fwd_here && reads(a, f.p_id);
    const bool writes_p = writes(a, f.p_id);
    const bool recipe = writes(a, f.q.id) || writes(a, f.k.id) || writes(a, f.divisor.id) ||
                        (f.mask.p && writes(a, f.mask.id));
    if (op.kind == Kind::FlashProbs && op.t[4].id == f.p_id) {
      records.erase(records.begin() + static_cast<std::ptrdiff_t>(r));
      continue;
    }
    if (touches || reads_p || recipe || (writes_p && !fwd_here && !full_write(op))) {
      rebuild.push_back(f);
      records.erase(records.begin() + static_cast<std::ptrdiff_t>(r));
      continue;
    }
    if (writes_p) {  // P redefined (a FlashFwd replaces the record below)
      records.erase(records.begin() + static_cast<std::ptrdiff_t>(r));
      continue;
    }
    if (writes(a, f.o.id)) f.o_valid = false;
    ++r;
  }
  if (op.kind == Kind::FlashFwd) {
    FlashRecord f;
    f.p_id = op.t[5].id;
    f.p = op.t[5];
    f.q = op.t[0];
    f.k = op.t[1];
    f.v = op.t[2];
    f.divisor = op.t[3];
    f.mask = op.t[4];
    f.o = op.t[6];
    f.desc = op.flash;
    records.push_back(f);
  }
  return rebuild;
}

Op flash_probs_op(const FlashRecord &f) {
  Op op{};
  op.kind = Kind::FlashProbs;
  op.flash = f.desc;
  op.t[0] = f.q;
  op.t[1] = f.k;
  op.t[2] = f.divisor;
  op.t[3] = f.mask;
  op.t[4] = f.p;
  return op;
}

// True when, from op `from` on, allocation `id` is redefined (fully
// written, or defined anew by a flash forward) or released before anything
// reads it: its current value is dead.
bool redefined_before_read(const std::vector<Op> &p, size_t from, uint64_t id) {
  for (size_t j = from; j < p.size(); ++j) {
    const Op &op = p[j];
    if (op.dead) continue;
    if (op.kind == Kind::Release) {
      if (op.t[0].id == id) return true;
      continue;
    }
    if (op.kind == Kind::MultiAdamW || op.kind == Kind::AllReduce) return false;
    if (op.kind == Kind::FlashFwd && op.t[5].id == id) return true;
    const Access a = access(op);
    if (reads(a, id)) return false;
    if (writes(a, id) && full_write(op)) return true;
  }
  return false;  // alive at the end: a later window may read it
}

// Inserts FlashProbs where a virtual P must exist (see step_flash_records);
// a P whose value is dead there (the next forward redefines it) is dropped.
uint64_t resolve_flash(std::vector<Op> &p) {
  std::vector<FlashRecord> records = g_flash ? g_flash->records() : std::vector<FlashRecord>{};
  bool any = !records.empty();
  for (const Op &op : p) any = any || (!op.dead && op.kind == Kind::FlashFwd);
  if (!any) return 0;
  std::vector<Op> out;
  out.reserve(p.size() + 4);
  uint64_t added = 0;
  for (size_t j = 0; j < p.size(); ++j) {
    for (const FlashRecord &f : step_flash_records(p[j], records)) {
      if (redefined_before_read(p, j, f.p_id)) continue;
      out.push_back(flash_probs_op(f));
      ++added;
    }
    out.push_back(std::move(p[j]));
  }
  p = std::move(out);
  return added;
}

}  // namespace

void update_flash_records(const std::vector<Op> &prog, std::vector<FlashRecord> &records) {
  for (const Op &op : prog) step_flash_records(op, records);
}

namespace {

// ------------------------------------------------------- grouped products
// (flattened products, op.i1 = 1, are ordinary M x N x K products here)
// mult(X, W -> C) [+ bias]; transpose(C viewed as [B, T, H, D], 1, 2 -> Y)
// with C read by nothing else: the split_heads of nn::MultiHeadAttention's
// query, key and value projections (include/nn/multi_head.h) done by the
// product's store, which writes Y's [B, H, T, D] layout directly
// (tl_gemm_desc.c_heads), so C is never written and the transpose never runs.
// Moving a write of `dst` from op j up to op i is safe only if no block
// released between them overlaps dst's addresses: the pool hands released
// blocks out again, so dst (allocated after such a release) may sit where a
// block that ops between i and j still read used to be.
bool no_reuse_between(const std::vector<Op> &p, size_t i, size_t j, const TRef &dst) {
  const uintptr_t d0 = reinterpret_cast<uintptr_t>(dst.p), d1 = d0 + dst.numel() * 4;
  for (size_t k = i + 1; k < j; ++k) {
    const Op &op = p[k];
    if (op.kind != Kind::Release) continue;
    const uintptr_t r0 = reinterpret_cast<uintptr_t>(op.t[0].p), r1 = r0 + op.n;
    if (r0 < d1 && d0 < r1) return false;
  }
  return true;
}

uint64_t fuse_head_split_store(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t i = 0; i < p.size(); ++i) {
    Op &g = p[i];
    if (g.dead || g.kind != Kind::Gemm || !g.t[2].p) continue;
    const tl_gemm_desc &d = g.gemm;
    if (d.group_mode != TL_GEMM_GROUP_NONE || d.batch_rank || d.beta != 0.0f || d.addend ||
        d.gelu_out || d.gelu_grad_x || d.c_heads || (d.ldc && d.ldc != d.n) ||
        d.precision == TL_GEMM_FP32)
      continue;
    const size_t j = first_reader(p, i, g.t[2].id);
    if (j == kNone) continue;
    const Op &tr = p[j];
    if (tr.kind != Kind::Transpose || tr.t[0].rank != 4 || tr.i0 != 1 || tr.i1 != 2 ||
        tr.t[0].p != g.t[2].p)
      continue;
    const TRef &src = tr.t[0], &dst = tr.t[1];
    const uint32_t B = src.shape[0], T = src.shape[1], H = src.shape[2], D = src.shape[3];
    if (static_cast<uint64_t>(B) * T != d.m || static_cast<uint64_t>(H) * D != d.n ||
        D % 32 || T % 32 || dst.rank != 4 || dst.shape[0] != B || dst.shape[1] != H ||
        dst.shape[2] != T || dst.shape[3] != D || (reinterpret_cast<uintptr_t>(dst.p) & 15u))
      continue;
    bool operand = false;  // Y must not be one of the product's inputs
    for (int k : {0, 1, 3})
      if (g.t[k].p && g.t[k].id == dst.id) operand = true;
    if (operand || !unchanged_between(p, i, j, g.t[2].id) ||
        !untouched_between(p, i, j, dst.id) || !dead_after(p, j, g.t[2].id) ||
        !no_reuse_between(p, i, j, dst))
      continue;
    // only the tensor-core kernel stores the head layout: fold only products
    // that take it (tl_gemm refuses a head-split store anywhere else)
    tl_gemm_desc folded_desc = g.gemm;
    folded_desc.c = dst.f();
    folded_desc.c_heads = H;
    folded_desc.c_head_rows = T;
    if (tl_gemm_on_tensor_cores(&folded_desc) != 1) continue;
    g.gemm.c = dst.f();
    g.gemm.c_heads = H;
    g.gemm.c_head_rows = T;
    g.t[2] = dst;
    p[j].dead = true;
    ++folded;
  }
  return folded;
}

bool groupable(const Op &op) {
  return !op.dead && op.kind == Kind::Gemm && op.gemm.group_mode == TL_GEMM_GROUP_NONE &&
         !op.gemm.gelu_out && !op.gemm.gelu_grad_x;
}

// Same product shape and layout (everything but the operand addresses).
bool same_product(const tl_gemm_desc &a, const tl_gemm_desc &b) {
  if (a.m != b.m || a.n != b.n || a.k != b.k || a.trans_a != b.trans_a ||
      a.trans_b != b.trans_b || a.precision != b.precision || a.lda != b.lda ||
      a.ldb != b.ldb || a.ldc != b.ldc || a.batch_rank != b.batch_rank ||
      a.c_heads != b.c_heads || a.c_head_rows != b.c_head_rows)
    return false;
  for (uint32_t d = 0; d < a.batch_rank; ++d)
    if (a.batch_shape[d] != b.batch_shape[d] || a.a_batch_stride[d] != b.a_batch_stride[d] ||
        a.b_batch_stride[d] != b.b_batch_stride[d] || a.c_batch_stride[d] != b.c_batch_stride[d])
      return false;
  return true;
}

// Products of one input by several weights (nn::MultiHeadAttention's
// w_q, w_k, w_v applied to one tensor, include/nn/multi_head.h; their weight
// gradients X^T dQ, X^T dK, X^T dV) run as one N-grouped launch, either at
// the first product's position (later weights and biases unchanged since
// then, later outputs untouched) or at the last one's (earlier operands
// unchanged until then, earlier outputs not read before it).
uint64_t group_shared_input(std::vector<Op> &p) {
  uint64_t folded = 0;
  auto clash = [&](const std::vector<size_t> &members, const Op &y) {
    for (size_t k : members) {
      const Op &z = p[k];
      for (uint64_t id : {z.t[0].id, z.t[1].id, z.t[2].id, z.t[3].id})
        if (id && id == y.t[2].id) return true;
      if (y.t[1].id == z.t[2].id || (y.t[3].p && y.t[3].id == z.t[2].id)) return true;
    }
    return false;
  };
  for (size_t i = 0; i < p.size(); ++i) {
    Op &x = p[i];
    if (!groupable(x) || x.gemm.beta != 0.0f || x.t[5].p) continue;
    std::vector<size_t> cand;
    for (size_t j = i + 1; j < p.size() && j < i + 256; ++j) {
      const Op &y = p[j];
      if (groupable(y) && y.gemm.beta == 0.0f && !y.t[5].p && same(y.t[0], x.t[0]) &&
          same_product(x.gemm, y.gemm))
        cand.push_back(j);
    }
    if (cand.empty()) continue;
    // hoist to i
    std::vector<size_t> members{i};
    for (size_t j : cand) {
      if (members.size() == TL_GEMM_MAX_GROUPS) break;
      const Op &y = p[j];
      if (!unchanged_between(p, i, j, x.t[0].id) || !unchanged_between(p, i, j, y.t[1].id) ||
          (y.t[3].p && !unchanged_between(p, i, j, y.t[3].id)) ||
          !untouched_between(p, i, j, y.t[2].id) || clash(members, y))
        continue;
      members.push_back(j);
    }
    size_t at = i;
    if (members.size() < 2) {
      // sink to the last candidate that keeps every earlier member valid
      members.assign(1, i);
      for (size_t j : cand) {
        if (members.size() == TL_GEMM_MAX_GROUPS) break;
        const Op &y = p[j];
        if (clash(members, y) || !unchanged_between(p, i, j, x.t[0].id)) continue;
        bool ok = true;
        for (size_t k : members) {
          const Op &z = p[k];
          for (const TRef *r : {&z.t[1], &z.t[3]})
            if (r->p && !unchanged_between(p, k, j, r->id)) ok = false;
          if (!untouched_between(p, k, j, z.t[2].id)) ok = false;
        }
        if (ok) members.push_back(j);
      }
      if (members.size() < 2) continue;
      at = members.back();
    }
    Op grouped = p[members.front()];
    tl_gemm_desc &g = grouped.gemm;
    g.group_mode = TL_GEMM_GROUP_N;
    g.groups = static_cast<uint32_t>(members.size());
    grouped.group_refs.clear();
    for (size_t k = 0; k < members.size(); ++k) {
      const Op &y = p[members[k]];
      g.b_group[k] = y.gemm.b;
      g.c_group[k] = y.gemm.c;
      g.bias_group[k] = y.gemm.bias;
      if (k > 0) {
        grouped.group_refs.push_back(y.t[1]);
        grouped.group_refs.push_back(y.t[2]);
        grouped.group_refs.push_back(y.t[3]);
      }
    }
    for (size_t k : members) p[k].dead = true;
    p[at] = std::move(grouped);
    folded += members.size() - 1;
  }
  return folded;
}

// The input gradient of a tensor used by several products, summed by the
// executor one product at a time (dX = dQ Wq^T, + dK Wk^T, + dV Wv^T after
// the accumulate folds: a product, one with it as addend, one accumulating
// in place): one K-grouped product over the concatenated K at the last
// product's position.
uint64_t group_summed_products(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t i = 0; i < p.size(); ++i) {
    if (!groupable(p[i]) || p[i].gemm.beta != 0.0f) continue;
    std::vector<size_t> chain{i};
    size_t cur = i;
    while (chain.size() < TL_GEMM_MAX_GROUPS) {
      const TRef out = p[cur].t[2];
      const size_t j = first_reader(p, cur, out.id);
      if (j == kNone) break;
      const Op &y = p[j];
      if (!groupable(y) || y.t[3].p || !same_product(p[i].gemm, y.gemm)) break;
      const bool as_addend = y.gemm.beta == 0.0f && same(y.t[5], out) && !same(y.t[0], out) &&
                             !same(y.t[1], out);
      const bool in_place = y.gemm.beta != 0.0f && !y.t[5].p && same(y.t[2], out) &&
                            !same(y.t[0], out) && !same(y.t[1], out);
      if (!as_addend && !in_place) break;
      if (as_addend && !dead_after(p, j, out.id)) break;
      chain.push_back(j);
      cur = j;
    }
    if (chain.size() < 2) continue;
    const size_t last = chain.back();
    bool ok = true;
    for (size_t k = 0; k + 1 < chain.size() && ok; ++k) {
      const Op &y = p[chain[k]];
      for (const TRef *r : {&y.t[0], &y.t[1], &y.t[3], &y.t[5]})
        if (r->p && !unchanged_between(p, chain[k], last, r->id)) ok = false;
    }
    if (!ok) continue;
    Op merged = p[last];
    const Op &first = p[chain.front()];
    tl_gemm_desc &g = merged.gemm;
    g.group_mode = TL_GEMM_GROUP_K;
    g.groups = static_cast<uint32_t>(chain.size());
    g.beta = 0.0f;
    g.bias = first.gemm.bias;
    g.addend = first.gemm.addend;
    merged.t[3] = first.t[3];
    merged.t[5] = first.t[5];
    merged.t[0] = first.t[0];
    merged.t[1] = first.t[1];
    g.a = first.gemm.a;
    g.b = first.gemm.b;
    merged.group_refs.clear();
    for (size_t k = 0; k < chain.size(); ++k) {
      const Op &y = p[chain[k]];
      g.a_group[k] = y.gemm.a;
      g.b_group[k] = y.gemm.b;
      if (k > 0) {
        merged.group_refs.push_back(y.t[0]);
        merged.group_refs.push_back(y.t[1]);
      }
    }
    for (size_t k = 0; k + 1 < chain.size(); ++k) p[chain[k]].dead = true;
    p[last] = std::move(merged);
    folded += chain.size() - 1;
  }
  return folded;
}

// --------------------------------------------------------- copy forwarding
bool elementwise(Kind k) {
  return k == Kind::Binary || k == Kind::Scalar || k == Kind::Unary || k == Kind::Copy ||
         k == Kind::GeluBwd;
}

// Points every read of allocation `from` in `op` at `to` (same element
// count; the op keeps its own view of the shape).
void retarget_reads(Op &op, const TRef &from, const TRef &to) {
  auto swap = [&](TRef &r) {
    if (r.p && r.id == from.id) {
      r.p = to.p;
      r.id = to.id;
    }
  };
  auto &t = op.t;
  switch (op.kind) {
    case Kind::Binary: case Kind::Xent: case Kind::Gather: case Kind::GeluBwd:
      swap(t[0]); swap(t[1]); break;
    case Kind::SoftmaxBwd: swap(t[0]); swap(t[1]); swap(t[3]); break;
    case Kind::Softmax: swap(t[0]); swap(t[2]); swap(t[3]); break;
    case Kind::XentBwd: swap(t[0]); swap(t[1]); swap(t[3]); break;
    case Kind::Scatter: swap(t[0]); swap(t[1]); swap(t[2]); break;
    case Kind::Clip: swap(t[0]); swap(t[1]); break;
    case Kind::RmsNormBwd: swap(t[0]); swap(t[1]); swap(t[2]); swap(t[4]); break;
    case Kind::DevCopy: swap(t[1]); break;
    case Kind::Gemm:
      swap(t[0]); swap(t[1]); swap(t[3]); swap(t[5]);
      op.gemm.a = static_cast<const float *>(t[0].p);
      op.gemm.b = static_cast<const float *>(t[1].p);
      op.gemm.bias = t[3].p ? t[3].f() : nullptr;
      op.gemm.addend = t[5].p ? t[5].f() : nullptr;
      break;
    default: swap(t[0]); break;  // single-input kinds
  }
}

// Op i left in T a value equal to the current value of S.  When every later
// read of that value can read S instead (S unchanged until the last such
// read; T's value then ends: released, fully overwritten, or window-local),
// retargets those reads to S and returns true; otherwise changes nothing.
bool forward_value(std::vector<Op> &p, size_t i, const TRef &T, const TRef &S) {
  std::vector<size_t> readers;
  bool ended = false, s_changed = false;
  for (size_t j = i + 1; j < p.size() && !ended; ++j) {
    const Op &op = p[j];
    if (op.dead) continue;
    if (op.kind == Kind::Release) {
      if (op.t[0].id == T.id) ended = true;
      else if (op.t[0].id == S.id) s_changed = true;
      continue;
    }
    if (op.kind == Kind::MultiAdamW || op.kind == Kind::AllReduce) {
      for (const auto &sl : op.multi)
        for (const TRef *r : {&sl.param, &sl.grad, &sl.out, &sl.m1, &sl.m2})
          if (r->id == T.id || r->id == S.id) return false;
      continue;
    }
    const Access a = access(op);
    const bool rT = reads(a, T.id), wT = writes(a, T.id), wS = writes(a, S.id);
    if (rT) {
      if (s_changed) return false;
      if (op.kind == Kind::Gemm && op.gemm.beta != 0.0f && op.t[2].id == T.id) return false;
      if (op.kind == Kind::HostWrite || op.kind == Kind::Fill || op.kind == Kind::DevCopy)
        return false;  // byte views of whole blocks
      if (wS && !elementwise(op.kind)) return false;  // would read S while writing it
      readers.push_back(j);
    }
    if (wT) {
      if (!full_write(op)) return false;
      ended = true;  // T's forwarded value ends here
    }
    if (wS) s_changed = true;
  }
  if (!ended && !(g_live && g_live->window_local(T.id))) return false;
  for (size_t j : readers) retarget_reads(p[j], T, S);
  return true;
}

// copy(S -> T) whose destination value can be read from S: the copy goes.
// This removes the executor's reshape copies (split_last_dim /
// merge_last_dims, execute.h:384-401, copies in the Metal runtime,
// runtime.cpp:571-593) and identity sum_to_shape copies
// (runtime.cpp:692-698).
uint64_t forward_copies(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t i = 0; i < p.size(); ++i) {
    Op &cp = p[i];
    if (cp.dead || cp.kind != Kind::Copy) continue;
    const TRef S = cp.t[0], T = cp.t[1];
    if (!S.p || !T.p || S.id == T.id || S.numel() != T.numel()) continue;
    if (!forward_value(p, i, T, S)) continue;
    cp.dead = true;
    ++folded;
  }
  return folded;
}

// Output slot of the ops whose single result may be redirected (-1: none).
int output_slot(const Op &op) {
  switch (op.kind) {
    case Kind::Scalar: case Kind::Unary: case Kind::Copy: case Kind::Reduce: case Kind::Argmax:
    case Kind::Transpose: case Kind::Softmax: case Kind::Rms: case Kind::RmsNorm:
      return 1;
    case Kind::Binary: case Kind::Xent: case Kind::XentBwd: case Kind::Gather: case Kind::Clip:
    case Kind::GeluBwd: case Kind::SoftmaxBwd: case Kind::Gemm:
      return 2;
    case Kind::Scatter: case Kind::RmsNormBwd:
      return 3;
    default:
      return -1;
  }
}

// copy(S -> G) where S was just produced for the copy: the producer writes G
// itself and the copy goes.  The executor accumulates every first gradient
// contribution by copying the freshly computed term into the gradient
// buffer (include/passes/context.h accumulate_grad); the weight-gradient
// product and bias-gradient sum now land in the gradient buffer directly.
uint64_t forward_producers(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t c = 0; c < p.size(); ++c) {
    Op &cp = p[c];
    if (cp.dead || cp.kind != Kind::Copy) continue;
    const TRef S = cp.t[0], G = cp.t[1];
    if (!S.p || !G.p || S.id == G.id || S.numel() != G.numel()) continue;
    // the producer: latest live op before the copy that touches S or G
    size_t x = kNone;
    for (size_t k = c; k-- > 0;) {
      const Op &op = p[k];
      if (op.dead) continue;
      if (op.kind == Kind::Release) {
        if (op.t[0].id == S.id || op.t[0].id == G.id) break;
        continue;
      }
      if (op.kind == Kind::MultiAdamW || op.kind == Kind::AllReduce) break;
      const Access a = access(op);
      if (reads(a, G.id) || writes(a, G.id) || reads(a, S.id)) break;
      if (writes(a, S.id)) {
        x = k;
        break;
      }
    }
    if (x == kNone) continue;
    Op &prod = p[x];
    const int slot = output_slot(prod);
    if (slot < 0 || prod.t[slot].id != S.id || !full_write(prod)) continue;
    if (prod.kind == Kind::Gemm && prod.gemm.beta != 0.0f) continue;
    if (!dead_after(p, c, S.id)) continue;
    prod.t[slot].p = G.p;
    prod.t[slot].id = G.id;
    if (prod.kind == Kind::Gemm) prod.gemm.c = G.f();
    cp.dead = true;
    ++folded;
  }
  return folded;
}

// Common subexpressions.  Reverse-mode rules embed the upstream gradient
// expression in every operand's gradient (include/passes/autograd.h), so
// the executor evaluates a shared upstream gradient once per path that
// uses it (attention's score gradient for both dQ and dK, the output
// projection's input gradient for each of dQ, dK, dV).  An op that repeats
// an earlier op (same kind and parameters, same input buffers holding the
// same values) is dropped when its result can be read from the earlier
// op's output instead.  All kernels are deterministic, so the values read
// are bit-identical to the recomputed ones.
bool cse_candidate(const Op &op, const Access &a) {
  switch (op.kind) {
    case Kind::Binary: case Kind::Scalar: case Kind::Unary: case Kind::Copy: case Kind::Reduce:
    case Kind::Argmax: case Kind::Transpose: case Kind::Softmax: case Kind::Rms:
    case Kind::RmsNorm: case Kind::Xent: case Kind::XentBwd: case Kind::Gather:
    case Kind::Scatter: case Kind::GeluBwd: case Kind::SoftmaxBwd: case Kind::RmsNormBwd:
      break;
    case Kind::Gemm:
      if (op.gemm.beta != 0.0f || op.gemm.gelu_out) return false;
      break;
    default:
      return false;
  }
  return a.nw == 1 && !reads(a, a.w[0]);
}

uint64_t eliminate_common(std::vector<Op> &p) {
  std::unordered_map<uint64_t, uint32_t> version;
  struct Seen {
    size_t op;
    TRef out;
    uint32_t out_version;
  };
  std::unordered_map<std::string, Seen> table;
  auto bump = [&](uint64_t id) { ++version[id]; };
  auto put = [](std::string &k, const void *d, size_t n) {
    k.append(static_cast<const char *>(d), n);
  };
  uint64_t folded = 0;
  std::string key;
  for (size_t i = 0; i < p.size(); ++i) {
    Op &op = p[i];
    if (op.dead) continue;
    if (op.kind == Kind::Release) {
      bump(op.t[0].id);
      continue;
    }
    if (op.kind == Kind::MultiAdamW || op.kind == Kind::AllReduce) {
      for (const auto &sl : op.multi)
        for (const TRef *r : {&sl.param, &sl.grad, &sl.out, &sl.m1, &sl.m2}) bump(r->id);
      continue;
    }
    const Access a = access(op);
    if (!cse_candidate(op, a)) {
      for (int w = 0; w < a.nw; ++w) bump(a.w[w]);
      continue;
    }
    const uint64_t out_id = a.w[0];
    key.clear();
    put(key, &op.kind, sizeof(op.kind));
    put(key, &op.code, sizeof(op.code));
    put(key, &op.f0, sizeof(op.f0));
    put(key, &op.f1, sizeof(op.f1));
    put(key, &op.i0, sizeof(op.i0));
    put(key, &op.i1, sizeof(op.i1));
    put(key, &op.u0, sizeof(op.u0));
    put(key, &op.n, sizeof(op.n));
    int out_slot = -1;
    for (int k = 0; k < 9; ++k) {
      const TRef &r = op.t[k];
      const uint8_t present = r.p ? 1 : 0;
      put(key, &present, 1);
      if (!r.p) continue;
      put(key, &r.rank, 1);
      put(key, r.shape, r.rank * sizeof(uint32_t));
      if (r.id == out_id) {
        out_slot = k;
        continue;
      }
      const uint32_t v = version[r.id];
      put(key, &r.id, sizeof(r.id));
      put(key, &v, sizeof(v));
    }
    if (op.kind == Kind::Gemm) {
      tl_gemm_desc g = op.gemm;  // pointers are covered by the operands above
      g.a = g.b = nullptr;
      g.c = g.gelu_out = nullptr;
      g.bias = nullptr;
      g.workspace = nullptr;
      g.workspace_bytes = 0;
      put(key, &g, sizeof(g));
    }
    auto it = table.find(key);
    if (it != table.end() && version[it->second.out.id] == it->second.out_version &&
        out_slot >= 0) {
      const TRef &S = it->second.out;
      const TRef &T = op.t[out_slot];
      if (S.id == T.id || forward_value(p, i, T, S)) {
        op.dead = true;  // T is not written: its readers now read S
        ++folded;
        continue;
      }
    }
    bump(out_id);
    if (out_slot >= 0) table[key] = Seen{i, op.t[out_slot], version[out_id]};
  }
  return folded;
}

// A sum over every dim but the last of a tensor whose rows are 16-byte
// multiples: the bias gradient that Runtime::sum_to_shape computes for a
// linear layer (include/nn/layer.h:16-39, bias [1, C]: [.., C] -> [1, C]).
bool column_sum(const Op &op) {
  if (op.dead || op.kind != Kind::Reduce || op.code != TL_REDUCE_SUM || !op.group_refs.empty())
    return false;
  const TRef &x = op.t[0], &y = op.t[1];
  return x.p && y.p && x.rank >= 2 && y.numel() == x.last() && x.numel() > x.last() &&
         x.last() % 4 == 0;
}

bool same_shape(const TRef &a, const TRef &b) {
  if (a.rank != b.rank) return false;
  for (int d = 0; d < a.rank; ++d)
    if (a.shape[d] != b.shape[d]) return false;
  return true;
}

// Column sums of same-shape tensors recorded close together (the bias
// gradients of the query, key and value projections after the attention
// backward) run as one grouped launch (tl_reduce_group, each result
// bit-identical to its own reduction) at the last member's position: every
// earlier member's input must be unchanged and its output untouched (not
// read, written or released) until then, and no member may read or write
// another's output.
uint64_t group_column_sums(std::vector<Op> &p) {
  uint64_t folded = 0;
  for (size_t i = 0; i < p.size(); ++i) {
    if (!column_sum(p[i])) continue;
    std::vector<size_t> members{i};
    for (size_t j = i + 1;
         j < p.size() && j < i + 128 && members.size() < TL_REDUCE_MAX_GROUPS; ++j) {
      const Op &y = p[j];
      if (y.kind == Kind::MultiAdamW || y.kind == Kind::AllReduce) break;
      if (!column_sum(y) || !same_shape(y.t[0], p[i].t[0]) || !same_shape(y.t[1], p[i].t[1]))
        continue;
      bool ok = true;
      for (size_t k : members) {
        const Op &z = p[k];
        if (y.t[1].id == z.t[0].id || y.t[1].id == z.t[1].id || y.t[0].id == z.t[1].id ||
            !unchanged_between(p, k, j, z.t[0].id) || !untouched_between(p, k, j, z.t[1].id))
          ok = false;
      }
      if (ok) members.push_back(j);
    }
    if (members.size() < 2) continue;
    const size_t at = members.back();
    Op grouped = p[members.front()];
    grouped.group_refs.clear();
    for (size_t k = 1; k < members.size(); ++k) {
      grouped.group_refs.push_back(p[members[k]].t[0]);
      grouped.group_refs.push_back(p[members[k]].t[1]);
    }
    grouped.workspace = members.size() * p[members.front()].workspace;
    for (size_t k : members) p[k].dead = true;
    p[at] = std::move(grouped);
    folded += members.size() - 1;
  }
  return folded;
}

bool is_opt(Kind k) {
  return k == Kind::SqNorm || k == Kind::Clip || k == Kind::AdamW;
}

// `Compiled::step(max_norm)` (include/passes/compile.h:236-258) records
//   SqNorm(g_i, n) for every gradient, Clip(g_i, n, c, g_i) for every
//   gradient, then AdamW(p_i, g_i, p_i, m1_i, m2_i, b1, b2, decay, lr, eps, t_i)
// and `Compiled::step()` records the AdamW calls alone.  Both become one
// MultiAdamW op (two launches: deterministic norm, then clip + update).
uint64_t fuse_step(std::vector<Op> &p) {
  std::vector<size_t> norms, clips, adams;
  size_t first = p.size(), last = 0;
  for (size_t i = 0; i < p.size(); ++i) {
    const Op &op = p[i];
    if (op.dead) continue;
    if (op.kind == Kind::SqNorm) norms.push_back(i);
    else if (op.kind == Kind::Clip) clips.push_back(i);
    else if (op.kind == Kind::AdamW) adams.push_back(i);
    else continue;
    first = std::min(first, i);
    last = std::max(last, i);
  }
  if (adams.empty()) return 0;
  // strict phase order and nothing but storage initialisation in between
  if (!norms.empty() && (clips.empty() || norms.back() > clips.front())) return 0;
  if (!clips.empty() && clips.back() > adams.front()) return 0;
  if (norms.empty() != clips.empty()) return 0;
  for (size_t i = first; i <= last; ++i) {
    const Op &op = p[i];
    if (op.dead || is_opt(op.kind)) continue;
    if (op.kind != Kind::Fill && op.kind != Kind::Release) return 0;
  }
  const Op &a0 = p[adams.front()];
  std::unordered_set<void *> grads;
  for (size_t i : adams) {
    const Op &op = p[i];
    for (int j = 5; j <= 8; ++j)
      if (op.t[j].p != a0.t[j].p) return 0;
    if (op.f0 != a0.f0) return 0;
    if (!grads.insert(op.t[1].p).second) return 0;  // each gradient updated once
  }
  void *sq = nullptr;
  float max_norm = 0.0f;
  if (!clips.empty()) {
    sq = p[norms.front()].t[1].p;
    max_norm = p[clips.front()].f0;
    std::unordered_set<void *> normed, clipped;
    for (size_t i : norms) {
      if (p[i].t[1].p != sq || !normed.insert(p[i].t[0].p).second) return 0;
    }
    for (size_t i : clips) {
      const Op &op = p[i];
      if (op.t[1].p != sq || op.f0 != max_norm || op.t[0].p != op.t[2].p) return 0;
      if (!clipped.insert(op.t[0].p).second) return 0;
    }
    if (normed != grads || clipped != grads) return 0;
  }
  Op fused;
  fused.kind = Kind::MultiAdamW;
  if (sq) fused.t[0] = p[norms.front()].t[1];
  for (int j = 5; j <= 8; ++j) fused.t[j] = a0.t[j];
  fused.f0 = max_norm;
  fused.f1 = a0.f0;
  uint64_t chunks = 0;
  for (size_t i : adams) {
    const Op &op = p[i];
    MultiSlot s;
    s.param = op.t[0];
    s.grad = op.t[1];
    s.out = op.t[2];
    s.m1 = op.t[3];
    s.m2 = op.t[4];
    s.step = op.u0;
    chunks += (op.t[0].numel() + TL_OPT_CHUNK - 1) / TL_OPT_CHUNK;
    fused.multi.push_back(s);
  }
  fused.workspace = tl_multi_clip_adamw_workspace_size(static_cast<uint32_t>(chunks));
  const uint64_t folded = norms.size() + clips.size() + adams.size() - 1;
  for (size_t i : norms) p[i].dead = true;
  for (size_t i : clips) p[i].dead = true;
  for (size_t i : adams) p[i].dead = true;
  p[adams.back()] = std::move(fused);
  return folded;
}

}  // namespace

void add_gradient_allreduce(std::vector<Op> &prog) {
  size_t first = prog.size();
  Op ar;
  ar.kind = Kind::AllReduce;
  std::unordered_set<void *> seen;
  for (size_t i = 0; i < prog.size(); ++i) {
    const Op &op = prog[i];
    if (op.dead) continue;
    const bool opt = op.kind == Kind::SqNorm || op.kind == Kind::Clip ||
                     op.kind == Kind::AdamW || op.kind == Kind::MultiAdamW;
    if (!opt) continue;
    first = std::min(first, i);
    if (op.kind == Kind::AdamW && seen.insert(op.t[1].p).second) {
      MultiSlot s{};
      s.grad = op.t[1];
      ar.multi.push_back(s);
    }
    if (op.kind == Kind::MultiAdamW)
      for (const MultiSlot &m : op.multi)
        if (seen.insert(m.grad.p).second) {
          MultiSlot s{};
          s.grad = m.grad;
          ar.multi.push_back(s);
        }
  }
  if (ar.multi.empty()) return;
  prog.insert(prog.begin() + static_cast<std::ptrdiff_t>(first), std::move(ar));
}

// One causal-mask check per mask per program: the first attention forward
// (fused or flash) that reads a mask through a runtime word checks it
// (Attention: u0 bit 0; FlashFwd: code bit 0), later ones read the word,
// until an op writes the mask.
void assign_mask_checks(std::vector<Op> &p) {
  std::unordered_set<uint64_t> checked;
  for (Op &op : p) {
    if (op.dead) continue;
    const bool fused = op.kind == Kind::Attention && op.code == TL_ATTN_FORWARD &&
                       op.attn.mask_flag != nullptr;
    const bool flash = op.kind == Kind::FlashFwd && op.flash.mask_flag != nullptr;
    if (fused || flash) {
      const bool first = checked.insert(op.t[4].id).second;
      if (fused) op.u0 = first ? 1u : 0u;
      else op.code = first ? 1 : 0;
      continue;
    }
    if (checked.empty()) continue;
    const Access a = access(op);
    for (int w = 0; w < a.nw; ++w) checked.erase(a.w[w]);
    if (op.kind == Kind::Release && op.t[0].p) checked.erase(op.t[0].id);
  }
}

uint64_t optimize(std::vector<Op> &prog, void *comm, const Liveness *live, FlashState *flash) {
  g_live = live;
  g_flash = flash && flash->enabled() ? flash : nullptr;
  uint64_t folded = 0;
  // Two rounds: fusion exposes further repeats (a repeated product whose
  // transposed operand lived in a released temporary reads the weight itself
  // once the transpose is folded), and removing repeats exposes fusions
  // whose intermediate had several (repeated) readers.
  for (int round = 0; round < 2; ++round) {
    folded += eliminate_common(prog);
    folded += forward_copies(prog);
    folded += forward_producers(prog);
    folded += fuse_weight_gradient(prog);
    folded += fold_transposes(prog);
    folded += fuse_gemm_epilogues(prog);
    folded += fuse_softmax_backward(prog);
    folded += fuse_rmsnorm_backward(prog);
    folded += fuse_pointwise_backward(prog);
  }
  // Folds that change an op's inputs (an added operand, a divisor, strided
  // operands) come last so they cannot hide a repeat from the
  // common-subexpression pass.
  folded += fold_head_transposes(prog);
  folded += fold_head_transposes(prog);  // a second transpose of the same product
  folded += fuse_gemm_accumulate(prog);
  folded += fuse_row_backward_tails(prog);
  folded += fuse_gemm_gelu_backward(prog);
  folded += fuse_score_softmax(prog);
  if (g_flash) {
    folded += fuse_flash_forward(prog);
    folded += fuse_flash_backward(prog);
  }
  folded += fuse_attention(prog);
  folded += fuse_head_split_store(prog);
  folded += group_summed_products(prog);
  folded += group_shared_input(prog);
  folded += group_column_sums(prog);
  folded += fuse_step(prog);
  if (comm) add_gradient_allreduce(prog);
  if (g_flash) resolve_flash(prog);
  assign_mask_checks(prog);
  g_live = nullptr;
  g_flash = nullptr;
  return folded;
}

}  // namespace cuda::internal

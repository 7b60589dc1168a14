// CPU test of the program optimiser (templit_b200/runtime/optimize.cpp):
// builds recorded programs by hand, in the shapes the typed executor emits
// them (include/passes/execute.h of JTPuffer/TempLit), and checks which
// rewrites happen - and that none happens when an intermediate is still
// observable.  Needs no GPU: nothing is launched.
#include "optimize.h"
#include "program.h"

#include <cstdio>
#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

using namespace cuda::internal;

namespace {

struct Failure : std::runtime_error {
  using std::runtime_error::runtime_error;
};
void require(bool ok, const std::string &what) {
  if (!ok) throw Failure(what);
}

uint64_t g_id = 1;
uintptr_t g_addr = 0x10000;

TRef tensor(std::vector<uint32_t> shape) {
  TRef t;
  t.p = reinterpret_cast<void *>(g_addr);
  g_addr += 0x100000;
  t.id = g_id++;
  t.rank = static_cast<uint8_t>(shape.size());
  for (size_t i = 0; i < shape.size(); ++i) t.shape[i] = shape[i];
  return t;
}

Op op(Kind k) {
  Op o;
  o.kind = k;
  return o;
}
Op release(const TRef &t) {
  Op o = op(Kind::Release);
  o.t[0] = t;
  o.n = t.numel() * 4;  // the block's bytes, as the runtime records them
  return o;
}
Op binary(int code, const TRef &a, const TRef &b, const TRef &c) {
  Op o = op(Kind::Binary);
  o.code = code;
  o.t[0] = a;
  o.t[1] = b;
  o.t[2] = c;
  return o;
}
Op gemm(const TRef &a, const TRef &b, const TRef &c, uint32_t m, uint32_t n, uint32_t k,
        uint32_t batch = 0) {
  Op o = op(Kind::Gemm);
  o.t[0] = a;
  o.t[1] = b;
  o.t[2] = c;
  o.gemm.a = static_cast<const float *>(a.p);
  o.gemm.b = static_cast<const float *>(b.p);
  o.gemm.c = c.f();
  o.gemm.m = m;
  o.gemm.n = n;
  o.gemm.k = k;
  if (batch) {
    o.gemm.batch_rank = 1;
    o.gemm.batch_shape[0] = batch;
    o.gemm.a_batch_stride[0] = uint64_t(m) * k;
    o.gemm.b_batch_stride[0] = uint64_t(k) * n;
    o.gemm.c_batch_stride[0] = uint64_t(m) * n;
  }
  return o;
}
Op transpose(const TRef &a, const TRef &out) {
  Op o = op(Kind::Transpose);
  o.t[0] = a;
  o.t[1] = out;
  o.i0 = a.rank - 2;
  o.i1 = a.rank - 1;
  return o;
}
Op reduce(const TRef &a, const TRef &out) {
  Op o = op(Kind::Reduce);
  o.code = TL_REDUCE_SUM;
  o.t[0] = a;
  o.t[1] = out;
  return o;
}
std::vector<const Op *> live(const std::vector<Op> &p) {
  std::vector<const Op *> v;
  for (const Op &o : p)
    if (!o.dead && o.kind != Kind::Release) v.push_back(&o);
  return v;
}

void linear_bias_gelu() {
  auto x = tensor({12288, 384}), w = tensor({384, 1536}), b = tensor({1, 1536});
  auto c = tensor({12288, 1536}), h = tensor({12288, 1536});
  std::vector<Op> p = {gemm(x, w, c, 12288, 1536, 384), binary(TL_ADD, c, b, c)};
  Op g = op(Kind::Unary);
  g.code = TL_GELU;
  g.t[0] = c;
  g.t[1] = h;
  p.push_back(g);
  require(optimize(p, nullptr) == 2, "two ops folded");
  auto v = live(p);
  require(v.size() == 1 && v[0]->gemm.bias == b.p && v[0]->gemm.gelu_out == h.p,
          "bias and GELU in the GEMM epilogue");
}

void weight_gradient_tn() {
  auto x = tensor({64, 192, 384}), g = tensor({64, 192, 1536});
  auto xt = tensor({64, 384, 192}), prod = tensor({64, 384, 1536}), dw = tensor({384, 1536});
  std::vector<Op> p = {transpose(x, xt), gemm(xt, g, prod, 384, 1536, 192, 64), reduce(prod, dw),
                       release(prod), release(xt)};
  require(optimize(p, nullptr) == 2, "transpose and product folded");
  auto v = live(p);
  require(v.size() == 1 && v[0]->kind == Kind::Gemm, "one GEMM");
  const auto &d = v[0]->gemm;
  require(d.trans_a == 1 && d.k == 64 * 192 && d.m == 384 && d.n == 1536 && d.batch_rank == 0 &&
              d.a == static_cast<const float *>(x.p) && d.c == dw.f(),
          "TN product with K = batch * T");
}

void weight_gradient_observable_product_kept() {
  auto x = tensor({8, 16, 32}), g = tensor({8, 16, 24});
  auto xt = tensor({8, 32, 16}), prod = tensor({8, 32, 24}), dw = tensor({32, 24});
  // the product is never released: it is observable after the program
  std::vector<Op> p = {transpose(x, xt), gemm(xt, g, prod, 32, 24, 16, 8), reduce(prod, dw),
                       release(xt)};
  optimize(p, nullptr);
  auto v = live(p);
  require(v.size() == 2 && v[0]->kind == Kind::Gemm && v[0]->gemm.trans_a == 1 &&
              v[1]->kind == Kind::Reduce,
          "only the transpose folds; product and reduction stay");
}

void transpose_into_b() {
  auto g = tensor({12288, 2048}), w = tensor({384, 2048}), wt = tensor({2048, 384});
  auto dx = tensor({12288, 384});
  std::vector<Op> p = {transpose(w, wt), gemm(g, wt, dx, 12288, 384, 2048), release(wt)};
  require(optimize(p, nullptr) == 1, "folded");
  auto v = live(p);
  require(v.size() == 1 && v[0]->gemm.trans_b == 1 && v[0]->gemm.b == static_cast<const float *>(w.p),
          "NT product on the stored weight");
}

void transpose_kept_when_read_later() {
  auto a = tensor({64, 6, 192, 64}), at = tensor({64, 6, 64, 192}), q = tensor({64, 6, 192, 64});
  auto s = tensor({64, 6, 192, 192});
  Op mm = gemm(q, at, s, 192, 192, 64, 384);
  Op later = op(Kind::Copy);
  later.t[0] = at;
  later.t[1] = tensor({64, 6, 64, 192});
  std::vector<Op> p = {transpose(a, at), mm, later};
  require(optimize(p, nullptr) == 0, "K^T saved for backward: no fold");
}

void softmax_backward() {
  auto g = tensor({64, 6, 192, 192}), y = tensor({64, 6, 192, 192}), d = tensor({64, 6, 192, 192});
  auto r = tensor({64, 6, 192, 1});
  std::vector<Op> p = {binary(TL_MUL, g, y, d), reduce(d, r), binary(TL_SUB, g, r, d),
                       binary(TL_MUL, y, d, d), release(r)};
  require(optimize(p, nullptr) == 3, "softmax derivative fused");
  auto v = live(p);
  require(v.size() == 1 && v[0]->kind == Kind::SoftmaxBwd && v[0]->t[2].id == d.id, "one row kernel");
}

void rmsnorm_backward() {
  auto x = tensor({64, 192, 384}), g = tensor({64, 192, 384}), y = tensor({64, 192, 384});
  auto d = tensor({64, 192, 384}), s = tensor({64, 192, 1}), m = tensor({64, 192, 1});
  Op rms = op(Kind::Rms);
  rms.t[0] = x;
  rms.t[1] = s;
  Op dv = op(Kind::Scalar);
  dv.code = TL_SCALAR_DIV;
  dv.t[0] = m;
  dv.t[1] = m;
  dv.f0 = 384.0f;
  std::vector<Op> p = {rms,
                       binary(TL_MUL, g, y, d),
                       reduce(d, m),
                       dv,
                       binary(TL_MUL, y, m, d),
                       binary(TL_SUB, g, d, d),
                       binary(TL_DIV, d, s, d),
                       release(m),
                       release(s)};
  require(optimize(p, nullptr) == 6, "RMSNorm derivative fused");
  auto v = live(p);
  require(v.size() == 1 && v[0]->kind == Kind::RmsNormBwd, "one row kernel");
}

void xent_and_gelu_backward() {
  auto z = tensor({64, 192, 2048}), t = tensor({64, 192}), dz = tensor({64, 192, 2048});
  auto root = tensor({64, 192, 1}), out = tensor({64, 192, 2048});
  Op xb = op(Kind::XentBwd);
  xb.t[0] = z;
  xb.t[1] = t;
  xb.t[2] = dz;
  auto x = tensor({64, 192, 1536}), gd = tensor({64, 192, 1536}), g = tensor({64, 192, 1536});
  auto o2 = tensor({64, 192, 1536});
  Op gdo = op(Kind::Unary);
  gdo.code = TL_GELU_DERIVATIVE;
  gdo.t[0] = x;
  gdo.t[1] = gd;
  std::vector<Op> p = {xb, binary(TL_MUL, root, dz, out), release(dz),
                       gdo, binary(TL_MUL, gd, g, o2), release(gd)};
  require(optimize(p, nullptr) == 2, "both fused");
  auto v = live(p);
  require(v.size() == 2 && v[0]->kind == Kind::XentBwd && v[0]->t[3].id == root.id &&
              v[0]->t[2].id == out.id && v[1]->kind == Kind::GeluBwd && v[1]->t[2].id == o2.id,
          "row-scaled CE backward and GELU backward");
}

void reused_address_is_not_confused() {
  // r is released, then a new allocation lands at the same address: the
  // optimiser must see two different values.
  auto g = tensor({8, 16}), y = tensor({8, 16}), d = tensor({8, 16}), r = tensor({8, 1});
  TRef r2 = r;
  r2.id = g_id++;  // same address, new allocation
  Op use = op(Kind::Copy);
  use.t[0] = r2;
  use.t[1] = tensor({8, 1});
  std::vector<Op> p = {binary(TL_MUL, g, y, d), reduce(d, r), binary(TL_SUB, g, r, d),
                       binary(TL_MUL, y, d, d), release(r), use};
  require(optimize(p, nullptr) == 3, "fused although the address is reused");
}

void fused_step() {
  std::vector<Op> p;
  auto sq = tensor({1});
  auto b1 = tensor({1, 1}), b2 = tensor({1, 1}), dc = tensor({1, 1}), lr = tensor({1, 1});
  std::vector<TRef> ps, gs;
  for (int i = 0; i < 3; ++i) {
    ps.push_back(tensor({384, 384}));
    gs.push_back(tensor({384, 384}));
  }
  for (int i = 0; i < 3; ++i) {
    Op n = op(Kind::SqNorm);
    n.t[0] = gs[i];
    n.t[1] = sq;
    p.push_back(n);
  }
  for (int i = 0; i < 3; ++i) {
    Op c = op(Kind::Clip);
    c.t[0] = gs[i];
    c.t[1] = sq;
    c.t[2] = gs[i];
    c.f0 = 1.0f;
    p.push_back(c);
  }
  for (int i = 0; i < 3; ++i) {
    Op a = op(Kind::AdamW);
    a.t[0] = ps[i];
    a.t[1] = gs[i];
    a.t[2] = ps[i];
    a.t[3] = tensor({384, 384});
    a.t[4] = tensor({384, 384});
    a.t[5] = b1;
    a.t[6] = b2;
    a.t[7] = dc;
    a.t[8] = lr;
    a.f0 = 1e-8f;
    a.u0 = 7;
    p.push_back(a);
  }
  require(optimize(p, nullptr) == 8, "9 optimiser ops -> 1");
  auto v = live(p);
  require(v.size() == 1 && v[0]->kind == Kind::MultiAdamW && v[0]->multi.size() == 3 &&
              v[0]->f0 == 1.0f && v[0]->multi[0].step == 7,
          "fused clip + AdamW");
  add_gradient_allreduce(p);
  v = live(p);
  require(v.size() == 2 && v[0]->kind == Kind::AllReduce && v[0]->multi.size() == 3,
          "data-parallel all-reduce ahead of the optimiser");
}


Op copy(const TRef &src, const TRef &dst) {
  Op o = op(Kind::Copy);
  o.t[0] = src;
  o.t[1] = dst;
  return o;
}

struct FixedLiveness : Liveness {
  std::vector<uint64_t> ids;
  bool window_local(uint64_t id) const override {
    for (uint64_t i : ids)
      if (i == id) return true;
    return false;
  }
};

// reshape copy (merge_last_dims) feeding one GEMM, then released: the GEMM
// reads the source and the copy goes
void copy_forwarded_to_reader() {
  auto s = tensor({64, 192, 384}), t = tensor({12288, 384}), w = tensor({384, 1536});
  auto c = tensor({12288, 1536});
  std::vector<Op> p = {copy(s, t), gemm(t, w, c, 12288, 1536, 384), release(t)};
  require(optimize(p, nullptr) == 1, "copy folded");
  auto v = live(p);
  require(v.size() == 1 && v[0]->t[0].id == s.id && v[0]->gemm.a == s.p,
          "GEMM reads the copy's source");
}

// the copy's destination outlives the program: kept, unless window-local
void copy_kept_when_observable() {
  auto s = tensor({4096}), t = tensor({4096}), u = tensor({4096});
  std::vector<Op> p = {copy(s, t), binary(TL_MUL, t, t, u)};
  require(optimize(p, nullptr) == 0, "observable copy kept");
  std::vector<Op> q = {copy(s, t), binary(TL_MUL, t, t, u)};
  FixedLiveness live_t;
  live_t.ids = {t.id};
  require(optimize(q, nullptr, &live_t) == 1, "window-local copy folded");
  auto v = live(q);
  require(v.size() == 1 && v[0]->t[0].id == s.id && v[0]->t[1].id == s.id, "both operands");
}

// the source changes before the destination is read: kept
void copy_kept_when_source_changes() {
  auto s = tensor({4096}), t = tensor({4096}), u = tensor({4096});
  std::vector<Op> p = {copy(s, t), binary(TL_ADD, u, u, s), binary(TL_MUL, t, t, u), release(t)};
  require(optimize(p, nullptr) == 0, "copy kept: source overwritten before the read");
  // a partial Storage write of the destination does not end the copied value
  auto a = tensor({4096}), b = tensor({4096}), c = tensor({4096});
  Op fill = op(Kind::Fill);
  fill.t[0] = b;
  fill.t[0].shape[0] = 4096 * 4;  // byte view of the block
  fill.n = 16;
  std::vector<Op> q = {copy(a, b), fill, binary(TL_MUL, b, b, c), release(b)};
  require(optimize(q, nullptr) == 0, "copy kept: partial overwrite");
}


// the upstream gradient evaluated once per path (same GEMM, same inputs):
// the second evaluation goes and its reader reads the first result
void common_gemm_evaluated_once() {
  auto g = tensor({12288, 384}), w = tensor({384, 384}), d1 = tensor({12288, 384});
  auto d2 = tensor({12288, 384}), x = tensor({12288, 384}), y = tensor({12288, 384});
  std::vector<Op> p = {gemm(g, w, d1, 12288, 384, 384), binary(TL_MUL, d1, d1, x),
                       gemm(g, w, d2, 12288, 384, 384), binary(TL_ADD, d2, x, y),
                       release(d2), release(d1)};
  require(optimize(p, nullptr) == 1, "second product folded");
  auto v = live(p);
  require(v.size() == 3 && v[2]->kind == Kind::Binary && v[2]->t[0].id == d1.id,
          "reader of the repeat reads the first product");
}

// an input changes between the two evaluations: both stay
void common_kept_when_input_changes() {
  auto g = tensor({4096}), d1 = tensor({4096}), d2 = tensor({4096}), x = tensor({4096});
  Op u1 = op(Kind::Unary), u2 = op(Kind::Unary);
  u1.code = u2.code = TL_EXP;
  u1.t[0] = u2.t[0] = g;
  u1.t[1] = d1;
  u2.t[1] = d2;
  std::vector<Op> p = {u1, binary(TL_ADD, d1, d1, g), u2, binary(TL_MUL, d2, d1, x),
                       release(d2)};
  require(optimize(p, nullptr) == 0, "input rewritten in between");
  // same buffer rewritten with the value it still holds: the repeat goes
  auto e = tensor({4096}), f = tensor({4096});
  Op v1 = op(Kind::Unary), v2 = op(Kind::Unary);
  v1.code = v2.code = TL_EXP;
  v1.t[0] = v2.t[0] = e;
  v1.t[1] = v2.t[1] = f;
  std::vector<Op> q = {v1, binary(TL_MUL, f, f, x), v2, binary(TL_ADD, f, x, x)};
  require(optimize(q, nullptr) == 1, "repeat into the same buffer folded");
}


// residual add of a product: the add moves into the GEMM epilogue
void residual_add_into_gemm() {
  auto x = tensor({12288, 384}), w = tensor({384, 384}), p0 = tensor({12288, 384});
  auto r = tensor({12288, 384}), o = tensor({12288, 384});
  std::vector<Op> p = {gemm(x, w, p0, 12288, 384, 384), binary(TL_ADD, r, p0, o), release(p0)};
  require(optimize(p, nullptr) == 1, "add folded");
  auto v = live(p);
  require(v.size() == 1 && v[0]->t[2].id == o.id && v[0]->gemm.addend == r.p &&
              v[0]->gemm.beta == 0.0f,
          "product written to the sum with the residual as addend");
  // in place: acc = acc + product
  auto acc = tensor({12288, 384}), p1 = tensor({12288, 384});
  std::vector<Op> q = {gemm(x, w, p1, 12288, 384, 384), binary(TL_ADD, acc, p1, acc),
                       release(p1)};
  require(optimize(q, nullptr) == 1, "accumulate folded");
  auto u = live(q);
  require(u.size() == 1 && u[0]->t[2].id == acc.id && u[0]->gemm.beta == 1.0f &&
              !u[0]->gemm.addend,
          "accumulated in place");
  // the product is read again: kept
  auto p2 = tensor({12288, 384}), o2 = tensor({12288, 384}), z = tensor({12288, 384});
  std::vector<Op> k = {gemm(x, w, p2, 12288, 384, 384), binary(TL_ADD, r, p2, o2),
                       binary(TL_MUL, p2, p2, z), release(p2)};
  require(optimize(k, nullptr) == 0, "product still read: kept");
}

// divide by sqrt(d), add the causal mask, softmax: one softmax op
void attention_scores_into_softmax() {
  auto sc = tensor({64, 6, 192, 192}), d = tensor({1, 1}), s1 = tensor({64, 6, 192, 192});
  auto m = tensor({1, 1, 192, 192}), s2 = tensor({64, 6, 192, 192}), pr = tensor({64, 6, 192, 192});
  Op sm = op(Kind::Softmax);
  sm.t[0] = s2;
  sm.t[1] = pr;
  std::vector<Op> p = {binary(TL_DIV, sc, d, s1), binary(TL_ADD, s1, m, s2), sm, release(s2),
                       release(s1)};
  require(optimize(p, nullptr) == 2, "divide and mask folded");
  auto v = live(p);
  require(v.size() == 1 && v[0]->kind == Kind::Softmax && v[0]->t[0].id == sc.id &&
              v[0]->t[2].id == d.id && v[0]->t[3].id == m.id,
          "softmax reads the raw scores, divisor and mask");
}

// softmax backward then divide; RMSNorm backward then residual add
void row_backward_tails() {
  auto g = tensor({64, 6, 192, 192}), y = tensor({64, 6, 192, 192}), t = tensor({64, 6, 192, 192});
  auto d = tensor({1, 1}), o = tensor({64, 6, 192, 192});
  Op sb = op(Kind::SoftmaxBwd);
  sb.t[0] = g;
  sb.t[1] = y;
  sb.t[2] = t;
  std::vector<Op> p = {sb, binary(TL_DIV, t, d, o), release(t)};
  require(optimize(p, nullptr) == 1, "divide folded");
  auto v = live(p);
  require(v.size() == 1 && v[0]->t[2].id == o.id && v[0]->t[3].id == d.id, "divisor attached");
  auto gr = tensor({12288, 384}), x = tensor({12288, 384}), yn = tensor({12288, 384});
  auto tr = tensor({12288, 384}), a = tensor({12288, 384});
  Op rb = op(Kind::RmsNormBwd);
  rb.t[0] = gr;
  rb.t[1] = x;
  rb.t[2] = yn;
  rb.t[3] = tr;
  std::vector<Op> q = {rb, binary(TL_ADD, a, tr, a), release(tr)};
  require(optimize(q, nullptr) == 1, "residual gradient folded");
  auto u = live(q);
  require(u.size() == 1 && u[0]->t[3].id == a.id && u[0]->t[4].id == a.id, "added in place");
}


// a projection then split_heads (transpose(1, 2) of its [B, T, H, D] view):
// the product stores the [B, H, T, D] layout itself and the transpose goes;
// kept when the projection is read again later
void head_split_store() {
  auto x = tensor({4, 192, 384}), w = tensor({384, 384}), c = tensor({4, 192, 384});
  auto y = tensor({4, 6, 192, 64});
  auto view = [](TRef t) {
    t.rank = 4;
    t.shape[0] = 4;
    t.shape[1] = 192;
    t.shape[2] = 6;
    t.shape[3] = 64;
    return t;
  };
  Op split = transpose(view(c), y);
  split.i0 = 1;
  split.i1 = 2;
  std::vector<Op> p = {gemm(x, w, c, 768, 384, 384), split, release(c)};
  require(optimize(p, nullptr) == 1, "transpose folded into the store");
  auto l = live(p);
  require(l.size() == 1 && l[0]->t[2].id == y.id && l[0]->gemm.c == y.f() &&
              l[0]->gemm.c_heads == 6 && l[0]->gemm.c_head_rows == 192,
          "head-split store of the product");
  auto c2 = tensor({4, 192, 384}), y2 = tensor({4, 6, 192, 64}), r = tensor({1, 384});
  Op split2 = transpose(view(c2), y2);
  split2.i0 = 1;
  split2.i1 = 2;
  std::vector<Op> q = {gemm(x, w, c2, 768, 384, 384), split2, reduce(c2, r), release(c2)};
  require(optimize(q, nullptr) == 0, "projection read again: kept");
  require(live(q).size() == 3 && !live(q)[0]->gemm.c_heads, "plain store kept");
}

// a product too small for the tensor cores (d 64, 2 heads, T 32, batch 1:
// 131k multiply-adds) runs on the CUDA-core kernel, which has no head-split
// store: the transpose stays
void head_split_store_small_product_kept() {
  auto x = tensor({1, 32, 64}), w = tensor({64, 64}), c = tensor({1, 32, 64});
  auto y = tensor({1, 2, 32, 32});
  TRef cv = c;
  cv.rank = 4;
  cv.shape[0] = 1;
  cv.shape[1] = 32;
  cv.shape[2] = 2;
  cv.shape[3] = 32;
  Op split = transpose(cv, y);
  split.i0 = 1;
  split.i1 = 2;
  std::vector<Op> p = {gemm(x, w, c, 32, 64, 64), split, release(c)};
  require(optimize(p, nullptr) == 0, "small product: no head-split store");
  auto l = live(p);
  require(l.size() == 2 && !l[0]->gemm.c_heads && l[1]->kind == Kind::Transpose,
          "product and transpose kept");
}

// the split's output reuses the address of a temporary that is read and
// released between the projection and the split (the pool's last-in
// first-out reuse): storing the head layout at the projection would
// overwrite the temporary before its reader runs, so the transpose stays
void head_split_store_reused_address_kept() {
  auto x = tensor({4, 192, 384}), w = tensor({384, 384}), c = tensor({4, 192, 384});
  auto z = tensor({4, 192, 384}), s = tensor({4, 192, 384});
  TRef y = z;  // same block address, new allocation
  y.id = g_id++;
  y.rank = 4;
  y.shape[0] = 4;
  y.shape[1] = 6;
  y.shape[2] = 192;
  y.shape[3] = 64;
  TRef cv = c;
  cv.rank = 4;
  cv.shape[0] = 4;
  cv.shape[1] = 192;
  cv.shape[2] = 6;
  cv.shape[3] = 64;
  Op split = transpose(cv, y);
  split.i0 = 1;
  split.i1 = 2;
  std::vector<Op> p = {gemm(x, w, c, 768, 384, 384), binary(TL_ADD, z, x, s), release(z), split,
                       release(c), reduce(s, tensor({1, 384}))};
  optimize(p, nullptr);
  bool kept = false;
  for (const Op *o : live(p)) kept = kept || o->kind == Kind::Transpose;
  require(kept, "released address reused by the split's output: transpose kept");
}

// attention head split / merge: the GEMMs address the [B, T, H, D] tensors
// through strides and both transposes go
void head_transposes_become_strides() {
  auto q = tensor({4, 192, 6, 64}), qh = tensor({4, 6, 192, 64}), kt = tensor({4, 6, 64, 192});
  auto s1 = tensor({4, 6, 192, 192}), pv = tensor({4, 6, 192, 64}), o = tensor({4, 192, 6, 64});
  auto v = tensor({4, 6, 192, 64});
  Op split = transpose(q, qh);
  split.i0 = 1;
  split.i1 = 2;
  Op merge = transpose(pv, o);
  merge.i0 = 1;
  merge.i1 = 2;
  std::vector<Op> p = {split, gemm(qh, kt, s1, 192, 192, 64, 24), release(qh),
                       gemm(s1, v, pv, 192, 64, 192, 24), merge, release(pv)};
  require(optimize(p, nullptr) == 2, "both transposes folded");
  auto l = live(p);
  require(l.size() == 2, "two products left");
  const tl_gemm_desc &g0 = l[0]->gemm;
  require(l[0]->t[0].id == q.id && g0.lda == 384 && g0.batch_rank == 2 &&
              g0.batch_shape[0] == 4 && g0.batch_shape[1] == 6 &&
              g0.a_batch_stride[0] == 192 * 384 && g0.a_batch_stride[1] == 64 &&
              g0.b_batch_stride[0] == 6 * 64 * 192 && g0.b_batch_stride[1] == 64 * 192,
          "scores read the heads of Q in place");
  const tl_gemm_desc &g1 = l[1]->gemm;
  require(l[1]->t[2].id == o.id && g1.ldc == 384 && g1.batch_rank == 2 &&
              g1.c_batch_stride[0] == 192 * 384 && g1.c_batch_stride[1] == 64,
          "the output lands in [B, T, H, D] directly");
}


// Q, K, V projections of one input: one N-grouped product; the summed input
// gradient dX = dQ Wq^T + dK Wk^T + dV Wv^T: one K-grouped product
void projections_grouped() {
  auto x = tensor({12288, 384}), wq = tensor({384, 384}), wk = tensor({384, 384});
  auto wv = tensor({384, 384}), q = tensor({12288, 384}), k = tensor({12288, 384});
  auto v = tensor({12288, 384});
  std::vector<Op> p = {gemm(x, wq, q, 12288, 384, 384), gemm(x, wk, k, 12288, 384, 384),
                       gemm(x, wv, v, 12288, 384, 384)};
  for (Op &o : p) o.i1 = 1;  // flattened [64, 192, 384] x [384, 384] products
  require(optimize(p, nullptr) == 2, "three projections grouped");
  auto l = live(p);
  require(l.size() == 1 && l[0]->gemm.group_mode == TL_GEMM_GROUP_N && l[0]->gemm.groups == 3 &&
              l[0]->gemm.b_group[2] == wv.p && l[0]->gemm.c_group[1] == k.p,
          "one launch, per-group weights and outputs");
  auto dq = tensor({12288, 384}), dk = tensor({12288, 384}), dv = tensor({12288, 384});
  auto pq = tensor({12288, 384}), dx = tensor({12288, 384});
  Op g1 = gemm(dq, wq, pq, 12288, 384, 384), g2 = gemm(dk, wk, dx, 12288, 384, 384),
     g3 = gemm(dv, wv, dx, 12288, 384, 384);
  g1.gemm.trans_b = g2.gemm.trans_b = g3.gemm.trans_b = 1;
  g2.t[5] = pq;
  g2.gemm.addend = pq.f();
  g3.gemm.beta = 1.0f;
  std::vector<Op> q2 = {g1, g2, g3, release(pq)};
  require(optimize(q2, nullptr) == 2, "three summed products grouped");
  auto m = live(q2);
  require(m.size() == 1 && m[0]->gemm.group_mode == TL_GEMM_GROUP_K && m[0]->gemm.groups == 3 &&
              m[0]->gemm.a_group[0] == dq.p && m[0]->gemm.b_group[2] == wv.p &&
              m[0]->t[2].id == dx.id && m[0]->gemm.beta == 0.0f && !m[0]->gemm.addend,
          "one K-grouped product into dX");
}


Op softmax_op(const TRef &x, const TRef &y, const TRef &div, const TRef &mask) {
  Op o = op(Kind::Softmax);
  o.t[0] = x;
  o.t[1] = y;
  o.t[2] = div;
  o.t[3] = mask;
  return o;
}

// attention forward: scores product, scaled masked softmax, P V -> one
// fused op at the P V product, with K read through its transposed copy
void attention_forward_fused() {
  const uint32_t B = 4, H = 6, T = 192, D = 64;
  auto q = tensor({B, H, T, D}), kt = tensor({B, H, D, T}), v = tensor({B, H, T, D});
  auto s1 = tensor({B, H, T, T}), pr = tensor({B, H, T, T}), o = tensor({B, H, T, D});
  auto div = tensor({1, 1}), mask = tensor({1, 1, T, T});
  std::vector<Op> p = {gemm(q, kt, s1, T, T, D, B * H), softmax_op(s1, pr, div, mask),
                       release(s1), gemm(pr, v, o, T, D, T, B * H)};
  require(optimize(p, nullptr) == 2, "two ops folded into the fused op");
  auto l = live(p);
  require(l.size() == 1 && l[0]->kind == Kind::Attention && l[0]->code == TL_ATTN_FORWARD,
          "one fused attention op");
  const tl_attn_desc &d = l[0]->attn;
  require(d.B == B && d.H == H && d.T == T && d.D == D && d.k.transposed == 1 &&
              d.k.row_stride == T && d.k.head_stride == D * T && d.q.transposed == 0 &&
              d.q.row_stride == D && d.q.batch_stride == H * T * D && d.p == pr.p &&
              d.mask == mask.p && d.divisor == div.p && d.o.p == o.p,
          "views of Q, K^T, V, O and the score tensors");
  // P read by another op before the P V product: kept unfused
  auto other = tensor({B, H, T, T});
  std::vector<Op> p2 = {gemm(q, kt, s1, T, T, D, B * H), softmax_op(s1, pr, div, mask),
                        release(s1), binary(TL_ADD, pr, pr, other),
                        gemm(pr, v, o, T, D, T, B * H)};
  optimize(p2, nullptr);
  for (const Op *x : live(p2)) require(x->kind != Kind::Attention, "P observed: not fused");
  // Q rewritten between the products: kept unfused
  std::vector<Op> p3 = {gemm(q, kt, s1, T, T, D, B * H), softmax_op(s1, pr, div, mask),
                        release(s1), binary(TL_ADD, v, v, q), gemm(pr, v, o, T, D, T, B * H)};
  optimize(p3, nullptr);
  for (const Op *x : live(p3)) require(x->kind != Kind::Attention, "Q changed: not fused");
}

// attention backward: dP = dO V^T, softmax derivative with the divisor,
// dQ = dS K -> one fused op; dK = dS^T Q and dV = P^T dO -> key-side ops
void attention_backward_fused() {
  const uint32_t B = 4, H = 6, T = 192, D = 64;
  auto d_o = tensor({B, H, T, D}), v = tensor({B, H, T, D}), pr = tensor({B, H, T, T});
  auto dp = tensor({B, H, T, T}), ds = tensor({B, H, T, T}), kt = tensor({B, H, D, T});
  auto dq = tensor({B, H, T, D}), q = tensor({B, H, T, D}), dk = tensor({B, H, T, D});
  auto dv = tensor({B, H, T, D}), div = tensor({1, 1});
  Op g1 = gemm(d_o, v, dp, T, T, D, B * H);
  g1.gemm.trans_b = 1;
  Op sb = op(Kind::SoftmaxBwd);
  sb.t[0] = dp;
  sb.t[1] = pr;
  sb.t[2] = ds;
  sb.t[3] = div;
  Op g2 = gemm(ds, kt, dq, T, D, T, B * H);
  g2.gemm.trans_b = 1;
  Op g3 = gemm(ds, q, dk, T, D, T, B * H);
  g3.gemm.trans_a = 1;
  Op g4 = gemm(pr, d_o, dv, T, D, T, B * H);
  g4.gemm.trans_a = 1;
  std::vector<Op> p = {g1, sb, release(dp), g2, g3, release(ds), g4};
  require(optimize(p, nullptr) == 2, "dP product and derivative folded");
  auto l = live(p);
  require(l.size() == 3 && l[0]->kind == Kind::Attention &&
              l[0]->code == TL_ATTN_BACKWARD_Q && l[0]->attn.k.transposed == 1 &&
              l[0]->attn.ds == ds.p && l[0]->attn.dq.p == dq.p,
          "query side fused, dS still written");
  require(l[1]->kind == Kind::Attention && l[1]->code == TL_ATTN_PRODUCT_TN &&
              l[1]->attn.ds == ds.p && l[1]->attn.q.p == q.p && l[1]->attn.dk.p == dk.p &&
              l[2]->kind == Kind::Attention && l[2]->attn.ds == pr.p && l[2]->attn.dk.p == dv.p,
          "dK and dV on the key-side kernel");
}



// dH = dY W2^T; GELU backward(x, dH) -> dX: the product's epilogue applies
// GELU'(x); kept apart when dH is read again
void gelu_backward_into_gemm() {
  auto dy = tensor({12288, 384}), w = tensor({1536, 384}), dh = tensor({12288, 1536});
  auto x = tensor({12288, 1536}), dx = tensor({12288, 1536}), other = tensor({12288, 1536});
  Op g = gemm(dy, w, dh, 12288, 1536, 384);
  g.gemm.trans_b = 1;
  g.i1 = 1;  // recorded as a batch of row blocks flattened into M
  Op gb = op(Kind::GeluBwd);
  gb.t[0] = x;
  gb.t[1] = dh;
  gb.t[2] = dx;
  std::vector<Op> p = {g, gb, release(dh)};
  require(optimize(p, nullptr) == 1, "GELU backward folded");
  auto l = live(p);
  require(l.size() == 1 && l[0]->kind == Kind::Gemm && l[0]->t[2].id == dx.id &&
              l[0]->gemm.gelu_grad_x == x.p && l[0]->gemm.c == dx.p && l[0]->t[6].id == x.id,
          "the product writes dX through GELU'(x)");
  std::vector<Op> q = {g, gb, binary(TL_ADD, dh, dh, other), release(dh)};
  optimize(q, nullptr);
  bool kept = false;
  for (const Op *o : live(q)) kept = kept || o->kind == Kind::GeluBwd;
  require(kept, "dH read again: not folded");
}

}  // namespace

// One causal check per mask per program, again after the mask is written.
void mask_checked_once_per_program() {
  const TRef q = tensor({64, 6, 192, 64}), mask = tensor({192, 192}), o = tensor({64, 6, 192, 64});
  uint32_t word = 0;
  auto fwd = [&]() {
    Op a = op(Kind::Attention);
    a.code = TL_ATTN_FORWARD;
    a.attn.pass = TL_ATTN_FORWARD;
    a.attn.mask_flag = &word;
    a.t[0] = q;
    a.t[4] = mask;
    a.t[6] = o;
    return a;
  };
  Op fill = op(Kind::Fill);
  fill.t[0] = mask;
  fill.n = mask.numel();
  std::vector<Op> p = {fwd(), fwd(), fill, fwd(), fwd()};
  assign_mask_checks(p);
  require(p[0].u0 == 1 && p[1].u0 == 0, "first forward checks, the second reads the word");
  require(p[3].u0 == 1 && p[4].u0 == 0, "a write to the mask calls for a new check");
}

// bias gradients of the query, key and value projections (sum_to_shape of
// dQ, dK, dV to [1, 384]) with other work between: one grouped reduction
// at the last one's position; kept apart when an input changes or an output
// is read in between
void bias_gradients_grouped() {
  auto sum = [](const TRef &x, const TRef &y) {
    Op o = op(Kind::Reduce);
    o.code = TL_REDUCE_SUM;
    o.t[0] = x;
    o.t[1] = y;
    o.workspace = 4096;
    return o;
  };
  auto dq = tensor({64, 192, 384}), dk = tensor({64, 192, 384}), dv = tensor({64, 192, 384});
  auto bq = tensor({1, 384}), bk = tensor({1, 384}), bv = tensor({1, 384});
  auto w = tensor({384, 384}), dx = tensor({64, 192, 384}), other = tensor({64, 192, 384});
  std::vector<Op> p = {sum(dv, bv), gemm(dv, w, dx, 12288, 384, 384), sum(dk, bk),
                       binary(TL_ADD, dx, dq, other), sum(dq, bq)};
  optimize(p, nullptr);
  auto l = live(p);
  require(l.size() == 3 && l[2]->kind == Kind::Reduce && l[2]->group_refs.size() == 4 &&
              l[2]->t[0].id == dv.id && l[2]->group_refs[0].id == dk.id &&
              l[2]->group_refs[3].id == bq.id && l[2]->workspace == 3 * 4096,
          "three column sums, one launch after the last");
  // dk rewritten before its sum's group position: dv's sum stays alone
  std::vector<Op> q = {sum(dv, bv), binary(TL_ADD, dq, dq, dv), sum(dk, bk)};
  optimize(q, nullptr);
  auto m = live(q);
  require(m.size() == 3 && m[0]->group_refs.empty() && m[2]->group_refs.empty(),
          "an input written in between keeps the sums apart");
  // an output read before the group position
  std::vector<Op> r = {sum(dv, bv), binary(TL_ADD, bv, bv, bk), sum(dk, bq)};
  optimize(r, nullptr);
  auto n = live(r);
  require(n.size() == 3 && n[0]->group_refs.empty(), "an output read in between keeps them apart");
  // different shapes
  auto wide = tensor({64, 192, 1536}), bw = tensor({1, 1536});
  std::vector<Op> s2 = {sum(dv, bv), sum(wide, bw)};
  optimize(s2, nullptr);
  require(live(s2).size() == 2, "different shapes are not grouped");
}

int main() {
  int failures = 0;
  const std::vector<std::pair<const char *, void (*)()>> cases = {
      {"linear_bias_gelu", linear_bias_gelu},
      {"weight_gradient_tn", weight_gradient_tn},
      {"weight_gradient_observable_product_kept", weight_gradient_observable_product_kept},
      {"transpose_into_b", transpose_into_b},
      {"head_split_store", head_split_store},
      {"head_split_store_small_product_kept", head_split_store_small_product_kept},
      {"head_split_store_reused_address_kept", head_split_store_reused_address_kept},
      {"transpose_kept_when_read_later", transpose_kept_when_read_later},
      {"softmax_backward", softmax_backward},
      {"rmsnorm_backward", rmsnorm_backward},
      {"xent_and_gelu_backward", xent_and_gelu_backward},
      {"reused_address_is_not_confused", reused_address_is_not_confused},
      {"fused_step", fused_step},
      {"copy_forwarded_to_reader", copy_forwarded_to_reader},
      {"copy_kept_when_observable", copy_kept_when_observable},
      {"copy_kept_when_source_changes", copy_kept_when_source_changes},
      {"common_gemm_evaluated_once", common_gemm_evaluated_once},
      {"common_kept_when_input_changes", common_kept_when_input_changes},
      {"residual_add_into_gemm", residual_add_into_gemm},
      {"attention_scores_into_softmax", attention_scores_into_softmax},
      {"row_backward_tails", row_backward_tails},
      {"head_transposes_become_strides", head_transposes_become_strides},
      {"projections_grouped", projections_grouped},
      {"attention_forward_fused", attention_forward_fused},
      {"attention_backward_fused", attention_backward_fused},
      {"gelu_backward_into_gemm", gelu_backward_into_gemm},
      {"mask_checked_once_per_program", mask_checked_once_per_program},
      {"bias_gradients_grouped", bias_gradients_grouped},
  };
  for (const auto &[name, fn] : cases) {
    try {
      fn();
      std::printf("PASS %s\n", name);
    } catch (const std::exception &e) {
      std::printf("FAIL %s: %s\n", name, e.what());
      ++failures;
    }
  }
  return failures ? 1 : 0;
}

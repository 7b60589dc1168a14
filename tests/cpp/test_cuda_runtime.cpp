// Known-answer tests of cuda::Runtime, one per case of the reference's Metal
// runtime suite (tests/test_metal_runtime.cpp:83-658 in JTPuffer/TempLit):
// same inputs, same closed-form expectations, same tolerances.  Plus the
// CUDA-specific behaviour: alias safety, device-side index errors, lazy
// recording of storage writes inside a window, and graph replay.
//
// Runs on a GPU; prints one "PASS <name>" line per case and exits non-zero
// on the first failure.
#include "my_cuda/runtime.h"
#include "templit_cuda.h"
#include "my_cuda/storage.h"
#include "optimiser/AdamW.h"
#include "passes/concepts.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <functional>
#include <initializer_list>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

using Tensor = RTensor<cuda::CUDA, cuda::kernel_type>;
using IndexTensor = RTensor<cuda::CUDA, cuda::index_type>;

static_assert(passes::Runnable<Tensor, cuda::Runtime>);

namespace {

struct Failure : std::runtime_error {
  using std::runtime_error::runtime_error;
};

void require(bool ok, const std::string &what) {
  if (!ok) throw Failure(what);
}

void put(Tensor &t, std::initializer_list<float> v) {
  require(v.size() == t.numel(), "fixture size");
  t.get_storage()->write(std::span<const float>(v.begin(), v.size()), 0);
}

template <typename T> std::vector<typename T::value_type> get(const T &t) {
  std::vector<typename T::value_type> v(t.numel());
  t.read(std::span<typename T::value_type>(v));
  return v;
}

void expect(const Tensor &t, const std::vector<float> &want, const std::string &name,
            float eps = 1e-5f) {
  const auto got = get(t);
  require(got.size() == want.size(), name + ": size " + std::to_string(got.size()));
  for (size_t i = 0; i < got.size(); ++i) {
    if (!(std::abs(got[i] - want[i]) < eps)) {
      throw Failure(name + ": index " + std::to_string(i) + " got " + std::to_string(got[i]) +
                    " expected " + std::to_string(want[i]));
    }
  }
}

void expect_shape(const Tensor &t, std::vector<uint32_t> s, const std::string &name) {
  require(t.shape() == s, name + ": shape");
}

template <typename E, typename F> bool throws(F &&f) {
  try {
    f();
  } catch (const E &) {
    return true;
  }
  return false;
}

void run(cuda::Runtime &rt, const std::function<void()> &body) {
  rt.start();
  try {
    body();
    rt.submit();
    rt.wait();
  } catch (...) {
    rt.abort();
    throw;
  }
}

// ---------------------------------------------------------------- cases
void lifecycle(cuda::Runtime &rt) {
  require(throws<std::logic_error>([&] { rt.submit(); }), "submit before start");
  rt.start();
  require(throws<std::logic_error>([&] { rt.start(); }), "double start");
  rt.abort();
  rt.start();
  rt.submit();
  require(throws<std::logic_error>([&] { rt.submit(); }), "double submit");
  rt.wait();
  require(throws<std::logic_error>([&] { rt.wait(); }), "double wait");
  Tensor a({1});
  require(throws<std::logic_error>([&] { rt.copy(a, a); }), "op outside a window");
}

void cleanup_idempotent(cuda::Runtime &) {
  cuda::Runtime r;
  r.cleanup();
  r.cleanup();
}

void binary_chain(cuda::Runtime &rt) {
  Tensor a({2, 2}), b({2, 2}), add({2, 2}), sub({2, 2}), mul({2, 2}), div({2, 2}), ch({2, 2});
  put(a, {1, 2, 3, 4});
  put(b, {5, 6, 7, 8});
  run(rt, [&] {
    rt.add(a, b, add);
    rt.sub(a, b, sub);
    rt.hadamard(a, b, mul);
    rt.divide(a, b, div);
    rt.hadamard(add, a, ch);
  });
  expect(add, {6, 8, 10, 12}, "add");
  expect(sub, {-4, -4, -4, -4}, "sub");
  expect(mul, {5, 12, 21, 32}, "hadamard");
  expect(div, {0.2f, 1.0f / 3.0f, 3.0f / 7.0f, 0.5f}, "divide");
  expect(ch, {6, 16, 30, 48}, "chained");
}

void broadcasting(cuda::Runtime &rt) {
  Tensor m({2, 3}), row({3}), out({2, 3});
  put(m, {1, 2, 3, 4, 5, 6});
  put(row, {10, 20, 30});
  run(rt, [&] { rt.add(m, row, out); });
  expect_shape(out, {2, 3}, "broadcast");
  expect(out, {11, 22, 33, 14, 25, 36}, "broadcast");
  Tensor bad({4});
  rt.start();
  require(throws<std::runtime_error>([&] { rt.add(m, bad, out); }), "invalid broadcast");
  rt.abort();
}

void scalar_ops(cuda::Runtime &rt) {
  Tensor in({2, 2}), added({2, 2}), divided({2, 2}), cubed({2, 2}), inplace({2, 2});
  put(in, {2, 4, 6, 8});
  put(inplace, {2, 4, 6, 8});
  run(rt, [&] {
    rt.add(in, 3.0f, added);
    rt.divide(in, 2.0f, divided);
    rt.pow(in, 3.0f, cubed);
    rt.divide(inplace, 2.0f, inplace);
    rt.pow(inplace, 2.0f, inplace);
  });
  expect(added, {5, 7, 9, 11}, "scalar add");
  expect(divided, {1, 2, 3, 4}, "scalar divide");
  expect(cubed, {8, 64, 216, 512}, "scalar power", 1e-3f);
  expect(inplace, {1, 4, 9, 16}, "in-place scalar power", 1e-3f);
  Tensor wrong({4});
  rt.start();
  require(throws<std::invalid_argument>([&] { rt.add(in, 1.0f, wrong); }), "scalar shape check");
  rt.abort();
}

void unary_ops(cuda::Runtime &rt) {
  Tensor in({4}), sq({4}), sg({4}), ex({4}), rt_({4});
  put(in, {0, 1, -1, 2});
  put(sq, {0, 1, 4, 9});
  run(rt, [&] {
    rt.sigmoid(in, sg);
    rt.exp(in, ex);
    rt.sqrt(sq, rt_);
  });
  expect(sg, {0.5f, 1.0f / (1.0f + std::exp(-1.0f)), 1.0f / (1.0f + std::exp(1.0f)),
              1.0f / (1.0f + std::exp(-2.0f))},
         "sigmoid");
  expect(ex, {1.0f, std::exp(1.0f), std::exp(-1.0f), std::exp(2.0f)}, "exp");
  expect(rt_, {0, 1, 2, 3}, "sqrt");
}

void rms(cuda::Runtime &rt) {
  Tensor in({2, 2}), r({2, 1}), n({2, 2});
  put(in, {3, 4, 0, 0});
  run(rt, [&] {
    rt.RMS(in, r);
    rt.RMSNorm(in, n);
  });
  const float first = std::sqrt(12.5f + 1e-6f);
  expect(r, {first, 1e-3f}, "RMS");  // an all-zero row gives sqrt(1e-6)
  expect(n, {3.0f / first, 4.0f / first, 0, 0}, "RMSNorm");
}

float gelu_ref(float x) {
  const float a = 0.7978845608f;
  return 0.5f * x * (1.0f + std::tanh(a * (x + 0.044715f * x * x * x)));
}
float gelu_d_ref(float x) {
  const float a = 0.7978845608f, b = 0.044715f, x2 = x * x;
  const float t = std::tanh(a * (x + b * x2 * x));
  return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * a * (1.0f + 3.0f * b * x2);
}

void gelu(cuda::Runtime &rt) {
  Tensor in({5}), out({5}), d({5});
  put(in, {-2, -1, 0, 1, 2});
  run(rt, [&] {
    rt.GELU(in, out);
    rt.GELU_derivative(in, d);
  });
  std::vector<float> w, wd;
  for (float x : {-2.f, -1.f, 0.f, 1.f, 2.f}) {
    w.push_back(gelu_ref(x));
    wd.push_back(gelu_d_ref(x));
  }
  expect(out, w, "GELU");
  expect(d, wd, "GELU derivative");
}

void matmul(cuda::Runtime &rt) {
  Tensor a({2, 3}), b({3, 2}), out({2, 2});
  put(a, {1, 2, 3, 4, 5, 6});
  put(b, {7, 8, 9, 10, 11, 12});
  Tensor ba({2, 2, 2}), bb({2, 2, 2}), bo({2, 2, 2});
  put(ba, {1, 2, 3, 4, 2, 0, 1, 2});
  put(bb, {5, 6, 7, 8, 1, 3, 4, 2});
  run(rt, [&] {
    rt.mult(a, b, out);
    rt.mult(ba, bb, bo);
  });
  expect(out, {58, 64, 139, 154}, "matmul");
  expect(bo, {19, 22, 43, 50, 2, 6, 9, 7}, "batched matmul");
  Tensor k({2, 2});
  rt.start();
  require(throws<std::invalid_argument>([&] { rt.mult(a, k, out); }), "inner dims");
  require(throws<std::runtime_error>([&] {
            Tensor v({3});
            rt.mult(v, b, out);
          }),
          "rank < 2");
  rt.abort();
}

void tiled_identity(cuda::Runtime &rt) {
  constexpr uint32_t n = 64, batches = 2;
  Tensor id({batches, n, n}), vals({batches, n, n}), out({batches, n, n});
  std::vector<float> iv(batches * n * n, 0.0f), xv(batches * n * n);
  for (uint32_t b = 0; b < batches; ++b)
    for (uint32_t r = 0; r < n; ++r) iv[b * n * n + r * n + r] = 1.0f;
  for (uint32_t i = 0; i < xv.size(); ++i) xv[i] = static_cast<float>(i % 31) - 15.0f;
  id.set(iv);
  vals.set(xv);
  run(rt, [&] { rt.mult(id, vals, out); });
  expect(out, xv, "tiled identity matmul");
}

void reductions(cuda::Runtime &rt) {
  Tensor in({2, 3});
  put(in, {1, 2, 3, 4, 5, 6});
  const std::vector<uint32_t> col = {2, 1}, row = {1, 3};
  Tensor total({1}), rs({2, 1}), cs(row), mx(col), tr({3, 2});
  run(rt, [&] {
    rt.sum(in, total);
    rt.sum(in, 1, rs);
    rt.sum_to_shape(in, row, cs);
    rt.max_to_shape(in, col, mx);
    rt.transpose(in, tr);
  });
  expect(total, {21}, "sum");
  expect(rs, {6, 15}, "axis sum");
  expect(cs, {5, 7, 9}, "sum_to_shape");
  expect(mx, {3, 6}, "max_to_shape");
  expect_shape(tr, {3, 2}, "transpose");
  expect(tr, {1, 4, 2, 5, 3, 6}, "transpose");
  rt.start();
  require(throws<std::out_of_range>([&] { rt.sum(in, 2, rs); }), "sum axis range");
  require(throws<std::out_of_range>([&] { rt.transpose(in, tr, 0, 5); }), "transpose range");
  rt.abort();
}

void sum_to_shape_multi(cuda::Runtime &rt) {
  Tensor in({2, 3, 4});
  std::vector<float> v(24);
  for (int i = 0; i < 24; ++i) v[i] = float(i + 1);
  in.set(v);
  const std::vector<uint32_t> na = {1, 3, 1}, adj = {2, 1, 1}, sc = {1, 1, 1}, tr = {4};
  Tensor a(na), b(adj), c(sc), d(tr);
  run(rt, [&] {
    rt.sum_to_shape(in, na, a);
    rt.sum_to_shape(in, adj, b);
    rt.sum_to_shape(in, sc, c);
    rt.sum_to_shape(in, tr, d);
  });
  expect(a, {68, 100, 132}, "sum_to_shape non-adjacent");
  expect(b, {78, 222}, "sum_to_shape adjacent");
  expect(c, {300}, "sum_to_shape all");
  expect(d, {66, 72, 78, 84}, "sum_to_shape lower rank");
}

void sum_to_shape_leading(cuda::Runtime &rt) {
  Tensor in({1, 4});
  put(in, {1, 2, 3, 4});
  const std::vector<uint32_t> s = {4};
  Tensor out(s);
  run(rt, [&] { rt.sum_to_shape(in, s, out); });
  expect(out, {1, 2, 3, 4}, "sum_to_shape removes leading singleton");
}

void softmax(cuda::Runtime &rt) {
  Tensor in({2, 3}), out({2, 3}), r1({3}), r1o({3}), r4({2, 2, 1, 3}), r4o({2, 2, 1, 3}),
      s1({2, 1}), s1o({2, 1});
  put(in, {1, 2, 3, 1, 1, 1});
  put(r1, {1, 2, 3});
  put(r4, {1, 2, 3, 3, 2, 1, 1000, 1001, 1002, -1000, -1000, -1000});
  put(s1, {4, -7});
  run(rt, [&] {
    rt.softmax(in, out);
    rt.softmax(r1, r1o);
    rt.softmax(r4, r4o);
    rt.softmax(s1, s1o);
  });
  const float den = std::exp(-2.0f) + std::exp(-1.0f) + 1.0f;
  const float lo = std::exp(-2.0f) / den, mid = std::exp(-1.0f) / den, hi = 1.0f / den;
  const float t = 1.0f / 3.0f;
  expect(out, {lo, mid, hi, t, t, t}, "softmax");
  expect(r1o, {lo, mid, hi}, "softmax rank one");
  expect(r4o, {lo, mid, hi, hi, mid, lo, lo, mid, hi, t, t, t}, "softmax rank four");
  expect(s1o, {1, 1}, "softmax singleton rows");
}

void cross_entropy(cuda::Runtime &rt) {
  Tensor logits({2, 2, 3});
  put(logits, {1, 2, 3, 1, 1, 1, 1000, 1001, 1002, -1, -2, -3});
  IndexTensor targets({2, 2});
  targets.set(std::vector<uint32_t>{2, 0, 1, 2});
  Tensor loss({2, 2, 1}), grad({2, 2, 3});
  run(rt, [&] {
    rt.cross_entropy(logits, targets, loss);
    rt.cross_entropy_derivative(logits, targets, grad);
  });
  const float den = std::exp(-2.0f) + std::exp(-1.0f) + 1.0f;
  const float lo = std::exp(-2.0f) / den, mid = std::exp(-1.0f) / den, hi = 1.0f / den;
  const float ld = std::log(den);
  expect(loss, {ld, std::log(3.0f), 1.0f + ld, 2.0f + ld}, "cross entropy", 1e-4f);
  expect(grad,
         {lo, mid, hi - 1.0f, -2.0f / 3.0f, 1.0f / 3.0f, 1.0f / 3.0f, lo, mid - 1.0f, hi, hi, mid,
          lo - 1.0f},
         "cross entropy derivative", 1e-4f);
  // a target outside the vocabulary gives +inf (math.metal:893-896,921-925)
  IndexTensor bad({2, 2});
  bad.set(std::vector<uint32_t>{2, 7, 1, 2});
  run(rt, [&] {
    rt.cross_entropy(logits, bad, loss);
    rt.cross_entropy_derivative(logits, bad, grad);
  });
  const auto l = get(loss), g = get(grad);
  require(std::isinf(l[1]) && l[1] > 0 && std::isfinite(l[0]), "invalid target loss = +inf");
  require(std::isinf(g[3]) && std::isinf(g[5]) && std::isfinite(g[0]), "invalid target grad = +inf");
}

void argmax(cuda::Runtime &rt) {
  Tensor small({2, 3});
  put(small, {1, 4, 2, 9, 3, 5});
  Tensor large({5000});
  std::vector<float> v(5000, 0.0f);
  v[4097] = 100.0f;
  large.set(v);
  IndexTensor so({1, 1}), lo({1, 1});
  run(rt, [&] {
    rt.argmax(small, so);
    rt.argmax(large, lo);
  });
  require(get(so)[0] == 3, "argmax small");
  require(get(lo)[0] == 4097, "argmax multi-pass");
}

void embedding(cuda::Runtime &rt) {
  Tensor w({4, 3});
  put(w, {1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12});
  IndexTensor ids({2, 2});
  ids.set(std::vector<uint32_t>{2, 0, 3, 1});
  Tensor out({2, 2, 3});
  run(rt, [&] { rt.embedding_lookup(w, ids, out); });
  expect(out, {7, 8, 9, 1, 2, 3, 10, 11, 12, 4, 5, 6}, "embedding lookup");
  // an id past the table raises on wait() instead of reading out of bounds
  IndexTensor bad({2, 2});
  bad.set(std::vector<uint32_t>{2, 0, 9, 1});
  rt.start();
  rt.embedding_lookup(w, bad, out);
  rt.submit();
  require(throws<std::out_of_range>([&] { rt.wait(); }), "embedding id range");
}

void scatter_index(cuda::Runtime &rt) {
  Tensor vals({2, 2, 3});
  put(vals, {1, 2, 3, 4, 5, 6, 10, 20, 30, 7, 8, 9});
  IndexTensor ids({2, 2});
  ids.set(std::vector<uint32_t>{2, 0, 2, 1});
  Tensor out({4, 3});
  put(out, {99, 99, 99, 99, 99, 99, 99, 99, 99, 99, 99, 99});
  run(rt, [&] { rt.scatter_index(vals, ids, out); });
  expect(out, {4, 5, 6, 7, 8, 9, 11, 22, 33, 0, 0, 0}, "scatter index");
}

void scatter_add_rows(cuda::Runtime &rt) {
  Tensor base({4, 3});
  put(base, {100, 101, 102, 103, 104, 105, 106, 107, 108, 109, 110, 111});
  Tensor vals({2, 2, 3});
  put(vals, {1, 2, 3, 4, 5, 6, 10, 20, 30, 7, 8, 9});
  IndexTensor ids({2, 2});
  ids.set(std::vector<uint32_t>{2, 0, 2, 1});
  Tensor out({4, 3});
  run(rt, [&] { rt.scatter_add_rows(base, ids, vals, out); });
  expect(out, {104, 106, 108, 110, 112, 114, 117, 129, 141, 109, 110, 111}, "scatter add rows");
}

void clipping(cuda::Runtime &rt) {
  Tensor first({3}), second({1});
  Tensor sq = Tensor::from_zeros({1});
  put(first, {3.0f, 4.0f, 0.0f});
  put(second, {12.0f});
  run(rt, [&] {
    rt.accumulate_gradient_squared_norm(first, sq);
    rt.accumulate_gradient_squared_norm(second, sq);
    rt.clip_gradient(first, sq, 1.0f, first);
    rt.clip_gradient(second, sq, 1.0f, second);
  });
  expect(sq, {169.0f}, "gradient squared norm");
  expect(first, {3.0f / 13.0f, 4.0f / 13.0f, 0.0f}, "clipped first gradient");
  expect(second, {12.0f / 13.0f}, "clipped second gradient");
  rt.start();
  require(throws<std::invalid_argument>([&] { rt.clip_gradient(first, sq, -1.0f, first); }),
          "max norm must be positive");
  rt.abort();
}

void adamw(cuda::Runtime &rt) {
  using AdamW = Optimiser::AdamW<Tensor>;
  Tensor p({4}), g({4});
  put(p, {1.0f, -2.0f, 3.0f, -4.0f});
  put(g, {0.5f, -0.25f, 1.0f, -0.75f});
  AdamW opt;
  auto params = AdamW::generate_params(0.01f, 0.9f, 0.999f, 1e-8f, 0.01f);
  std::vector<float> want{1.0f, -2.0f, 3.0f, -4.0f};
  const std::vector<float> gv{0.5f, -0.25f, 1.0f, -0.75f};
  std::vector<float> m1(4, 0.0f), m2(4, 0.0f);
  for (uint32_t step = 1; step <= 2; ++step) {
    run(rt, [&] { opt.update(rt, params, p, g, p); });
    const float c1 = 1.0f - std::pow(0.9f, float(step));
    const float c2 = 1.0f - std::pow(0.999f, float(step));
    for (size_t i = 0; i < 4; ++i) {
      m1[i] = 0.9f * m1[i] + 0.1f * gv[i];
      m2[i] = 0.999f * m2[i] + 0.001f * gv[i] * gv[i];
      want[i] = want[i] * 0.9999f - 0.01f * (m1[i] / c1) / (std::sqrt(m2[i] / c2) + 1e-8f);
    }
    expect(p, want, "AdamW step " + std::to_string(step), 1e-5f);
  }
}

// -------------------------------------------------------- CUDA-specific
void storage_semantics(cuda::Runtime &rt) {
  // clone / compare / fill through the device
  Tensor a({3});
  put(a, {1, 2, 3});
  Tensor b = a.clone();
  require(a == b, "clone compares equal");
  b.get_storage()->fill(7.0f);
  expect(b, {7, 7, 7}, "fill");
  require(!(a == b), "compare detects difference");
  // a tensor created and written inside a window is written in program order
  Tensor out({1, 2});
  run(rt, [&] {
    Tensor tmp = Tensor::from_values({{1.0f, 2.0f}});
    rt.copy(tmp, out);
    Tensor tmp2 = Tensor::from_values({{3.0f, 4.0f}});
    rt.add(out, tmp2, out);
  });
  expect(out, {4, 6}, "in-window writes keep program order");
  require(throws<std::out_of_range>([&] {
            std::vector<float> v(4);
            a.get_storage()->write(std::span<const float>(v), 0);
          }),
          "write bounds");
}

void alias_safety(cuda::Runtime &rt) {
  Tensor x({2, 3}), bias({1, 3});
  put(x, {1, 2, 3, 4, 5, 6});
  put(bias, {1, 1, 1});
  run(rt, [&] {
    rt.add(x, bias, x);
    rt.hadamard(x, x, x);
  });
  expect(x, {4, 9, 16, 25, 36, 49}, "in-place broadcast ops");
}

void graph_replay(cuda::Runtime &rt) {
  // the same program twice is captured, a third time is replayed
  Tensor a({64, 96}), b({96, 32}), c({64, 32}), d({64, 32});
  std::vector<float> av(64 * 96), bv(96 * 32);
  for (size_t i = 0; i < av.size(); ++i) av[i] = float(int(i % 7) - 3);
  for (size_t i = 0; i < bv.size(); ++i) bv[i] = float(int(i % 5) - 2);
  a.set(av);
  b.set(bv);
  std::vector<float> want(64 * 32, 0.0f);
  for (int i = 0; i < 64; ++i)
    for (int j = 0; j < 32; ++j) {
      float s = 0;
      for (int k = 0; k < 96; ++k) s += av[i * 96 + k] * bv[k * 32 + j];
      want[i * 32 + j] = s + s;
    }
  const auto before = rt.stats();
  for (int it = 0; it < 4; ++it) {
    run(rt, [&] {
      rt.mult(a, b, c);
      rt.add(c, c, d);
    });
    expect(d, want, "graph replay iteration " + std::to_string(it));
  }
  const auto after = rt.stats();
  require(after.graph_captures > before.graph_captures, "a graph was captured");
  require(after.graph_replays >= before.graph_replays + 2, "the graph was replayed");
}

// The attention composite of nn::MultiHeadAttention (include/nn/
// multi_head.h:45-52) recorded op by op: the forward runs as one flash
// attention launch that leaves P unwritten (its recipe is kept), and P is
// rebuilt exactly when something else needs it: a host read, and an op of a
// later window that reads it.
void flash_attention_virtual_probs(cuda::Runtime &rt) {
  rt.set_flash_attention(2);  // T = 128 would take the short-sequence kernels
  const uint32_t H = 2, T = 128, D = 64;
  Tensor q({1, H, T, D}), k({1, H, T, D}), v({1, H, T, D}), div({1, 1}), mask({1, 1, T, T});
  Tensor p({1, H, T, T}), o({1, H, T, D}), p2({1, H, T, T});
  std::vector<float> qv(H * T * D), kv(H * T * D), vv(H * T * D), mv(T * T);
  for (size_t i = 0; i < qv.size(); ++i) {
    qv[i] = std::sin(0.37f * float(i)) * 1.5f;
    kv[i] = std::cos(0.23f * float(i)) * 1.5f;
    vv[i] = std::sin(0.11f * float(i) + 1.0f);
  }
  for (uint32_t r = 0; r < T; ++r)
    for (uint32_t c = 0; c < T; ++c) mv[r * T + c] = c > r ? -INFINITY : 0.0f;
  q.set(qv);
  k.set(kv);
  v.set(vv);
  mask.set(mv);
  put(div, {8.0f});
  auto forward = [&] {
    Tensor kt({1, H, D, T}), s({1, H, T, T}), sd({1, H, T, T}), sm({1, H, T, T});
    rt.transpose(k, kt);
    rt.mult(q, kt, s);
    rt.divide(s, div, sd);
    rt.add(sd, mask, sm);
    rt.softmax(sm, p);
    rt.mult(p, v, o);
  };
  // the softmax of the scores in double precision
  std::vector<double> want(H * T * T), ov(H * T * D, 0.0);
  for (uint32_t h = 0; h < H; ++h)
    for (uint32_t r = 0; r < T; ++r) {
      double mx = -1e300;
      std::vector<double> row(T);
      for (uint32_t c = 0; c < T; ++c) {
        double acc = 0;
        for (uint32_t d = 0; d < D; ++d)
          acc += double(qv[(h * T + r) * D + d]) * double(kv[(h * T + c) * D + d]);
        row[c] = c > r ? -1e300 : acc / 8.0;
        mx = std::max(mx, row[c]);
      }
      double sum = 0;
      for (uint32_t c = 0; c < T; ++c) sum += row[c] <= -1e299 ? 0.0 : std::exp(row[c] - mx);
      for (uint32_t c = 0; c < T; ++c) {
        const double pv = row[c] <= -1e299 ? 0.0 : std::exp(row[c] - mx) / sum;
        want[(h * T + r) * T + c] = pv;
        for (uint32_t d = 0; d < D; ++d) ov[(h * T + r) * D + d] += pv * vv[(h * T + c) * D + d];
      }
    }
  auto close = [&](const std::vector<float> &got, const std::vector<double> &ref,
                   const std::string &what) {
    double num = 0, den = 0;
    for (size_t i = 0; i < got.size(); ++i) {
      num += (got[i] - ref[i]) * (got[i] - ref[i]);
      den += ref[i] * ref[i];
    }
    require(std::sqrt(num / den) < 2e-3, what + ": relative error " +
                                             std::to_string(std::sqrt(num / den)));
  };
  const auto s0 = rt.stats();
  for (int it = 0; it < 3; ++it) {
    run(rt, forward);
    close(get(o), ov, "attention output");
  }
  const auto s1 = rt.stats();
  require(s1.flash_forward >= s0.flash_forward + 3, "the forward ran on the flash kernels");
  // the host reads P: it is written out from the recipe first
  close(get(p), want, "P read by the host");
  require(rt.stats().flash_rebuilt == s1.flash_rebuilt + 1, "P rebuilt for the host read");
  // an op of a later window reads P
  run(rt, forward);
  const auto s2 = rt.stats();
  run(rt, [&] { rt.add(p, p, p2); });
  require(rt.stats().flash_rebuilt == s2.flash_rebuilt + 1, "P rebuilt for the reading op");
  std::vector<double> twice(want.size());
  for (size_t i = 0; i < want.size(); ++i) twice[i] = 2 * want[i];
  close(get(p2), twice, "P read by a later op");
  // a window that writes the recipe's input first rebuilds P from the old one
  run(rt, forward);
  run(rt, [&] { rt.add(q, q, q); });
  close(get(p), want, "P kept across a change of Q");
  rt.set_flash_attention(1);
}

// A kernel wait that runs out inside a window: wait() throws
// std::runtime_error (src/my_metal/runtime.cpp:310-317 raises on command
// buffer errors), and the runtime keeps working afterwards.
void wait_timeout(cuda::Runtime &rt) {
  uint32_t *waited = nullptr;
  require(tl_malloc(reinterpret_cast<void **>(&waited), 16) == TL_OK, "scratch");
  rt.start();
  require(tl_check_wait_timeout(2000000, waited, cuda::stream()) == TL_OK, "launch");
  rt.submit();
  require(throws<std::runtime_error>([&] { rt.wait(); }), "wait() reports the timeout");
  tl_free(waited);
  Tensor a({2, 2}), b({2, 2}), c({2, 2});
  put(a, {1, 2, 3, 4});
  put(b, {1, 0, 0, 1});
  run(rt, [&] { rt.mult(a, b, c); });
  expect(c, {1, 2, 3, 4}, "runtime usable after a timeout");
}

}  // namespace

int main(int argc, char **argv) {
  cuda::init();
  const std::string only = argc > 1 ? argv[1] : "";
  int failures = 0;
  {
    cuda::Runtime rt;
    const std::vector<std::pair<const char *, void (*)(cuda::Runtime &)>> cases = {
        {"lifecycle", lifecycle},
        {"cleanup_idempotent", cleanup_idempotent},
        {"binary_chain", binary_chain},
        {"broadcasting", broadcasting},
        {"scalar_ops", scalar_ops},
        {"unary_ops", unary_ops},
        {"rms", rms},
        {"gelu", gelu},
        {"matmul", matmul},
        {"tiled_identity", tiled_identity},
        {"reductions", reductions},
        {"sum_to_shape_multi", sum_to_shape_multi},
        {"sum_to_shape_leading", sum_to_shape_leading},
        {"softmax", softmax},
        {"cross_entropy", cross_entropy},
        {"argmax", argmax},
        {"embedding", embedding},
        {"scatter_index", scatter_index},
        {"scatter_add_rows", scatter_add_rows},
        {"clipping", clipping},
        {"adamw", adamw},
        {"storage_semantics", storage_semantics},
        {"alias_safety", alias_safety},
        {"graph_replay", graph_replay},
        {"flash_attention_virtual_probs", flash_attention_virtual_probs},
        {"wait_timeout", wait_timeout},
    };
    for (const auto &[name, fn] : cases) {
      if (!only.empty() && only != name) continue;
      try {
        fn(rt);
        std::printf("PASS %s\n", name);
      } catch (const std::exception &e) {
        std::printf("FAIL %s: %s\n", name, e.what());
        ++failures;
      }
      std::fflush(stdout);
    }
  }
  cuda::shutdown();
  return failures ? 1 : 0;
}

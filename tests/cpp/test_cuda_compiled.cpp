// Compiled-graph tests on cuda::Runtime: the reference's passes::Compiled
// executor driving the CUDA backend through prepare/forward/backward/step.
// Cases follow the reference's tests/test_meta.cpp (generic cases
// :39-195, Metal-only block :197-380, closing graph :398-427) and the
// decoder-block gradient check of tests/test_attention.cpp:128-197
// (JTPuffer/TempLit), with the same expectations and tolerances.
#include "expr/api.h"
#include "my_cuda/runtime.h"
#include "my_cuda/storage.h"
#include "nn/attention.h"
#include "nn/decoder_block.h"
#include "nn/layer.h"
#include "optimiser/sgd.h"
#include "passes/compile.h"
#include "passes/get_at_path.h"

#include <cmath>
#include <cstdio>
#include <functional>
#include <random>
#include <span>
#include <stdexcept>
#include <string>
#include <vector>

using Mat = RTensor<cuda::CUDA, cuda::kernel_type>;
using IndexMat = RTensor<cuda::CUDA, cuda::index_type>;
using Runtime = cuda::Runtime;
using SGD = Optimiser::SGD<Mat>;

namespace {

struct Failure : std::runtime_error {
  using std::runtime_error::runtime_error;
};
void require(bool ok, const std::string &what) {
  if (!ok) throw Failure(what);
}
bool near(float a, float b, float eps) { return std::abs(a - b) < eps; }

struct CountingRuntime : Runtime {
  size_t hadamard_calls = 0;
  void hadamard(const Mat &a, const Mat &b, Mat &destination) {
    ++hadamard_calls;
    Runtime::hadamard(a, b, destination);
  }
};
static_assert(passes::Runnable<Mat, CountingRuntime>);

void gradient_context() {
  using Path = passes::graph_path<passes::graph_root, 0>;
  passes::GradientContext<Mat, passes::type_list<Path>> g;
  Runtime rt;
  require(!g.has_gradient<Path>(), "starts empty");
  g.for_each_slot([]<typename P>(auto &grad) { grad = Mat({1, 2}); });
  rt.start();
  g.accumulate<Path>(rt, Mat::from_values({{1.0f, 2.0f}}));
  g.accumulate<Path>(rt, Mat::from_values({{3.0f, 4.0f}}));
  rt.submit();
  rt.wait();
  require(g.has_gradient<Path>(), "has gradient");
  require(g.get_node<Path>() == Mat::from_values({{4.0f, 6.0f}}), "accumulated 4,6");
  g.clear();
  require(!g.has_gradient<Path>(), "cleared");
}

void rebinds_inputs() {
  Runtime rt;
  expr::tensor::GradTensor<Mat> lhs(Mat::from_values({{1.0f}}));
  expr::tensor::NoGradTensor<Mat> rhs(Mat::from_values({{2.0f}}));
  auto e = expr::add(lhs, rhs);
  auto c = passes::compile<Mat, SGD>(e, rt, SGD::generate_params(0.0f));
  c.prepare();
  require(c.forward().get(0, 0) == 3.0f, "1+2");
  passes::get_at_path<passes::graph_path<passes::graph_root, 0>>(e).set_value(
      Mat::from_values({{4.0f}}));
  require(c.forward().get(0, 0) == 6.0f, "4+2");
}

void recovers_after_failure() {
  Runtime rt;
  expr::tensor::NoGradTensor<Mat> lhs(Mat::from_values({{1.0f, 2.0f}}));
  expr::tensor::NoGradTensor<Mat> rhs(Mat::from_values({{1.0f, 2.0f, 3.0f}}));
  auto e = expr::add(lhs, rhs);
  auto c = passes::compile<Mat, SGD>(e, rt, SGD::generate_params(0.0f));
  bool threw = false;
  try {
    c.prepare();
  } catch (const std::invalid_argument &) {
    threw = true;
  }
  require(threw, "bad shapes throw at prepare");
  rhs.set_value(Mat::from_values({{3.0f, 4.0f}}));
  c.prepare();
  require(c.forward() == Mat::from_values({{4.0f, 6.0f}}), "recovered");
}

void let_evaluates_once() {
  CountingRuntime rt;
  expr::tensor::NoGradTensor<Mat> lhs(Mat::from_values({{1.0f, 2.0f}, {3.0f, 4.0f}}));
  expr::tensor::NoGradTensor<Mat> rhs(Mat::from_values({{5.0f, 6.0f}, {7.0f, 8.0f}}));
  auto value = expr::hadamard(lhs, rhs);
  auto reused = expr::let(value, [](auto input) { return expr::add(input, input); });
  auto e = expr::add(reused, rhs);
  auto c = passes::compile<Mat, SGD>(e, rt, SGD::generate_params(0.0f));
  c.prepare();
  rt.hadamard_calls = 0;
  const Mat r = c.forward();
  require(rt.hadamard_calls == 1, "let evaluated once");
  require(r == Mat::from_values({{15.0f, 30.0f}, {49.0f, 72.0f}}), "let value");
}

void let_local_gradient() {
  Runtime rt;
  expr::tensor::GradTensor<Mat> input(Mat::from_values({{2.0f}}));
  auto value = expr::hadamard(input, input);
  auto e = expr::let(value, [](auto local) { return expr::add(local, local); });
  auto c = passes::compile<Mat, SGD>(e, rt, SGD::generate_params(1.0f));
  c.prepare();
  require(c.forward().get(0, 0) == 8.0f, "forward 8");
  c.backward(Mat(1.0f));
  c.step();
  require(input.get_value().get(0, 0) == -6.0f, "2 - 8 = -6");
}

void sgd_updates_in_place() {
  Runtime rt;
  expr::tensor::GradTensor<Mat> p(Mat::from_values({{1.0f}}));
  expr::tensor::NoGradTensor<Mat> k(Mat::from_values({{2.0f}}));
  auto e = expr::add(p, k);
  auto c = passes::compile<Mat, SGD>(e, rt, SGD::generate_params(0.5f));
  c.prepare();
  require(c.forward().get(0, 0) == 3.0f, "forward");
  c.backward(Mat(1.0f));
  const auto *storage = p.get_value().get_storage();
  c.step();
  require(p.get_value().get_storage() == storage, "updated in place");
  require(c.forward().get(0, 0) == 2.5f, "after step");
}

void attention_shape_ops() {
  Runtime rt;
  Mat v({1, 3, 4});
  v.set(std::vector<float>{1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12});
  expr::tensor::NoGradTensor<Mat> input(std::move(v));
  auto split = expr::split_last_dim<2, 2>(input);
  auto heads = expr::transpose<1, 2>(split);
  auto ch = passes::compile<Mat, SGD>(heads, rt, SGD::generate_params(0.0f));
  ch.prepare();
  const auto hr = ch.forward();
  require(hr.shape() == std::vector<uint32_t>{1, 2, 3, 2}, "heads shape");
  Mat expect({1, 2, 3, 2});
  expect.set(std::vector<float>{1, 2, 5, 6, 9, 10, 3, 4, 7, 8, 11, 12});
  require(hr == expect, "heads values");
  auto ordered = expr::transpose<1, 2>(std::move(heads));
  auto merged = expr::merge_last_dims<2, 2>(std::move(ordered));
  auto cm = passes::compile<Mat, SGD>(merged, rt, SGD::generate_params(0.0f));
  cm.prepare();
  const auto mr = cm.forward();
  require(mr.shape() == std::vector<uint32_t>{1, 3, 4}, "merged shape");
  require(mr == input.get_value(), "round trip");
}

void rms_expressions() {
  Runtime rt;
  Mat iv({2, 2});
  iv.set(std::vector<float>{3.0f, 4.0f, 0.0f, 0.0f});
  expr::tensor::NoGradTensor<Mat> input(std::move(iv));
  auto cr = passes::compile<Mat, SGD>(expr::rms(input), rt, SGD::generate_params(0.0f));
  cr.prepare();
  const float first = std::sqrt(12.5f + 1e-6f);
  Mat r = cr.forward();
  require(near(r.get(0, 0), first, 1e-5f) && near(r.get(1, 0), 1e-3f, 1e-5f), "rms");
  auto cn = passes::compile<Mat, SGD>(expr::rms_norm(input), rt, SGD::generate_params(0.0f));
  cn.prepare();
  Mat n = cn.forward();
  require(near(n.get(0, 0), 3.0f / first, 1e-5f) && near(n.get(0, 1), 4.0f / first, 1e-5f) &&
              near(n.get(1, 0), 0.0f, 1e-5f) && near(n.get(1, 1), 0.0f, 1e-5f),
          "rmsnorm");

  expr::tensor::GradTensor<Mat> gi(Mat::from_values({{3.0f, 4.0f}}));
  auto cg = passes::compile<Mat, SGD>(expr::rms(gi), rt, SGD::generate_params(1.0f));
  cg.prepare();
  cg.forward();
  cg.backward(Mat(1.0f));
  cg.step();
  const float rms = std::sqrt(12.5f + 1e-6f);
  require(near(gi.get_value().get(0, 0), 3.0f - 3.0f / (2.0f * rms), 1e-5f) &&
              near(gi.get_value().get(0, 1), 4.0f - 4.0f / (2.0f * rms), 1e-5f),
          "rms gradient");

  expr::tensor::GradTensor<Mat> ni(Mat::from_values({{3.0f, 4.0f}}));
  auto cng = passes::compile<Mat, SGD>(expr::rms_norm(ni), rt, SGD::generate_params(1.0f));
  cng.prepare();
  Mat out = cng.forward();
  cng.backward(Mat::from_values({{1.0f, 2.0f}}));
  cng.step();
  const float mean = (out.get(0, 0) + 2.0f * out.get(0, 1)) / 2.0f;
  const float g0 = (1.0f - out.get(0, 0) * mean) / rms;
  const float g1 = (2.0f - out.get(0, 1) * mean) / rms;
  require(near(ni.get_value().get(0, 0), 3.0f - g0, 1e-5f) &&
              near(ni.get_value().get(0, 1), 4.0f - g1, 1e-5f),
          "rmsnorm gradient");
}

void embedding_sgd() {
  Runtime rt;
  expr::tensor::GradTensor<Mat> w(
      Mat::from_values({{1, 2, 3}, {4, 5, 6}, {7, 8, 9}, {10, 11, 12}}));
  IndexMat iv({2, 2});
  iv.set(std::vector<uint32_t>{2, 0, 2, 1});
  expr::tensor::NoGradTensor<IndexMat> ids(std::move(iv));
  auto c = passes::compile<Mat, SGD>(expr::embedding_lookup(w, ids), rt, SGD::generate_params(0.5f));
  c.prepare();
  Mat expect({2, 2, 3});
  expect.set(std::vector<float>{7, 8, 9, 1, 2, 3, 7, 8, 9, 4, 5, 6});
  require(c.forward() == expect, "embedding forward");
  Mat rg({2, 2, 3});
  rg.set(std::vector<float>(12, 1.0f));
  c.backward(rg);
  c.step();
  require(w.get_value() ==
              Mat::from_values({{0.5f, 1.5f, 2.5f}, {3.5f, 4.5f, 5.5f}, {6.0f, 7.0f, 8.0f},
                                {10.0f, 11.0f, 12.0f}}),
          "embedding SGD through scatter");
}

float gelu_d(float x) {
  const float a = 0.7978845608f, b = 0.044715f, x2 = x * x;
  const float t = std::tanh(a * (x + b * x2 * x));
  return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * a * (1.0f + 3.0f * b * x2);
}

void gelu_backward() {
  Runtime rt;
  expr::tensor::GradTensor<Mat> input(Mat::from_values({{-1.0f, 0.0f, 1.0f}}));
  auto c = passes::compile<Mat, SGD>(expr::gelu(input), rt, SGD::generate_params(1.0f));
  c.prepare();
  c.forward();
  c.backward(Mat::from_values({{1.0f, 1.0f, 1.0f}}));
  c.step();
  require(near(input.get_value().get(0, 0), -1.0f - gelu_d(-1.0f), 1e-5f) &&
              near(input.get_value().get(0, 1), 0.0f - gelu_d(0.0f), 1e-5f) &&
              near(input.get_value().get(0, 2), 1.0f - gelu_d(1.0f), 1e-5f),
          "gelu backward");
}

void cross_entropy_backward() {
  Runtime rt;
  expr::tensor::GradTensor<Mat> logits(Mat::from_values({{1.0f, 2.0f, 3.0f}, {1.0f, 1.0f, 1.0f}}));
  IndexMat tv({2});
  tv.set(std::vector<uint32_t>{2, 0});
  expr::tensor::NoGradTensor<IndexMat> targets(std::move(tv));
  auto c = passes::compile<Mat, SGD>(expr::loss::cross_entropy(logits, targets), rt,
                                     SGD::generate_params(1.0f));
  c.prepare();
  Mat losses = c.forward();
  require(losses.shape() == std::vector<uint32_t>{2, 1}, "loss shape");
  const float den = std::exp(-2.0f) + std::exp(-1.0f) + 1.0f;
  const float lo = std::exp(-2.0f) / den, mid = std::exp(-1.0f) / den, hi = 1.0f / den;
  require(near(losses.get(0, 0), std::log(den), 1e-4f) &&
              near(losses.get(1, 0), std::log(3.0f), 1e-4f),
          "losses");
  Mat rg({2, 1});
  rg.set(std::vector<float>{2.0f, 0.5f});
  c.backward(rg);
  c.step();
  Mat &u = logits.get_value();
  require(near(u.get(0, 0), 1.0f - 2.0f * lo, 1e-4f) && near(u.get(0, 1), 2.0f - 2.0f * mid, 1e-4f) &&
              near(u.get(0, 2), 3.0f - 2.0f * (hi - 1.0f), 1e-4f) &&
              near(u.get(1, 0), 1.0f + 1.0f / 3.0f, 1e-4f) &&
              near(u.get(1, 1), 1.0f - 1.0f / 6.0f, 1e-4f) &&
              near(u.get(1, 2), 1.0f - 1.0f / 6.0f, 1e-4f),
          "cross entropy backward with root gradient");
}

void closing_graph() {
  Runtime rt;
  std::mt19937 gen(1);
  nn::Layer<Mat> query(128, 64, gen);
  expr::tensor::GradTensor input(Mat({1, 128}));
  expr::tensor::GradTensor input_1(Mat({64, 1}));
  input.get_value().set(std::vector<float>(128, 0.01f));
  input_1.get_value().set(std::vector<float>(64, 0.02f));
  auto scores = expr::mult(query(input), input_1);
  auto probabilities = expr::softmax(expr::sqrt(expr::sigmoid(scores)));
  auto normalised = expr::divide(expr::hadamard(probabilities, probabilities), probabilities);
  auto loss = expr::loss::sqe(normalised, probabilities);
  auto c = passes::compile<Mat, SGD>(loss, rt, SGD::generate_params(0.0f));
  c.prepare();
  auto r = c.forward();
  require(r.shape() == std::vector<uint32_t>{1, 1}, "loss shape");
  Mat rg(1.0f);
  c.zero_grad();
  c.backward(rg);
  c.backward(rg);
  c.zero_grad();
}

template <typename T> class GradientRecorder {
public:
  struct Shared {};
  inline static std::vector<std::vector<float>> gradients;
  template <typename Run> void update(Run &, const Shared &, const T &, const T &g, T &) {
    auto &v = gradients.emplace_back(g.numel());
    g.read(std::span(v));
  }
};

void decoder_block_gradients_distinct() {
  using Recorder = GradientRecorder<Mat>;
  constexpr uint32_t B = 1, T = 3, D = 8;
  Runtime rt;
  expr::tensor::NoGradTensor<Mat> input(Mat({B, T, D}));
  expr::tensor::NoGradTensor<Mat> mask(nn::causal_mask<cuda::CUDA, float>(T, T));
  std::mt19937 gen(7);
  nn::DecoderBlock<Mat, D, 2> block(gen);
  auto output = block(input, mask);
  auto c = passes::compile<Mat, Recorder>(output, rt, Recorder::Shared{});
  c.prepare();
  size_t identical = 0;
  for (size_t s = 0; s < 3; ++s) {
    std::vector<float> iv(B * T * D), gv(B * T * D);
    for (size_t i = 0; i < iv.size(); ++i) {
      iv[i] = float((s + 1) * (i + 1)) / 31.0f;
      gv[i] = float((s + 2) * (i + 3)) / 29.0f;
    }
    Mat x({B, T, D});
    x.set(iv);
    input.set_value(std::move(x));
    Mat rg({B, T, D});
    rg.set(gv);
    c.zero_grad();
    (void)c.forward();
    c.backward(rg);
    Recorder::gradients.clear();
    c.step();
    require(Recorder::gradients.size() == 12, "all 12 parameter gradients");
    for (const auto &g : Recorder::gradients)
      for (float v : g) require(std::isfinite(v), "finite gradients");
    if (Recorder::gradients[3] == Recorder::gradients[11]) ++identical;
  }
  require(identical == 0, "mlp_2 and attention output bias gradients differ");
}

}  // namespace

int main(int argc, char **argv) {
  cuda::init();
  const std::string only = argc > 1 ? argv[1] : "";
  int failures = 0;
  const std::vector<std::pair<const char *, void (*)()>> cases = {
      {"gradient_context", gradient_context},
      {"rebinds_inputs", rebinds_inputs},
      {"recovers_after_failure", recovers_after_failure},
      {"let_evaluates_once", let_evaluates_once},
      {"let_local_gradient", let_local_gradient},
      {"sgd_updates_in_place", sgd_updates_in_place},
      {"attention_shape_ops", attention_shape_ops},
      {"rms_expressions", rms_expressions},
      {"embedding_sgd", embedding_sgd},
      {"gelu_backward", gelu_backward},
      {"cross_entropy_backward", cross_entropy_backward},
      {"closing_graph", closing_graph},
      {"decoder_block_gradients_distinct", decoder_block_gradients_distinct},
  };
  for (const auto &[name, fn] : cases) {
    if (!only.empty() && only != name) continue;
    try {
      fn();
      std::printf("PASS %s\n", name);
    } catch (const std::exception &e) {
      std::printf("FAIL %s: %s\n", name, e.what());
      ++failures;
    }
    std::fflush(stdout);
  }
  cuda::shutdown();
  return failures ? 1 : 0;
}

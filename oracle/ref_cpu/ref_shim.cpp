// TEST INFRASTRUCTURE: a C ABI over the reference's own CPU runtime
// (src/CPU/cpu.cpp and include/CPU/runtime.h of JTPuffer/TempLit, compiled
// from the reference sources by oracle/ref_cpu/Makefile into
// oracle/_ref/libref_cpu.so).  Used to pin the oracle and as the
// "reference" CPU baseline; never linked by the product.
//
//  * ref_op: one rank-2 op of cpu:: (mult, add, sub, hadamard, divide,
//    softmax, sum_to_shape, transpose, sigmoid, sqrt) on host arrays.
//  * ref_mlp_train: the configuration-1 MLP training loop (sigmoid hidden
//    layer, squared-error loss, SGD) compiled by passes::compile onto
//    cpu::Runtime, exactly the reference's compiled path.
#include "CPU/runtime.h"
#include "expr/api.h"
#include "optimiser/sgd.h"
#include "passes/compile.h"

#include <chrono>
#include <cstdint>
#include <cstring>
#include <span>
#include <string>
#include <vector>

namespace {

using Mat = RTensor<cpu::CPU, float>;

Mat make(const float *data, uint32_t rows, uint32_t cols) {
  Mat m({rows, cols});
  m.set(std::span<const float>(data, static_cast<size_t>(rows) * cols));
  return m;
}

void store(const Mat &m, float *out) {
  std::vector<float> v(m.numel());
  m.read(v);
  std::memcpy(out, v.data(), v.size() * sizeof(float));
}

thread_local std::string g_error;

}  // namespace

extern "C" {

const char *ref_last_error(void) { return g_error.c_str(); }

// op: 0 mult, 1 add, 2 sub, 3 hadamard, 4 divide, 5 softmax, 6 sum_to_shape,
// 7 transpose, 8 sigmoid, 9 sqrt.  a is [ar, ac], b is [br, bc] (binary ops),
// out has [or, oc] (given for sum_to_shape and the broadcast ops).
int ref_op(int op, const float *a, uint32_t ar, uint32_t ac, const float *b, uint32_t br,
           uint32_t bc, float *out, uint32_t orows, uint32_t ocols) {
  try {
    cpu::Runtime rt;
    Mat A = make(a, ar, ac);
    Mat O({orows, ocols});
    switch (op) {
      case 0: rt.mult(A, make(b, br, bc), O); break;
      case 1: rt.add(A, make(b, br, bc), O); break;
      case 2: rt.sub(A, make(b, br, bc), O); break;
      case 3: rt.hadamard(A, make(b, br, bc), O); break;
      case 4: rt.divide(A, make(b, br, bc), O); break;
      case 5: rt.softmax(A, O); break;
      case 6: {
        const std::vector<uint32_t> shape{orows, ocols};
        rt.sum_to_shape(A, shape, O);
        break;
      }
      case 7: rt.transpose(A, O); break;
      case 8: rt.sigmoid(A, O); break;
      case 9: rt.sqrt(A, O); break;
      default: g_error = "unknown op"; return 1;
    }
    store(O, out);
    return 0;
  } catch (const std::exception &e) {
    g_error = e.what();
    return 1;
  }
}

// Configuration-1 MLP: loss = sqe(linear(sigmoid(linear(X, W1, b1)), W2, b2), Y)
// with root gradient `root` everywhere and SGD(lr) for `steps` iterations.
// Weights are updated in place; losses[s] receives the summed loss of step s;
// *seconds the wall time of the training loop.
int ref_mlp_train(const float *X, uint32_t batch, uint32_t in, uint32_t hidden, uint32_t outd,
                  float *W1, float *b1, float *W2, float *b2, const float *Y, float root,
                  float lr, int steps, float *losses, double *seconds) {
  try {
    using SGD = Optimiser::SGD<Mat>;
    cpu::Runtime rt;
    expr::tensor::NoGradTensor<Mat> x(make(X, batch, in));
    expr::tensor::NoGradTensor<Mat> y(make(Y, batch, outd));
    expr::tensor::GradTensor<Mat> w1(make(W1, in, hidden)), bb1(make(b1, 1, hidden));
    expr::tensor::GradTensor<Mat> w2(make(W2, hidden, outd)), bb2(make(b2, 1, outd));
    auto h = expr::sigmoid(expr::linear(x, w1, bb1));
    auto loss = expr::loss::sqe(expr::linear(h, w2, bb2), y);
    auto compiled = passes::compile<Mat, SGD>(loss, rt, SGD::generate_params(lr));
    compiled.prepare();
    Mat rg({batch, outd});
    rg.set(std::vector<float>(static_cast<size_t>(batch) * outd, root));
    std::vector<float> lv(static_cast<size_t>(batch) * outd);
    const auto t0 = std::chrono::steady_clock::now();
    for (int s = 0; s < steps; ++s) {
      compiled.zero_grad();
      const Mat l = compiled.forward();
      l.read(lv);
      double acc = 0;
      for (float v : lv) acc += v;
      if (losses) losses[s] = static_cast<float>(acc);
      compiled.backward(rg);
      compiled.step();
    }
    const auto t1 = std::chrono::steady_clock::now();
    if (seconds) *seconds = std::chrono::duration<double>(t1 - t0).count();
    store(w1.get_value(), W1);
    store(bb1.get_value(), b1);
    store(w2.get_value(), W2);
    store(bb2.get_value(), b2);
    return 0;
  } catch (const std::exception &e) {
    g_error = e.what();
    return 1;
  }
}

}  // extern "C"

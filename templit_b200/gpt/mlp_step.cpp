// Configuration 1 of the benchmark suite on cuda::Runtime: the MLP training
// loop (sigmoid hidden layer, squared-error loss, SGD) compiled by the
// reference's passes::compile, as the reference compiles it for its CPU
// runtime.  Exported through include/templit_gpt.h (tlg_mlp_train).
#include "templit_gpt.h"

#include "expr/api.h"
#include "my_cuda/runtime.h"
#include "my_cuda/storage.h"
#include "optimiser/sgd.h"
#include "passes/compile.h"

#include <chrono>
#include <cstring>
#include <span>
#include <string>
#include <vector>

namespace {

using Mat = RTensor<cuda::CUDA, cuda::kernel_type>;
thread_local std::string g_mlp_error;

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

}  // namespace

extern "C" int tlg_mlp_train(const float *X, uint32_t batch, uint32_t in, uint32_t hidden,
                             uint32_t outd, float *W1, float *b1, float *W2, float *b2,
                             const float *Y, float root, float lr, int steps, int gemm_precision,
                             float *losses, double *seconds) {
  try {
    using SGD = Optimiser::SGD<Mat>;
    cuda::init();
    cuda::Runtime rt;
    rt.set_gemm_precision(gemm_precision);
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
    cuda::synchronize();
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
    cuda::synchronize();
    const auto t1 = std::chrono::steady_clock::now();
    if (seconds) *seconds = std::chrono::duration<double>(t1 - t0).count();
    store(w1.get_value(), W1);
    store(bb1.get_value(), b1);
    store(w2.get_value(), W2);
    store(bb2.get_value(), b2);
    return 0;
  } catch (const std::exception &e) {
    g_mlp_error = e.what();
    return 1;
  }
}

extern "C" const char *tlg_mlp_last_error(void) { return g_mlp_error.c_str(); }

// Forward-only GPT inference over any TempLit runtime, as src/generate.cpp
// (JTPuffer/TempLit) sets it up: a batch-1 nn::GPT whose logits graph is
// compiled on its own (generate.cpp:57-69), driven token by token by the
// reference's inference::autoregression (include/inference.h:45-97: the
// whole context recomputed per token, top-k sampling on the host from
// logits.get()).  Instantiated for cuda::Runtime by gpt_step.cpp and for
// the host oracle by oracle/cpu_gpt.
#pragma once

#include "gpt_driver.h"
#include "inference.h"

#include <random>
#include <span>
#include <vector>

namespace templit_b200 {

struct InferBase {
  virtual ~InferBase() = default;
  // logits [seq, vocab] of one window of `seq` tokens
  virtual void logits(const uint32_t *tokens, float *out) = 0;
  // tokens emitted by inference::autoregression (at most max_out kept);
  // returns how many it emitted
  virtual uint32_t generate(const uint32_t *prompt, uint32_t n, uint32_t eos, uint32_t seed,
                            uint32_t top_k, float temperature, uint32_t min_length,
                            uint32_t *out, uint32_t max_out) = 0;
  virtual void params(std::vector<float> &out, uint32_t &tensors) = 0;
  virtual void set_params(const float *in, uint64_t count) = 0;
};

template <typename Mat, typename Run, typename Model>
class InferDriver final : public InferBase {
  using IndexMat = typename Mat::template rebind<uint32_t>;
  using Opt = Optimiser::AdamW<Mat>;
  using Indices = expr::tensor::Tensor<IndexMat>;
  using Graph = decltype(std::declval<const Model &>()(std::declval<Indices &>()));
  using CompiledT = passes::Compiled<Mat, std::remove_cvref_t<Graph>, Run, Opt>;

  tlg_config cfg_;
  Run &runtime_;
  Indices input_;
  std::mt19937 gen_;
  Model model_;
  std::unique_ptr<CompiledT> compiled_;

  static std::unique_ptr<CompiledT> build(const Model &model, Indices &input, Run &runtime) {
    // generate.cpp:63-66: the optimiser is part of the compiled type only
    return std::make_unique<CompiledT>(model(input), runtime, Opt::generate_params(0.0001f));
  }

public:
  InferDriver(const tlg_config &c, Run &runtime)
      : cfg_(c), runtime_(runtime), input_(IndexMat({1, c.seq})), gen_(c.seed),
        model_(1, c.seq, gen_), compiled_(build(model_, input_, runtime_)) {
    input_.get_value().set(std::vector<uint32_t>(c.seq, 0));
    compiled_->prepare();
    if (c.init_std > 0.0f) redraw_compiled(*compiled_, c.seed, c.init_std);
  }

  void logits(const uint32_t *tokens, float *out) override {
    input_.get_value().set(std::span<const uint32_t>(tokens, cfg_.seq));
    const Mat l = compiled_->forward();
    l.read(std::span<float>(out, l.numel()));
  }

  uint32_t generate(const uint32_t *prompt, uint32_t n, uint32_t eos, uint32_t seed,
                    uint32_t top_k, float temperature, uint32_t min_length, uint32_t *out,
                    uint32_t max_out) override {
    uint32_t emitted = 0;
    inference::autoregression(*compiled_, input_, std::span<const uint32_t>(prompt, n), eos,
                              std::mt19937(seed), top_k, temperature, min_length,
                              [&](uint32_t token) {
                                if (emitted < max_out) out[emitted] = token;
                                ++emitted;
                              });
    return emitted;
  }

  void params(std::vector<float> &out, uint32_t &tensors) override {
    compiled_params(*compiled_, out, tensors);
  }
  void set_params(const float *in, uint64_t count) override {
    set_compiled_params(*compiled_, in, count);
  }
};

}  // namespace templit_b200

// GPT training driver over any TempLit runtime: builds the model, the
// cross-entropy loss and the AdamW optimiser and compiles them with
// passes::compile exactly as src/train.cpp:89-113 (JTPuffer/TempLit) does,
// then runs the loop body of train.cpp:120-157 one iteration at a time.
// Instantiated for cuda::Runtime by gpt_step.cpp.
#pragma once

#include "expr/cross-entropy.h"
#include "nn/GPT.h"
#include "optimiser/AdamW.h"
#include "passes/compile.h"
#include "templit_gpt.h"

#include <cmath>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <random>
#include <span>
#include <stdexcept>
#include <string>
#include <vector>

namespace templit_b200 {

// Flat in-memory archive (WritableArchive + ReadableArchive with scopes) used
// to move parameters in and out through Compiled::save / Compiled::load, and
// checkpoints in the file layout of the reference's Archive
// (src/model_utils/archive.cpp:33-73): entries `scope/.../name`, each as
// u32 name length, name bytes, u32 blob length, blob (host byte order).
class FlatArchive {
  std::map<std::string, std::vector<std::byte>> *store_;
  std::string prefix_;

public:
  using Store = std::map<std::string, std::vector<std::byte>>;
  explicit FlatArchive(std::map<std::string, std::vector<std::byte>> *s, std::string p = "")
      : store_(s), prefix_(std::move(p)) {}
  void write(const std::string &name, std::span<const std::byte> v) {
    (*store_)[prefix_ + name].assign(v.begin(), v.end());
  }

  // Writes every entry (any order is valid: the reference restores by name).
  static void commit(const Store &store, std::ostream &out) {
    for (const auto &[name, blob] : store) {
      const uint32_t name_len = static_cast<uint32_t>(name.size());
      const uint32_t blob_len = static_cast<uint32_t>(blob.size());
      if (name_len != name.size() || blob_len != blob.size())
        throw std::runtime_error("archive entry too large: " + name);
      out.write(reinterpret_cast<const char *>(&name_len), sizeof(name_len));
      out.write(name.data(), static_cast<std::streamsize>(name.size()));
      out.write(reinterpret_cast<const char *>(&blob_len), sizeof(blob_len));
      out.write(reinterpret_cast<const char *>(blob.data()),
                static_cast<std::streamsize>(blob.size()));
    }
    if (!out) throw std::runtime_error("checkpoint write failed");
  }

  // Reads entries until the stream ends (a truncated last entry is dropped,
  // as the reference's Archive::restore does).
  static void restore(Store &store, std::istream &in) {
    for (;;) {
      uint32_t name_len = 0, blob_len = 0;
      if (!in.read(reinterpret_cast<char *>(&name_len), sizeof(name_len))) break;
      std::string name(name_len, '\0');
      if (!in.read(name.data(), name_len)) break;
      if (!in.read(reinterpret_cast<char *>(&blob_len), sizeof(blob_len))) break;
      std::vector<std::byte> blob(blob_len);
      if (!in.read(reinterpret_cast<char *>(blob.data()), blob_len)) break;
      store[name] = std::move(blob);
    }
  }
  void read(const std::string &name, std::span<std::byte> v) const {
    auto it = store_->find(prefix_ + name);
    if (it == store_->end() || it->second.size() != v.size())
      throw std::runtime_error("archive entry missing or mis-sized: " + prefix_ + name);
    std::memcpy(v.data(), it->second.data(), v.size());
  }
  FlatArchive scope(const std::string &name) const { return FlatArchive(store_, prefix_ + name + "/"); }
};

// Every parameter of a compiled network (Compiled::save order) as one flat
// float array; `tensors` = how many parameter tensors.
template <typename C>
void compiled_params(C &compiled, std::vector<float> &out, uint32_t &tensors) {
  std::map<std::string, std::vector<std::byte>> store;
  FlatArchive ar(&store);
  compiled.save(ar);
  out.clear();
  tensors = 0;
  for (;; ++tensors) {
    auto it = store.find("parameters/" + std::to_string(tensors) + "/data");
    if (it == store.end()) break;
    const size_t n = it->second.size() / sizeof(float);
    const size_t o = out.size();
    out.resize(o + n);
    std::memcpy(out.data() + o, it->second.data(), it->second.size());
  }
}

template <typename C>
void set_compiled_params(C &compiled, const float *in, uint64_t count) {
  std::map<std::string, std::vector<std::byte>> store;
  FlatArchive ar(&store);
  compiled.save(ar);
  uint64_t off = 0;
  for (uint32_t i = 0;; ++i) {
    auto it = store.find("parameters/" + std::to_string(i) + "/data");
    if (it == store.end()) break;
    const size_t n = it->second.size() / sizeof(float);
    if (off + n > count) throw std::invalid_argument("too few parameter values");
    std::memcpy(it->second.data(), in + off, n * sizeof(float));
    off += n;
  }
  if (off != count) throw std::invalid_argument("parameter count mismatch");
  compiled.load(ar);
}

// Re-draws every weight N(0, std) (std::mt19937(seed + 7919)) and zeroes
// every bias ([1, n] tensors): the synthetic initialisation of the
// benchmark configurations.
template <typename C>
void redraw_compiled(C &compiled, uint32_t seed, float std) {
  std::vector<float> all;
  uint32_t tensors = 0;
  compiled_params(compiled, all, tensors);
  std::map<std::string, std::vector<std::byte>> store;
  FlatArchive ar(&store);
  compiled.save(ar);
  std::normal_distribution<float> dist(0.0f, std);
  std::mt19937 g(seed + 7919u);
  size_t off = 0;
  for (uint32_t i = 0; i < tensors; ++i) {
    const std::string key = "parameters/" + std::to_string(i) + "/";
    const auto &size = store[key + "size"];
    std::vector<uint32_t> shape(size.size() / 4);
    std::memcpy(shape.data(), size.data(), size.size());
    size_t n = 1;
    for (uint32_t d : shape) n *= d;
    const bool bias = shape.size() == 2 && shape[0] == 1;
    for (size_t j = 0; j < n; ++j) all[off + j] = bias ? 0.0f : dist(g);
    off += n;
  }
  set_compiled_params(compiled, all.data(), all.size());
}

struct DriverBase {
  virtual ~DriverBase() = default;
  virtual void set_batch(const uint32_t *tokens, const uint32_t *targets) = 0;
  virtual float train_step() = 0;
  virtual void forward(float *losses) = 0;
  virtual void params(std::vector<float> &out, uint32_t &tensors) = 0;
  virtual void set_params(const float *in, uint64_t count) = 0;
  // Checkpoint of the parameters (and the AdamW state) in the reference's
  // archive format, through Compiled::save / save_optimisers.
  virtual void save(const std::string &path, bool optimiser) = 0;
  virtual void load(const std::string &path, bool optimiser) = 0;
};

template <typename Mat, typename Run, typename Model>
class GptDriver final : public DriverBase {
  using IndexMat = typename Mat::template rebind<uint32_t>;
  using Opt = Optimiser::AdamW<Mat>;
  using Indices = expr::tensor::Tensor<IndexMat>;
  using Loss = decltype(expr::loss::cross_entropy(std::declval<const Model &>()(std::declval<Indices &>()),
                                                  std::declval<Indices &>()));
  using CompiledT = passes::Compiled<Mat, std::remove_cvref_t<Loss>, Run, Opt>;

  tlg_config cfg_;
  Run &runtime_;
  Indices input_;
  Indices targets_;
  std::mt19937 gen_;
  Model model_;
  std::unique_ptr<CompiledT> compiled_;
  Mat root_grad_;
  std::vector<float> losses_;
  uint32_t micro_;                         // forward / backward passes per step
  std::vector<uint32_t> tokens_, targets_host_;  // all micro-batches of a step

  static std::unique_ptr<CompiledT> build(const Model &model, Indices &input, Indices &targets,
                                          Run &runtime, const tlg_config &c) {
    auto graph = model(input);
    auto loss = expr::loss::cross_entropy(std::move(graph), targets);
    auto params = Opt::generate_params(c.lr, c.beta1, c.beta2, c.eps, c.weight_decay);
    return std::make_unique<CompiledT>(std::move(loss), runtime, std::move(params));
  }

public:
  GptDriver(const tlg_config &c, Run &runtime)
      : cfg_(c), runtime_(runtime), input_(IndexMat({c.batch, c.seq})),
        targets_(IndexMat({c.batch, c.seq})), gen_(c.seed), model_(c.batch, c.seq, gen_),
        compiled_(build(model_, input_, targets_, runtime_, c)),
        root_grad_(Mat({c.batch, c.seq, 1})),
        losses_(static_cast<size_t>(c.batch) * c.seq),
        micro_(c.micro_batches > 1 ? c.micro_batches : 1) {
    // zero ids so prepare() sees valid inputs
    std::vector<uint32_t> zeros(losses_.size(), 0);
    input_.get_value().set(zeros);
    targets_.get_value().set(zeros);
    compiled_->prepare();
    const float world = static_cast<float>(c.world ? c.world : 1);
    root_grad_.set(std::vector<float>(
        losses_.size(), 1.0f / (static_cast<float>(losses_.size()) * world *
                                static_cast<float>(micro_))));
    if (c.init_std > 0.0f) redraw(c.init_std);
  }

  void redraw(float std) { redraw_compiled(*compiled_, cfg_.seed, std); }

  void set_batch(const uint32_t *tokens, const uint32_t *targets) override {
    const size_t n = losses_.size();
    if (micro_ > 1) {  // kept on the host; each pass loads its slice
      tokens_.assign(tokens, tokens + n * micro_);
      targets_host_.assign(targets, targets + n * micro_);
      return;
    }
    input_.get_value().set(std::span<const uint32_t>(tokens, n));
    targets_.get_value().set(std::span<const uint32_t>(targets, n));
  }

  // The reference loop body (src/train.cpp:120-157): zero_grad, forward,
  // read the losses, backward, step.  The losses are read after the
  // backward and optimiser windows are queued (nothing in them writes the
  // loss tensor), so with a deferred wait the host records those windows
  // while the GPU still runs the forward pass.
  float train_step() override {
    if (micro_ > 1) return train_step_micro();
    compiled_->zero_grad();
    const Mat loss = compiled_->forward();
    compiled_->backward(root_grad_);
    if (cfg_.clip > 0.0f) compiled_->step(cfg_.clip);
    else compiled_->step();
    loss.read(losses_);
    double acc = 0.0;
    for (float v : losses_) acc += v;
    return static_cast<float>(acc / static_cast<double>(losses_.size()));
  }

  // Gradient accumulation: one zero_grad, micro_ forward / backward passes
  // (later backward calls add to the gradients, include/passes/context.h:
  // 74-89) with root gradient 1 / (all tokens of the step), one step.
  float train_step_micro() {
    const size_t n = losses_.size();
    if (tokens_.size() != n * micro_) throw std::logic_error("no batch set for the step");
    compiled_->zero_grad();
    double acc = 0.0;
    for (uint32_t m = 0; m < micro_; ++m) {
      input_.get_value().set(std::span<const uint32_t>(tokens_.data() + m * n, n));
      targets_.get_value().set(std::span<const uint32_t>(targets_host_.data() + m * n, n));
      const Mat loss = compiled_->forward();
      compiled_->backward(root_grad_);
      loss.read(losses_);
      for (float v : losses_) acc += v;
    }
    if (cfg_.clip > 0.0f) compiled_->step(cfg_.clip);
    else compiled_->step();
    return static_cast<float>(acc / static_cast<double>(n * micro_));
  }

  void forward(float *losses) override {
    const Mat loss = compiled_->forward();
    loss.read(std::span<float>(losses, losses_.size()));
  }

  void params(std::vector<float> &out, uint32_t &tensors) override {
    compiled_params(*compiled_, out, tensors);
  }

  void set_params(const float *in, uint64_t count) override {
    set_compiled_params(*compiled_, in, count);
  }

  // Any archive type of the reference (include/model_utils/archive_concepts.h).
  template <typename A> void save_archive(A &ar, bool optimiser) {
    compiled_->save(ar);
    if (optimiser) compiled_->save_optimisers(ar);
  }
  template <typename A> void load_archive(A &ar, bool optimiser) {
    compiled_->load(ar);
    if (optimiser) compiled_->load_optimisers(ar);
  }

  void save(const std::string &path, bool optimiser) override {
    FlatArchive::Store store;
    FlatArchive ar(&store);
    save_archive(ar, optimiser);
    std::ofstream out(path, std::ios::binary);
    if (!out) throw std::runtime_error("cannot open " + path);
    FlatArchive::commit(store, out);
  }

  void load(const std::string &path, bool optimiser) override {
    std::ifstream in(path, std::ios::binary);
    if (!in) throw std::runtime_error("cannot open " + path);
    FlatArchive::Store store;
    FlatArchive::restore(store, in);
    FlatArchive ar(&store);
    load_archive(ar, optimiser);
  }
};

}  // namespace templit_b200

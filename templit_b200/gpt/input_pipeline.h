// Token input pipeline of the training loop (src/train.cpp:75-77,142-144):
// the reference's Dataset::load_tokens (a raw file of host-order uint32
// tokens, model_utils/dataset.cpp:65-82), its split after the training
// fraction at the next end-of-text token (id 256, dataset.cpp:16-40) and
// Loader::get_batch (model_utils/loader.cpp:23-43: per sequence a start
// drawn by std::uniform_int_distribution<size_t>(0, n - T - 1) from a
// std::mt19937, inputs = tokens[s, s + T), targets = tokens[s + 1, s + T + 1)),
// restated so the same seed draws the same batches.  A background thread
// draws batch i + 1 into pinned host memory while batch i is in use, so the
// copy to the device (Storage::set) is asynchronous and never waits for the
// previous training step.
#pragma once

#include "templit_cuda.h"

#include <algorithm>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <iterator>
#include <mutex>
#include <random>
#include <span>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace templit_b200 {

class TokenPipeline {
public:
  static constexpr uint32_t kEndOfText = 256;

  TokenPipeline(const std::string &path, double training_fraction, bool validation,
                uint32_t batch, uint32_t seq, uint32_t seed)
      : gen_(seed), batch_(batch), seq_(seq) {
    if (batch == 0 || seq == 0) throw std::invalid_argument("batch dimensions must be non-zero");
    load(path);
    split(training_fraction);
    data_ = validation ? std::span<const uint32_t>(tokens_).subspan(split_)
                       : std::span<const uint32_t>(tokens_).first(split_);
    if (data_.empty()) throw std::invalid_argument("loader dataset must not be empty");
    if (static_cast<size_t>(seq) + 1 > data_.size())
      throw std::invalid_argument("sample length exceeds dataset size");
    const size_t n = static_cast<size_t>(batch) * seq;
    for (auto &slot : slots_)
      for (uint32_t *&p : slot.buf) {
        void *mem = nullptr;
        if (tl_host_alloc(&mem, n * sizeof(uint32_t)) != 0)
          throw std::runtime_error("pinned allocation failed");
        p = static_cast<uint32_t *>(mem);
      }
    fill(slots_[0]);
    slots_[0].ready = true;
    slots_[1].free = true;
    worker_ = std::thread([this] { run(); });
  }

  ~TokenPipeline() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    if (worker_.joinable()) worker_.join();
    for (auto &slot : slots_)
      for (uint32_t *p : slot.buf)
        if (p) tl_host_free(p);
  }

  TokenPipeline(const TokenPipeline &) = delete;
  TokenPipeline &operator=(const TokenPipeline &) = delete;

  // The next batch, in pinned memory, valid until the next call (which
  // hands its slot back to the worker for the batch after).
  void next(const uint32_t **inputs, const uint32_t **targets) {
    std::unique_lock<std::mutex> lk(mu_);
    Slot &s = slots_[cursor_];
    cv_.wait(lk, [&] { return s.ready; });
    *inputs = s.buf[0];
    *targets = s.buf[1];
    s.ready = false;
    if (handed_out_) slots_[cursor_ ^ 1].free = true;  // the previous batch is done with
    handed_out_ = true;
    cursor_ ^= 1;
    lk.unlock();
    cv_.notify_all();
  }

  size_t tokens() const { return tokens_.size(); }
  size_t split_index() const { return split_; }

private:
  struct Slot {
    uint32_t *buf[2] = {nullptr, nullptr};  // inputs, targets
    bool ready = false, free = false;
  };

  void load(const std::string &path) {
    std::ifstream in(path, std::ios::binary);
    if (!in) throw std::runtime_error("failed to read token dataset");
    const std::vector<char> bytes{std::istreambuf_iterator<char>(in),
                                  std::istreambuf_iterator<char>()};
    if (bytes.size() % sizeof(uint32_t) != 0) throw std::runtime_error("invalid token dataset size");
    tokens_.resize(bytes.size() / sizeof(uint32_t));
    if (!bytes.empty()) std::memcpy(tokens_.data(), bytes.data(), bytes.size());
  }

  void split(double fraction) {
    if (fraction <= 0.0 || fraction >= 1.0)
      throw std::invalid_argument("training fraction must be between zero and one");
    if (tokens_.size() < 2) throw std::invalid_argument("dataset must contain at least two tokens");
    const size_t target = static_cast<size_t>(static_cast<double>(tokens_.size()) * fraction);
    const auto boundary = std::find(tokens_.begin() + static_cast<std::ptrdiff_t>(target),
                                    tokens_.end(), kEndOfText);
    split_ = boundary == tokens_.end()
                 ? target
                 : static_cast<size_t>(std::distance(tokens_.begin(), boundary)) + 1;
    if (split_ == 0 || split_ >= tokens_.size())
      throw std::invalid_argument("dataset split produced an empty partition");
  }

  void fill(Slot &s) {
    std::uniform_int_distribution<size_t> start(0, data_.size() - (seq_ + 1));
    for (uint32_t b = 0; b < batch_; ++b) {
      const size_t s0 = start(gen_);
      std::memcpy(s.buf[0] + static_cast<size_t>(b) * seq_, data_.data() + s0,
                  seq_ * sizeof(uint32_t));
      std::memcpy(s.buf[1] + static_cast<size_t>(b) * seq_, data_.data() + s0 + 1,
                  seq_ * sizeof(uint32_t));
    }
  }

  void run() {
    uint32_t target = 1;  // slot the worker fills next
    for (;;) {
      std::unique_lock<std::mutex> lk(mu_);
      cv_.wait(lk, [&] { return stop_ || slots_[target].free; });
      if (stop_) return;
      slots_[target].free = false;
      lk.unlock();
      fill(slots_[target]);
      lk.lock();
      slots_[target].ready = true;
      lk.unlock();
      cv_.notify_all();
      target ^= 1;
    }
  }

  std::vector<uint32_t> tokens_;
  size_t split_ = 0;
  std::span<const uint32_t> data_;
  std::mt19937 gen_;
  uint32_t batch_, seq_;
  Slot slots_[2];
  uint32_t cursor_ = 0;
  std::mutex mu_;
  std::condition_variable cv_;
  std::thread worker_;
  bool stop_ = false, handed_out_ = false;
};

}  // namespace templit_b200

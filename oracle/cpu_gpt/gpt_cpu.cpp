// TEST INFRASTRUCTURE: the GPT training step of include/templit_gpt.h on the
// host oracle runtime (host_runtime.h): the reference's nn::GPT and
// passes::Compiled executor with every runtime op restated on the CPU.
// Exposed as tlo_* (oracle) so it can never be mistaken for the product.
#include "host_runtime.h"

#include "gpt_driver.h"
#include "gpt_infer.h"
#include "model_utils/Dataset.h"
#include "model_utils/archive.h"
#include "model_utils/loader.h"

#include <dlfcn.h>

#include <fstream>

#include <chrono>
#include <cstring>
#include <memory>
#include <string>

namespace {

using Mat = cpu_ref::Mat;
using GPT4 = nn::GPT<Mat, 2048, 192, 384, 6>;
thread_local std::string g_error;

struct Handle {
  cpu_ref::Runtime runtime;
  std::unique_ptr<templit_b200::DriverBase> driver;
};

struct InferHandle {
  cpu_ref::Runtime runtime;
  std::unique_ptr<templit_b200::InferBase> driver;
};

template <typename F> int guarded(F &&f) {
  try {
    f();
    return 0;
  } catch (const std::exception &e) {
    g_error = e.what();
  }
  return 1;
}

}  // namespace

static_assert(passes::Runnable<Mat, cpu_ref::Runtime>);

extern "C" int tlo_create(const tlg_config *c, void **handle);

namespace {

// Family 12 lives in libgpt_cpu_deep.so beside this library (see
// gpt_cpu_deep.cpp), opened on the first request.
templit_b200::DriverBase *deep_driver(const tlg_config *c, cpu_ref::Runtime *rt) {
  using Fn = templit_b200::DriverBase *(*)(const tlg_config *, cpu_ref::Runtime *, std::string *);
  static Fn fn = [] {
    Dl_info info{};
    if (!dladdr(reinterpret_cast<void *>(&tlo_create), &info) || !info.dli_fname) return Fn{};
    std::string dir(info.dli_fname);
    dir = dir.substr(0, dir.find_last_of('/') + 1);
    void *lib = dlopen((dir + "libgpt_cpu_deep.so").c_str(), RTLD_NOW | RTLD_GLOBAL);
    return lib ? reinterpret_cast<Fn>(dlsym(lib, "tlo_deep_driver_new")) : Fn{};
  }();
  if (!fn) throw std::runtime_error("family 12 needs oracle/_build/libgpt_cpu_deep.so");
  std::string error;
  templit_b200::DriverBase *d = fn(c, rt, &error);
  if (!d) throw std::runtime_error(error);
  return d;
}

}  // namespace

extern "C" {

const char *tlo_last_error(void) { return g_error.c_str(); }

int tlo_create(const tlg_config *c, void **handle) {
  return guarded([&] {
    if (c->family != 4 && c->family != 12)
      throw std::invalid_argument("oracle GPT supports families 4 and 12");
    auto h = std::make_unique<Handle>();
    if (c->family == 12)
      h->driver.reset(deep_driver(c, &h->runtime));
    else
      h->driver =
          std::make_unique<templit_b200::GptDriver<Mat, cpu_ref::Runtime, GPT4>>(*c, h->runtime);
    *handle = h.release();
  });
}

int tlo_destroy(void *h) {
  return guarded([&] { delete static_cast<Handle *>(h); });
}

int tlo_set_batch(void *h, const uint32_t *x, const uint32_t *y) {
  return guarded([&] { static_cast<Handle *>(h)->driver->set_batch(x, y); });
}

int tlo_train_step(void *h, float *mean_loss) {
  return guarded([&] {
    const float l = static_cast<Handle *>(h)->driver->train_step();
    if (mean_loss) *mean_loss = l;
  });
}

int tlo_forward(void *h, float *losses) {
  return guarded([&] { static_cast<Handle *>(h)->driver->forward(losses); });
}

int tlo_param_count(void *h, uint64_t *count, uint32_t *tensors) {
  return guarded([&] {
    std::vector<float> all;
    uint32_t t = 0;
    static_cast<Handle *>(h)->driver->params(all, t);
    *count = all.size();
    if (tensors) *tensors = t;
  });
}

int tlo_get_params(void *h, float *out, uint64_t count) {
  return guarded([&] {
    std::vector<float> all;
    uint32_t t = 0;
    static_cast<Handle *>(h)->driver->params(all, t);
    if (all.size() != count) throw std::invalid_argument("parameter count mismatch");
    std::memcpy(out, all.data(), count * sizeof(float));
  });
}

int tlo_set_allreduce(void *h, cpu_ref::Runtime::AllReduceFn fn, void *ctx) {
  return guarded([&] {
    auto *hd = static_cast<Handle *>(h);
    hd->runtime.allreduce = fn;
    hd->runtime.allreduce_ctx = ctx;
  });
}

int tlo_set_params(void *h, const float *in, uint64_t count) {
  return guarded([&] { static_cast<Handle *>(h)->driver->set_params(in, count); });
}

// Checkpoints through the reference's own Archive (src/model_utils/
// archive.cpp, compiled into this library): the format the CUDA library's
// tlg_save / tlg_load must match.
int tlo_save(void *h, const char *path, int optimiser) {
  return guarded([&] {
    auto *d = dynamic_cast<templit_b200::GptDriver<Mat, cpu_ref::Runtime, GPT4> *>(
        static_cast<Handle *>(h)->driver.get());
    if (!d) throw std::invalid_argument("not a family-4 model");
    Archive archive;
    d->save_archive(archive, optimiser != 0);
    std::ofstream out(path, std::ios::binary);
    archive.commit(out);
    if (!out) throw std::runtime_error("checkpoint write failed");
  });
}

int tlo_load(void *h, const char *path, int optimiser) {
  return guarded([&] {
    auto *d = dynamic_cast<templit_b200::GptDriver<Mat, cpu_ref::Runtime, GPT4> *>(
        static_cast<Handle *>(h)->driver.get());
    if (!d) throw std::invalid_argument("not a family-4 model");
    std::ifstream in(path, std::ios::binary);
    if (!in) throw std::runtime_error(std::string("cannot open ") + path);
    Archive archive;
    archive.restore(in);
    d->load_archive(archive, optimiser != 0);
  });
}

// The reference's own Dataset::load_tokens + Loader::get_batch (compiled
// into this library): n batches of [batch, seq] inputs and targets.
int tlo_loader_batches(const char *path, double training_fraction, int validation,
                       uint32_t batch, uint32_t seq, uint32_t seed, uint32_t n,
                       uint32_t *inputs, uint32_t *targets) {
  return guarded([&] {
    std::ifstream in(path, std::ios::binary);
    Dataset dataset = Dataset::load_tokens(in, training_fraction);
    Loader loader(validation ? dataset.validation_split() : dataset.training_split(), seed);
    const size_t per = static_cast<size_t>(batch) * seq;
    for (uint32_t i = 0; i < n; ++i) {
      const auto &b = loader.get_batch(batch, seq);
      std::memcpy(inputs + i * per, b.inputs.data(), per * sizeof(uint32_t));
      std::memcpy(targets + i * per, b.targets.data(), per * sizeof(uint32_t));
    }
  });
}

// ---------------------------------------------------------------- inference
int tlo_infer_create(const tlg_config *c, void **handle) {
  return guarded([&] {
    if (c->family != 4) throw std::invalid_argument("oracle GPT supports family 4");
    auto h = std::make_unique<InferHandle>();
    h->driver =
        std::make_unique<templit_b200::InferDriver<Mat, cpu_ref::Runtime, GPT4>>(*c, h->runtime);
    *handle = h.release();
  });
}

int tlo_infer_destroy(void *h) {
  return guarded([&] { delete static_cast<InferHandle *>(h); });
}

int tlo_infer_set_params(void *h, const float *in, uint64_t count) {
  return guarded([&] { static_cast<InferHandle *>(h)->driver->set_params(in, count); });
}

int tlo_infer_logits(void *h, const uint32_t *tokens, float *logits) {
  return guarded([&] { static_cast<InferHandle *>(h)->driver->logits(tokens, logits); });
}

int tlo_infer_generate(void *h, const uint32_t *prompt, uint32_t n_prompt, uint32_t eos,
                       uint32_t seed, uint32_t top_k, float temperature, uint32_t min_length,
                       uint32_t *out, uint32_t max_out, uint32_t *n_out) {
  return guarded([&] {
    const uint32_t n = static_cast<InferHandle *>(h)->driver->generate(
        prompt, n_prompt, eos, seed, top_k, temperature, min_length, out, max_out);
    if (n_out) *n_out = n;
  });
}

}  // extern "C"

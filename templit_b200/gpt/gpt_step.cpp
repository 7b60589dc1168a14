// The GPT training step on cuda::Runtime behind the C ABI of
// include/templit_gpt.h.  Family 4 is the reference's own nn::GPT
// (include/nn/GPT.h: vocab 2048, max sequence 192, d_model 384, 6 heads,
// 4 blocks - the model of src/train.cpp:23-27,98-99); family 12 the
// 12-block d_model 768 variant (deep_gpt.h, in libtemplit_gpt_deep.so).
#include "templit_gpt.h"

#include "gpt_driver.h"
#include "gpt_infer.h"
#include "input_pipeline.h"
#include "my_cuda/runtime.h"
#include "my_cuda/storage.h"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <fstream>
#include <memory>
#include <string>

namespace {

using Mat = RTensor<cuda::CUDA, cuda::kernel_type>;
using GPT4 = nn::GPT<Mat, 2048, 192, 384, 6>;

thread_local std::string g_error;

struct Handle {
  std::unique_ptr<cuda::Runtime> runtime;
  std::unique_ptr<templit_b200::DriverBase> driver;
  ncclComm_t comm = nullptr;
  int profile_steps = 0;
};

struct InferHandle {
  std::unique_ptr<cuda::Runtime> runtime;
  std::unique_ptr<templit_b200::InferBase> driver;
};

template <typename F> int guarded(F &&f) {
  try {
    f();
    return 0;
  } catch (const std::exception &e) {
    g_error = e.what();
  } catch (...) {
    g_error = "unknown exception";
  }
  return 1;
}

// The 12-block model lives in libtemplit_gpt_deep.so beside this library
// (its compile takes over an hour, so it is built on its own); opened on
// the first family-12 request.
std::unique_ptr<templit_b200::DriverBase> deep_driver(const tlg_config &c, cuda::Runtime &rt) {
  using Fn = templit_b200::DriverBase *(*)(const tlg_config *, cuda::Runtime *, std::string *);
  static Fn fn = [] {
    Dl_info info{};
    if (!dladdr(reinterpret_cast<void *>(&tlg_create), &info) || !info.dli_fname) return Fn{};
    std::string dir(info.dli_fname);
    dir = dir.substr(0, dir.find_last_of('/') + 1);
    void *lib = dlopen((dir + "libtemplit_gpt_deep.so").c_str(), RTLD_NOW | RTLD_GLOBAL);
    return lib ? reinterpret_cast<Fn>(dlsym(lib, "tlg_deep_driver_new")) : Fn{};
  }();
  if (!fn)
    throw std::runtime_error("family 12 needs libtemplit_gpt_deep.so (make -C templit_b200 "
                             "gpt-deep)");
  std::string error;
  templit_b200::DriverBase *d = fn(&c, &rt, &error);
  if (!d) throw std::runtime_error(error);
  return std::unique_ptr<templit_b200::DriverBase>(d);
}

std::unique_ptr<templit_b200::DriverBase> make_driver(const tlg_config &c, cuda::Runtime &rt) {
  if (c.family == 4) {
    if (c.seq == 0 || c.seq > 192) throw std::invalid_argument("family 4 takes seq in [1, 192]");
    return std::make_unique<templit_b200::GptDriver<Mat, cuda::Runtime, GPT4>>(c, rt);
  }
  if (c.family == 12) return deep_driver(c, rt);
  throw std::invalid_argument("unsupported GPT family " + std::to_string(c.family));
}

}  // namespace

extern "C" {

const char *tlg_last_error(void) { return g_error.c_str(); }

int tlg_create(const tlg_config *config, void **handle) {
  return guarded([&] {
    if (!config || !handle) throw std::invalid_argument("null argument");
    *handle = nullptr;
    cuda::init();
    auto h = std::make_unique<Handle>();
    h->runtime = std::make_unique<cuda::Runtime>();
    h->runtime->set_fusion(config->fusion != 0);
    h->runtime->set_graphs(config->graphs != 0);
    h->runtime->set_gemm_precision(config->gemm_precision);
    h->runtime->set_deferred_wait(config->deferred_wait != 0);
    if (config->flash_attention < -1 || config->flash_attention > 1)
      throw std::invalid_argument("flash_attention is -1, 0 or 1");
    if (config->flash_attention != 0) h->runtime->set_flash_attention(config->flash_attention + 1);
    h->driver = make_driver(*config, *h->runtime);
    *handle = h.release();
  });
}

int tlg_destroy(void *handle) {
  return guarded([&] {
    Handle *h = static_cast<Handle *>(handle);
    if (!h) return;
    h->driver.reset();
    h->runtime.reset();
    if (h->comm) ncclCommDestroy(h->comm);
    delete h;
  });
}

int tlg_set_batch(void *handle, const uint32_t *tokens, const uint32_t *targets) {
  return guarded([&] { static_cast<Handle *>(handle)->driver->set_batch(tokens, targets); });
}

int tlg_train_step(void *handle, float *mean_loss) {
  return guarded([&] {
    Handle *h = static_cast<Handle *>(handle);
    const float l = h->driver->train_step();
    if (mean_loss) *mean_loss = l;
    if (h->profile_steps > 0 && --h->profile_steps == 0) h->runtime->end_profile();
  });
}

int tlg_forward(void *handle, float *losses) {
  return guarded([&] { static_cast<Handle *>(handle)->driver->forward(losses); });
}

int tlg_param_count(void *handle, uint64_t *count, uint32_t *tensors) {
  return guarded([&] {
    std::vector<float> all;
    uint32_t t = 0;
    static_cast<Handle *>(handle)->driver->params(all, t);
    if (count) *count = all.size();
    if (tensors) *tensors = t;
  });
}

int tlg_get_params(void *handle, float *out, uint64_t count) {
  return guarded([&] {
    std::vector<float> all;
    uint32_t t = 0;
    static_cast<Handle *>(handle)->driver->params(all, t);
    if (count != all.size()) throw std::invalid_argument("parameter count mismatch");
    std::memcpy(out, all.data(), all.size() * sizeof(float));
  });
}

int tlg_set_params(void *handle, const float *in, uint64_t count) {
  return guarded([&] { static_cast<Handle *>(handle)->driver->set_params(in, count); });
}

void *tlg_stream(void *) { return cuda::stream(); }

int tlg_stats(void *handle, uint64_t out[TLG_STATS]) {
  return guarded([&] {
    const cuda::RuntimeStats &s = static_cast<Handle *>(handle)->runtime->stats();
    out[0] = s.windows;
    out[1] = s.ops_recorded;
    out[2] = s.ops_launched;
    out[3] = s.kernel_launches;
    out[4] = s.graph_replays;
    out[5] = s.graph_captures;
    out[6] = s.fused_ops;
    out[7] = cuda::memory_stats().peak_in_use;
    out[8] = s.host_record_ns;
    out[9] = s.host_submit_ns;
    out[10] = s.optimiser_cache_hits;
  });
}

int tlg_nccl_unique_id(uint8_t id[128]) {
  return guarded([&] {
    static_assert(sizeof(ncclUniqueId) == 128);
    ncclUniqueId u;
    const ncclResult_t r = ncclGetUniqueId(&u);
    if (r != ncclSuccess) throw std::runtime_error(ncclGetErrorString(r));
    std::memcpy(id, &u, 128);
  });
}

int tlg_set_communicator(void *handle, const uint8_t id[128], int nranks, int rank) {
  return guarded([&] {
    Handle *h = static_cast<Handle *>(handle);
    ncclUniqueId u;
    std::memcpy(&u, id, 128);
    cuda::init();
    const ncclResult_t r = ncclCommInitRank(&h->comm, nranks, u, rank);
    if (r != ncclSuccess) throw std::runtime_error(ncclGetErrorString(r));
    h->runtime->set_communicator(h->comm);
  });
}

int tlg_profile(void *handle, const char *path, int steps) {
  return guarded([&] {
    Handle *h = static_cast<Handle *>(handle);
    h->runtime->start_profile(path);
    h->profile_steps = steps;
  });
}

int tlg_save(void *handle, const char *path, int optimiser) {
  return guarded([&] {
    if (!path) throw std::invalid_argument("null path");
    static_cast<Handle *>(handle)->driver->save(path, optimiser != 0);
  });
}

int tlg_load(void *handle, const char *path, int optimiser) {
  return guarded([&] {
    if (!path) throw std::invalid_argument("null path");
    static_cast<Handle *>(handle)->driver->load(path, optimiser != 0);
  });
}

// ----------------------------------------------------------- input pipeline
int tlg_loader_create(const char *path, double training_fraction, int validation,
                      uint32_t batch, uint32_t seq, uint32_t seed, void **handle) {
  return guarded([&] {
    if (!path || !handle) throw std::invalid_argument("null argument");
    *handle = nullptr;
    cuda::init();  // pinned memory needs the device
    *handle = new templit_b200::TokenPipeline(path, training_fraction, validation != 0, batch,
                                              seq, seed);
  });
}

int tlg_loader_next(void *handle, const uint32_t **inputs, const uint32_t **targets) {
  return guarded([&] {
    if (!handle || !inputs || !targets) throw std::invalid_argument("null argument");
    static_cast<templit_b200::TokenPipeline *>(handle)->next(inputs, targets);
  });
}

int tlg_loader_destroy(void *handle) {
  return guarded([&] { delete static_cast<templit_b200::TokenPipeline *>(handle); });
}

// ---------------------------------------------------------------- inference
int tlg_infer_create(const tlg_config *config, void **handle) {
  return guarded([&] {
    if (!config || !handle) throw std::invalid_argument("null argument");
    *handle = nullptr;
    if (config->family != 4) throw std::invalid_argument("inference supports family 4");
    if (config->seq == 0 || config->seq > 192)
      throw std::invalid_argument("family 4 takes seq in [1, 192]");
    cuda::init();
    auto h = std::make_unique<InferHandle>();
    h->runtime = std::make_unique<cuda::Runtime>();
    h->runtime->set_fusion(config->fusion != 0);
    h->runtime->set_graphs(config->graphs != 0);
    h->runtime->set_gemm_precision(config->gemm_precision);
    h->driver =
        std::make_unique<templit_b200::InferDriver<Mat, cuda::Runtime, GPT4>>(*config, *h->runtime);
    *handle = h.release();
  });
}

int tlg_infer_destroy(void *handle) {
  return guarded([&] {
    InferHandle *h = static_cast<InferHandle *>(handle);
    if (!h) return;
    h->driver.reset();
    h->runtime.reset();
    delete h;
  });
}

int tlg_infer_param_count(void *handle, uint64_t *count) {
  return guarded([&] {
    std::vector<float> all;
    uint32_t t = 0;
    static_cast<InferHandle *>(handle)->driver->params(all, t);
    if (count) *count = all.size();
  });
}

int tlg_infer_get_params(void *handle, float *out, uint64_t count) {
  return guarded([&] {
    std::vector<float> all;
    uint32_t t = 0;
    static_cast<InferHandle *>(handle)->driver->params(all, t);
    if (count != all.size()) throw std::invalid_argument("parameter count mismatch");
    std::memcpy(out, all.data(), all.size() * sizeof(float));
  });
}

int tlg_infer_set_params(void *handle, const float *in, uint64_t count) {
  return guarded([&] { static_cast<InferHandle *>(handle)->driver->set_params(in, count); });
}

int tlg_infer_logits(void *handle, const uint32_t *tokens, float *logits) {
  return guarded([&] { static_cast<InferHandle *>(handle)->driver->logits(tokens, logits); });
}

int tlg_infer_generate(void *handle, const uint32_t *prompt, uint32_t n_prompt, uint32_t eos,
                       uint32_t seed, uint32_t top_k, float temperature, uint32_t min_length,
                       uint32_t *out, uint32_t max_out, uint32_t *n_out) {
  return guarded([&] {
    const uint32_t n = static_cast<InferHandle *>(handle)->driver->generate(
        prompt, n_prompt, eos, seed, top_k, temperature, min_length, out, max_out);
    if (n_out) *n_out = n;
  });
}

}  // extern "C"

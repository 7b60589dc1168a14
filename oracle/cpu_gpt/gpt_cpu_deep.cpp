// TEST INFRASTRUCTURE: the configuration-5 GPT (12 pre-RMSNorm decoder
// blocks, d_model 768, 12 heads, FFN 3072, vocab 2048, T up to 1024) on the
// host oracle runtime (host_runtime.h): the reference's decoder blocks,
// embeddings and projection (include/nn/) in DeepGPT, driven by the
// reference's passes::Compiled.  Built on its own into libgpt_cpu_deep.so
// (its compile takes over an hour); libgpt_cpu.so opens it for family 12.
#include "host_runtime.h"

#include "deep_gpt.h"
#include "gpt_driver.h"

#include <memory>
#include <string>

extern "C" templit_b200::DriverBase *tlo_deep_driver_new(const tlg_config *c,
                                                         cpu_ref::Runtime *rt,
                                                         std::string *error) {
  try {
    using Deep = templit_b200::DeepGPT<cpu_ref::Mat, 2048, 1024, 768, 12, 12>;
    if (c->seq == 0 || c->seq > 1024) throw std::invalid_argument("family 12 takes seq in [1, 1024]");
    return new templit_b200::GptDriver<cpu_ref::Mat, cpu_ref::Runtime, Deep>(*c, *rt);
  } catch (const std::exception &e) {
    *error = e.what();
  } catch (...) {
    *error = "unknown exception";
  }
  return nullptr;
}

// Entry point of libtemplit_gpt_deep.so, the library of the configuration-5
// GPT (gpt_deep.cpp), which libtemplit_gpt.so opens on the first family-12
// request: the 12-block model's compile takes over an hour, so it is built
// on its own (`make -C templit_b200 gpt-deep`) and the four-block library
// does not link it.  Both libraries come from the same compiler and share
// the C++ types passed here.
#include "gpt_driver.h"
#include "my_cuda/runtime.h"

#include <memory>
#include <string>

namespace templit_b200 {
// gpt_deep.cpp: the 12-block model (DeepGPT<..., 2048, 1024, 768, 12, 12>)
std::unique_ptr<DriverBase> make_deep_driver(const tlg_config &c, cuda::Runtime &rt);
}  // namespace templit_b200

// A new family-12 driver on `rt`, or nullptr with *error set.
extern "C" templit_b200::DriverBase *tlg_deep_driver_new(const tlg_config *c, cuda::Runtime *rt,
                                                         std::string *error) {
  try {
    return templit_b200::make_deep_driver(*c, *rt).release();
  } catch (const std::exception &e) {
    *error = e.what();
  } catch (...) {
    *error = "unknown exception";
  }
  return nullptr;
}

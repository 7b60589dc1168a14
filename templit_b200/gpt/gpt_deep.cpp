// The configuration-5 GPT (12 pre-RMSNorm decoder blocks, d_model 768, 12
// heads, FFN 3072, vocab 2048, sequences up to 1024) on cuda::Runtime: the
// reference's decoder blocks, embeddings and projection (include/nn/) in
// DeepGPT, compiled by the reference's passes::Compiled.  Its own
// translation unit: the expression types of twelve blocks take the compiler
// a while, and the four-block library should not wait for them.
#include "deep_gpt.h"
#include "gpt_driver.h"
#include "my_cuda/runtime.h"
#include "my_cuda/storage.h"

#include <stdexcept>

namespace templit_b200 {

std::unique_ptr<DriverBase> make_deep_driver(const tlg_config &c, cuda::Runtime &rt) {
  using Mat = RTensor<cuda::CUDA, cuda::kernel_type>;
  using Deep = DeepGPT<Mat, 2048, 1024, 768, 12, 12>;
  if (c.seq == 0 || c.seq > 1024) throw std::invalid_argument("family 12 takes seq in [1, 1024]");
  return std::make_unique<GptDriver<Mat, cuda::Runtime, Deep>>(c, rt);
}

}  // namespace templit_b200

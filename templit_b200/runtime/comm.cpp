// Data-parallel gradient exchange over NCCL (NVLink 5 / NVSwitch on B200).
// The reference has no multi-device path; this is the one exchange step of
// batch data parallelism: an in-place sum of every gradient across ranks.
// By default the per-tensor sums run as one NCCL group
// (all_reduce_gradients); with TL_FLAT_ALLREDUCE=1 the runtime packs the
// gradients into one flat buffer (tl_multi_grad_flat) and sums it with a
// single all-reduce (all_reduce_flat): one NCCL call instead of one per
// tensor (52 for the d384 GPT, most of them bias and norm vectors).
#include "optimize.h"

#include <nccl.h>

#include <string>

namespace cuda::internal {

void all_reduce_gradients(const Op &op, void *comm, void *stream) {
  if (!comm) throw std::logic_error("gradient all-reduce without a communicator");
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ncclResult_t r = ncclGroupStart();
  if (r != ncclSuccess)
    throw std::runtime_error(std::string("ncclGroupStart: ") + ncclGetErrorString(r));
  for (const MultiSlot &slot : op.multi) {
    r = ncclAllReduce(slot.grad.p, slot.grad.p, slot.grad.numel(), ncclFloat32, ncclSum, c, s);
    if (r != ncclSuccess) {
      ncclGroupEnd();
      throw std::runtime_error(std::string("ncclAllReduce: ") + ncclGetErrorString(r));
    }
  }
  r = ncclGroupEnd();
  if (r != ncclSuccess)
    throw std::runtime_error(std::string("ncclGroupEnd: ") + ncclGetErrorString(r));
}

void all_reduce_flat(float *flat, size_t count, void *comm, void *stream) {
  if (!comm) throw std::logic_error("gradient all-reduce without a communicator");
  const ncclResult_t r = ncclAllReduce(flat, flat, count, ncclFloat32, ncclSum,
                                       static_cast<ncclComm_t>(comm),
                                       static_cast<cudaStream_t>(stream));
  if (r != ncclSuccess)
    throw std::runtime_error(std::string("ncclAllReduce: ") + ncclGetErrorString(r));
}

}  // namespace cuda::internal

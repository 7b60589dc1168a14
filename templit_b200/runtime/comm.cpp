// Data-parallel gradient exchange over NCCL (NVLink 5 / NVSwitch on B200).
// The reference has no multi-device path; this is the one exchange step of
// batch data parallelism: an in-place sum of every gradient across ranks,
// issued as one NCCL group so it runs as a single fused collective launch.
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

}  // namespace cuda::internal

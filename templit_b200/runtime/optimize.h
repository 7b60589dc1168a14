// Program optimiser and data-parallel hooks of the recording runtime.
#pragma once

#include "program.h"

#include <cstdint>
#include <vector>

namespace cuda::internal {

// Rewrites a recorded program in place (ops folded into fused kernels are
// marked dead) and returns the number of recorded ops that were folded.
// Every rewrite preserves the values of all tensors that outlive the
// program; intermediates it skips are ones released inside the program.
// With a communicator, gradients read by the optimiser are first summed
// across ranks (see add_gradient_allreduce).
uint64_t optimize(std::vector<Op> &prog, void *comm);

// Inserts one AllReduce op ahead of the first optimiser op of a program
// that updates parameters, covering every gradient that op sequence reads.
void add_gradient_allreduce(std::vector<Op> &prog);

// Executes an AllReduce op: in-place ncclAllReduce(sum) of each gradient
// in op.multi, grouped into one NCCL launch.
void all_reduce_gradients(const Op &op, void *comm, void *stream);

}  // namespace cuda::internal

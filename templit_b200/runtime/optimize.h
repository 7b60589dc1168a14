// Program optimiser and data-parallel hooks of the recording runtime.
#pragma once

#include "program.h"

#include <cstdint>
#include <vector>

namespace cuda::internal {

// Allocation ids an op reads / writes.
struct Access {
  uint64_t r[16];
  int nr = 0;
  uint64_t w[6];
  int nw = 0;
  void read(const TRef &t) {
    if (t.p) r[nr++] = t.id;
  }
  void write(const TRef &t) {
    if (t.p) w[nw++] = t.id;
  }
};
Access access(const Op &op);
// True when `op` replaces the whole allocation it writes (Storage writes,
// fills and clones may cover only part of it; SqNorm accumulates).
bool full_write(const Op &op);

// What the runtime knows about values that outlive a program.  A buffer is
// window-local when, over the training windows observed so far, every
// window that touched it wrote it before reading it and the host never read
// it: its value at the end of a window is never used, like the executor's
// private temporaries (include/passes/mem_lower.h gives every expression
// node its own temporary, consumed by its parent inside the same program).
struct Liveness {
  virtual ~Liveness() = default;
  virtual bool window_local(uint64_t id) const = 0;
};

// Rewrites a recorded program in place (ops folded into fused kernels are
// marked dead) and returns the number of recorded ops that were folded.
// Every rewrite preserves the values of all tensors that outlive the
// program; intermediates it skips are ones released inside the program or
// window-local according to `live` (may be null: nothing is window-local).
// With a communicator, gradients read by the optimiser are first summed
// across ranks (see add_gradient_allreduce).
uint64_t optimize(std::vector<Op> &prog, void *comm, const Liveness *live = nullptr);

// Inserts one AllReduce op ahead of the first optimiser op of a program
// that updates parameters, covering every gradient that op sequence reads.
void add_gradient_allreduce(std::vector<Op> &prog);

// Executes an AllReduce op: in-place ncclAllReduce(sum) of each gradient
// in op.multi, grouped into one NCCL launch.
void all_reduce_gradients(const Op &op, void *comm, void *stream);

}  // namespace cuda::internal

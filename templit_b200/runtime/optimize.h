// Program optimiser and data-parallel hooks of the recording runtime.
#pragma once

#include "program.h"

#include <cstdint>
#include <vector>

namespace cuda::internal {

// Allocation ids an op reads / writes.
struct Access {
  uint64_t r[20];
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

// A softmax output P = softmax(Q K^T / divisor + mask) of the attention
// composite that a flash forward left unwritten: P is defined by its
// recipe (the inputs below and the row log-sum-exp in desc.lse) until an op
// other than the flash backward reads it, which first rebuilds it
// (FlashProbs).  Writing or releasing a recipe input also rebuilds P first.
struct FlashRecord {
  uint64_t p_id = 0;
  TRef p, q, k, v, o, divisor, mask;
  tl_flash_desc desc{};  // q, k, v, o views; divisor, mask, mask_flag, lse; B, H, T, D
  bool o_valid = true;   // O still holds the forward's output
};

// The runtime's side of flash attention: the records earlier windows left
// and the buffers the kernels need beyond their operands.
struct FlashState {
  virtual ~FlashState() = default;
  virtual bool enabled() const = 0;
  // true: every attention composite the flash kernels take; false: only
  // those the short-sequence fused kernels cannot (T above 192)
  virtual bool always() const = 0;
  // records of P tensors left virtual by programs already launched
  virtual const std::vector<FlashRecord> &records() const = 0;
  // runtime-owned [B, H, T] log-sum-exp buffer of P (stable per P)
  virtual float *lse_buffer(uint64_t p_id, size_t bytes) = 0;
  // a device word for the causal-mask check of mask allocation `mask_id`
  virtual uint32_t *mask_word(uint64_t mask_id) = 0;
};

// Applies a launched program's effect on the flash records in order:
// FlashFwd adds (or replaces) P's record, FlashProbs, a write of P or its
// release removes it, a write of O marks it stale.
void update_flash_records(const std::vector<Op> &prog, std::vector<FlashRecord> &records);

// Rewrites a recorded program in place (ops folded into fused kernels are
// marked dead) and returns the number of recorded ops that were folded.
// Every rewrite preserves the values of all tensors that outlive the
// program; intermediates it skips are ones released inside the program or
// window-local according to `live` (may be null: nothing is window-local).
// With a communicator, gradients read by the optimiser are first summed
// across ranks (see add_gradient_allreduce).
// With `flash` enabled, the attention composite runs on the flash kernels
// (any sequence length) and its P stays virtual.
uint64_t optimize(std::vector<Op> &prog, void *comm, const Liveness *live = nullptr,
                  FlashState *flash = nullptr);

// Marks the first attention forward (fused: u0 bit 0; flash: code bit 0)
// that reads each runtime-checked mask in a program, and the first after
// any write to the mask, as the one that runs the causal-mask check.
void assign_mask_checks(std::vector<Op> &prog);

// Inserts one AllReduce op ahead of the first optimiser op of a program
// that updates parameters, covering every gradient that op sequence reads.
void add_gradient_allreduce(std::vector<Op> &prog);

// Executes an AllReduce op: in-place ncclAllReduce(sum) of each gradient
// in op.multi, grouped into one NCCL launch.
// In-place sum across ranks of every gradient of an AllReduce op (one NCCL
// group of per-tensor all-reduces).
void all_reduce_gradients(const Op &op, void *comm, void *stream);
// In-place sum across ranks of `count` floats at `flat` (one NCCL call).
void all_reduce_flat(float *flat, size_t count, void *comm, void *stream);

}  // namespace cuda::internal

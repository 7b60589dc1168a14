// Internal interfaces shared by the backend's device layer (device.cpp) and
// the recording runtime (runtime.cpp).  Not installed.
#pragma once

#include "my_cuda/cuda.h"
#include "templit_cuda.h"

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

namespace cuda::internal {

// The open recording window of a Runtime.  Storage operations on blocks
// allocated inside the window are appended to its program; releases are
// noted so the optimiser knows which values die inside the program.
struct Recorder {
  virtual ~Recorder() = default;
  virtual uint64_t window() const = 0;
  virtual void record_write(const detail::Block &dst, size_t offset, const void *src,
                            size_t bytes) = 0;
  virtual void record_fill(const detail::Block &dst, uint32_t pattern, size_t count) = 0;
  virtual void record_copy(const detail::Block &dst, const detail::Block &src,
                           size_t bytes) = 0;
  virtual void record_release(const detail::Block &block) = 0;
};

Recorder *active_recorder();
void set_active_recorder(Recorder *r);

// Told about immediate (not recorded) host accesses to device blocks, before
// they happen: a runtime whose programs leave a tensor's value implicit (a
// flash attention P kept as its recipe) makes it real before the host reads
// it or a write replaces part of it, and forgets it when it is released.
struct HostAccessHook {
  virtual ~HostAccessHook() = default;
  virtual void before_host_access(uint64_t id, bool write, bool full) = 0;
  virtual void on_release(uint64_t id) = 0;
};
void add_host_access_hook(HostAccessHook *h);
void remove_host_access_hook(HostAccessHook *h);
uint64_t next_window_id();
// True when the block's value has been read outside a recorded program
// (Storage::read / compare on the host, or an immediate clone) since it
// was allocated.
bool host_observed(uint64_t id);

// Throws std::runtime_error with the library's message unless status == TL_OK.
inline void check(int status, const char *what) {
  if (status != TL_OK) {
    throw std::runtime_error(std::string(what) + ": " + tl_last_error());
  }
}

void ensure_init();

}  // namespace cuda::internal

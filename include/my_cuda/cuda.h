// Device tag and process-wide device state of the TempLit `cuda` backend.
// Counterpart of include/my_metal/metal.h (metal::Metal, init, shutdown,
// kernel_type, index_type) in JTPuffer/TempLit.
#pragma once

#include <cstddef>
#include <cstdint>

namespace cuda {

// Device tag used as RTensor<cuda::CUDA, T>.
struct CUDA {};

using kernel_type = float;
using index_type = uint32_t;

// Selects the GPU and creates the backend's stream.  device < 0 picks
// LOCAL_RANK from the environment (one process per GPU), else device 0.
// Storage constructed before init() initialises the backend implicitly.
void init(int device = -1);
// Waits for outstanding work and releases cached device memory.
void shutdown();
bool initialised();
// The cudaStream_t (as void*) every Storage copy and Runtime launch uses.
void *stream();
// Blocks until all work issued to stream() has finished.
void synchronize();

// Device-memory pool statistics (bytes).
struct MemoryStats {
  size_t reserved;  // obtained from the driver and cached
  size_t in_use;    // held by live Storage objects and runtime workspaces
  size_t peak_in_use;
};
MemoryStats memory_stats();

namespace detail {

// A device allocation from the caching pool.  `id` is unique for the life
// of the process (never reused), so recorded programs can tell two
// allocations that happen to share an address apart.
struct Block {
  void *ptr = nullptr;
  size_t bytes = 0;
  uint64_t id = 0;
  uint64_t window = 0;  // recording window open at allocation (0 = none)
};

Block allocate(size_t bytes);
void release(const Block &block) noexcept;

// Storage-level data movement.  While a Runtime has a recording window
// open, operations on storage allocated inside that window are appended to
// the window's program (they must run after the ops recorded before them);
// everything else happens immediately, ordered on stream().
void write(const Block &dst, size_t offset_bytes, const void *src, size_t bytes);
void read(const Block &src, size_t offset_bytes, void *dst, size_t bytes);
void fill32(const Block &dst, uint32_t pattern, size_t count);
void copy(const Block &dst, const Block &src, size_t bytes);
bool equal(const Block &a, const Block &b, size_t bytes);
// Invalidates host copies of device data (called before device work runs).
void device_changed();

}  // namespace detail
}  // namespace cuda

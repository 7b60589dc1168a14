// Process-wide device state of the `cuda` backend: device selection, the
// backend stream, the caching device-memory pool and the Storage data paths.
// Counterpart of src/my_metal/metal.cpp and the MTL::Buffer handling in
// include/my_metal/storage.h (JTPuffer/TempLit).
//
// Pool.  Device memory is obtained from the driver in size-rounded blocks
// and cached on release; a request takes the smallest cached block of at
// least its rounded size (within 2x), so the executor's per-step
// temporaries are served without driver calls and, for a repeated program,
// at the same addresses (which is what lets a captured CUDA graph replay).
// Reuse is stream-ordered: every launch goes to one stream, so memory freed
// by the host while a program is queued can only be rewritten by work
// queued after it.
#include "internal.h"

#include <cstdlib>
#include <algorithm>
#include <cstring>
#include <iterator>
#include <map>
#include <mutex>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace cuda {
namespace {

struct State {
  bool initialised = false;
  int device = 0;
  void *stream = nullptr;
  std::multimap<size_t, void *> free_blocks;
  std::unordered_map<void *, size_t> block_size;  // every block obtained
  size_t reserved = 0;
  size_t in_use = 0;
  size_t peak = 0;
  uint64_t next_id = 1;
  uint64_t window_counter = 0;
  internal::Recorder *recorder = nullptr;
  std::vector<internal::HostAccessHook *> hooks;
  // blocks whose value was read outside a recorded program (host reads,
  // immediate device copies), until released
  std::unordered_set<uint64_t> observed;
  // Host mirror of the last block read in pieces (element-wise RTensor::get
  // reads of logits): valid while no device write or launch has happened
  // since it was taken (`epoch` and the library's launch counter).
  uint64_t epoch = 0;
  struct Mirror {
    uint64_t id = 0, epoch = 0, launches = 0;
    std::vector<unsigned char> bytes;
  } mirror;
};

State &state() {
  static State s;
  return s;
}

size_t round_size(size_t bytes) {
  if (bytes == 0) bytes = 1;
  const size_t small = 512, large = size_t(2) << 20;
  return bytes < (size_t(1) << 20) ? (bytes + small - 1) / small * small
                                   : (bytes + large - 1) / large * large;
}

void release_cached() {
  State &s = state();
  if (s.free_blocks.empty()) return;
  tl_stream_sync(s.stream);
  for (auto &kv : s.free_blocks) {
    tl_free(kv.second);
    s.reserved -= kv.first;
    s.block_size.erase(kv.second);
  }
  s.free_blocks.clear();
}

}  // namespace

namespace internal {

void ensure_init() {
  if (!state().initialised) cuda::init(-1);
}

Recorder *active_recorder() { return state().recorder; }
void add_host_access_hook(HostAccessHook *h) { state().hooks.push_back(h); }
void remove_host_access_hook(HostAccessHook *h) {
  auto &v = state().hooks;
  v.erase(std::remove(v.begin(), v.end(), h), v.end());
}
void set_active_recorder(Recorder *r) { state().recorder = r; }
uint64_t next_window_id() { return ++state().window_counter; }
bool host_observed(uint64_t id) { return state().observed.count(id) != 0; }

}  // namespace internal

void init(int device) {
  State &s = state();
  if (s.initialised) return;
  if (device < 0) {
    const char *lr = std::getenv("LOCAL_RANK");
    device = lr ? std::atoi(lr) : 0;
  }
  internal::check(tl_device_init(device), "cuda::init");
  void *stream = nullptr;
  internal::check(tl_stream_create(&stream), "cuda::init stream");
  s.device = device;
  s.stream = stream;
  s.initialised = true;
}

void shutdown() {
  State &s = state();
  if (!s.initialised) return;
  tl_stream_sync(s.stream);
  release_cached();
  tl_stream_destroy(s.stream);
  s.stream = nullptr;
  s.initialised = false;
}

bool initialised() { return state().initialised; }

void *stream() {
  internal::ensure_init();
  return state().stream;
}

void synchronize() {
  internal::ensure_init();
  internal::check(tl_stream_sync(state().stream), "cuda::synchronize");
}

MemoryStats memory_stats() {
  const State &s = state();
  return MemoryStats{s.reserved, s.in_use, s.peak};
}

namespace detail {

Block allocate(size_t bytes) {
  internal::ensure_init();
  State &s = state();
  const size_t want = round_size(bytes);
  Block b;
  b.bytes = want;
  auto it = s.free_blocks.lower_bound(want);
  if (it != s.free_blocks.end() && it->first <= 2 * want) {
    // the most recently released block of the best size (last-in,
    // first-out): a window that allocates and releases the same sequence
    // every step then gets the same addresses every step
    it = std::prev(s.free_blocks.upper_bound(it->first));
    b.ptr = it->second;
    b.bytes = it->first;
    s.free_blocks.erase(it);
  } else {
    void *p = nullptr;
    if (tl_malloc(&p, want) != TL_OK) {
      release_cached();
      internal::check(tl_malloc(&p, want), "device allocation");
    }
    b.ptr = p;
    s.block_size[p] = want;
    s.reserved += want;
  }
  b.id = s.next_id++;
  internal::Recorder *r = s.recorder;
  b.window = r ? r->window() : 0;
  s.in_use += b.bytes;
  if (s.in_use > s.peak) s.peak = s.in_use;
  return b;
}

void release(const Block &block) noexcept {
  if (!block.ptr) return;
  State &s = state();
  for (internal::HostAccessHook *h : s.hooks) h->on_release(block.id);
  if (s.recorder) s.recorder->record_release(block);
  s.observed.erase(block.id);
  s.in_use -= block.bytes;
  s.free_blocks.emplace(block.bytes, block.ptr);
}

namespace {
bool recorded_here(const Block &b) {
  internal::Recorder *r = state().recorder;
  return r && b.window != 0 && b.window == r->window();
}
}  // namespace

void device_changed() { ++state().epoch; }

void host_access(const Block &b, bool write, bool full) {
  for (internal::HostAccessHook *h : state().hooks) h->before_host_access(b.id, write, full);
}

void write(const Block &dst, size_t offset_bytes, const void *src, size_t bytes) {
  if (bytes == 0) return;
  device_changed();
  if (recorded_here(dst)) {
    state().recorder->record_write(dst, offset_bytes, src, bytes);
    return;
  }
  host_access(dst, true, offset_bytes == 0 && bytes >= dst.bytes);
  internal::check(tl_memcpy_h2d(static_cast<char *>(dst.ptr) + offset_bytes, src, bytes,
                                state().stream),
                  "Storage::write");
}

void read(const Block &src, size_t offset_bytes, void *dst, size_t bytes) {
  if (bytes == 0) return;
  State &s = state();
  if (!s.hooks.empty()) host_access(src, false, false);
  s.observed.insert(src.id);
  State::Mirror &m = s.mirror;
  const bool fresh = m.id == src.id && m.epoch == s.epoch && m.launches == tl_kernel_launches();
  if (fresh && offset_bytes + bytes <= m.bytes.size()) {
    std::memcpy(dst, m.bytes.data() + offset_bytes, bytes);
    return;
  }
  // a piece of a block up to 16 MB: bring the whole block over once, so the
  // next element reads are host copies
  constexpr size_t kMirrorMax = size_t(16) << 20;
  if (bytes < src.bytes && src.bytes <= kMirrorMax) {
    m.bytes.resize(src.bytes);
    internal::check(tl_memcpy_d2h(m.bytes.data(), src.ptr, src.bytes, s.stream), "Storage::read");
    internal::check(tl_stream_sync(s.stream), "Storage::read sync");
    m.id = src.id;
    m.epoch = s.epoch;
    m.launches = tl_kernel_launches();
    std::memcpy(dst, m.bytes.data() + offset_bytes, bytes);
    return;
  }
  internal::check(tl_memcpy_d2h(dst, static_cast<const char *>(src.ptr) + offset_bytes, bytes,
                                s.stream),
                  "Storage::read");
  internal::check(tl_stream_sync(s.stream), "Storage::read sync");
}

void fill32(const Block &dst, uint32_t pattern, size_t count) {
  if (count == 0) return;
  device_changed();
  if (recorded_here(dst)) {
    state().recorder->record_fill(dst, pattern, count);
    return;
  }
  host_access(dst, true, count * 4 >= dst.bytes);
  internal::check(tl_fill_u32(dst.ptr, pattern, count, state().stream), "Storage::fill");
}

void copy(const Block &dst, const Block &src, size_t bytes) {
  if (bytes == 0) return;
  device_changed();
  if (recorded_here(dst) || recorded_here(src)) {
    state().recorder->record_copy(dst, src, bytes);
    return;
  }
  host_access(src, false, false);
  host_access(dst, true, bytes >= dst.bytes);
  state().observed.insert(src.id);
  internal::check(tl_memcpy_d2d(dst.ptr, src.ptr, bytes, state().stream), "Storage::clone");
}

bool equal(const Block &a, const Block &b, size_t bytes) {
  if (bytes == 0) return true;
  std::vector<unsigned char> ha(bytes), hb(bytes);
  read(a, 0, ha.data(), bytes);
  read(b, 0, hb.data(), bytes);
  return std::memcmp(ha.data(), hb.data(), bytes) == 0;
}

}  // namespace detail
}  // namespace cuda

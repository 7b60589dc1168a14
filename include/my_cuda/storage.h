// Storage<cuda::CUDA, T>: ref-counted device buffer behind RTensor.
// Counterpart of include/my_metal/storage.h in JTPuffer/TempLit, with the
// same interface (public ref_count, explicit size constructor, write/read
// bounds-checked with std::out_of_range, fill, clone, compare) so that it
// satisfies the Writable/Readable/Fillable/Comparable/CloneableStorage
// concepts of include/RTensor/storage.h.
//
// Memory comes from the backend's caching pool (cuda::detail::allocate).
// write/read/fill/clone/compare are synchronous with respect to the host,
// like the unified-memory Metal buffers they replace: a value written is
// visible to every later launch, a value read reflects every finished one.
#pragma once

#include "RTensor/storage.h"
#include "my_cuda/cuda.h"

#include <cstddef>
#include <span>
#include <stdexcept>

template <typename T> class Storage<cuda::CUDA, T> {
public:
  explicit Storage(size_t size)
      : ref_count(1), size_(size), block_(cuda::detail::allocate(size * sizeof(T))) {}
  Storage(const Storage &) = delete;
  Storage &operator=(const Storage &) = delete;
  Storage(Storage &&) = delete;
  Storage &operator=(Storage &&) = delete;
  ~Storage() { cuda::detail::release(block_); }

  int ref_count;

  // Device address of element 0.
  T *data() { return static_cast<T *>(block_.ptr); }
  const T *data() const { return static_cast<const T *>(block_.ptr); }
  size_t size() const { return size_; }
  const cuda::detail::Block &block() const { return block_; }

  void write(std::span<const T> values, size_t offset) {
    if (offset + values.size() > size_) {
      throw std::out_of_range("write out of bounds");
    }
    cuda::detail::write(block_, offset * sizeof(T), values.data(), values.size_bytes());
  }

  void read(std::span<T> out, size_t offset) const {
    if (offset + out.size() > size_) {
      throw std::out_of_range("read out of bounds");
    }
    cuda::detail::read(block_, offset * sizeof(T), out.data(), out.size_bytes());
  }

  void fill(T value) {
    static_assert(sizeof(T) == 4, "fill supports 32-bit element types");
    uint32_t pattern;
    __builtin_memcpy(&pattern, &value, 4);
    cuda::detail::fill32(block_, pattern, size_);
  }

  Storage *clone() const {
    Storage *other = new Storage(size_);
    cuda::detail::copy(other->block_, block_, size_ * sizeof(T));
    return other;
  }

  bool compare(const Storage &other) const {
    if (other.size_ != size_) {
      return false;
    }
    return cuda::detail::equal(block_, other.block_, size_ * sizeof(T));
  }

private:
  size_t size_ = 0;
  cuda::detail::Block block_;
};

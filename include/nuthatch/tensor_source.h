// Positioned reads from one file (reference: src/io/tensor_source.h:18-39).
// POSIX pread with a short-read loop; thread-safe (pread leaves the file
// position alone).
#ifndef NUTHATCH_B200_TENSOR_SOURCE_H_
#define NUTHATCH_B200_TENSOR_SOURCE_H_

#include <cstddef>
#include <memory>
#include <string>

namespace nuthatch {

class TensorSource {
 public:
  // nullptr if the file cannot be opened read-only.
  static std::unique_ptr<TensorSource> Open(const std::string& path);
  ~TensorSource();

  TensorSource(const TensorSource&) = delete;
  TensorSource& operator=(const TensorSource&) = delete;

  // Reads exactly `size` bytes at `offset` into `out`; false on a read error
  // or end of file before `size` bytes (tensor_source.cc:62-73).
  bool ReadAt(size_t offset, size_t size, void* out) const;

  size_t file_size() const { return size_; }

 private:
  TensorSource(int fd, size_t size) : fd_(fd), size_(size) {}
  int fd_ = -1;
  size_t size_ = 0;
};

}  // namespace nuthatch

#endif  // NUTHATCH_B200_TENSOR_SOURCE_H_

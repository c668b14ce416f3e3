// GGUF (v2/v3) metadata reader.  The reference parses GGUF through ggml's
// gguf.h (olmoe_model.cc:59-60, streaming_model.cc:22-23,
// expert_reader.cc:13-14); this is this project's own parser of the same
// on-disk format: header, typed key/value pairs, tensor infos, aligned data.
#ifndef NUTHATCH_B200_GGUF_FILE_H_
#define NUTHATCH_B200_GGUF_FILE_H_

#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

namespace nuthatch {

// ggml type ids this build supports on device.
enum GgmlType : int32_t { kTypeF32 = 0, kTypeQ4K = 12, kTypeQ6K = 14 };

// Bytes of one row of n values of `type` (0 if unsupported / not a block multiple).
size_t RowBytes(int32_t type, int64_t n);

struct GgufTensorInfo {
  std::string name;
  int32_t type = -1;
  int64_t ne[4] = {1, 1, 1, 1};
  uint32_t n_dims = 0;
  uint64_t offset = 0;  // absolute file offset of the data
  size_t nbytes = 0;
  size_t nb[4] = {0, 0, 0, 0};  // byte strides (nb[1] = row bytes)
};

class GgufFile {
 public:
  // nullptr on a missing file, bad magic/version, truncation or an
  // unsupported tensor type.
  static std::unique_ptr<GgufFile> Open(const std::string& path);

  bool GetU32(const std::string& key, uint32_t* out) const;
  bool GetF32(const std::string& key, float* out) const;
  bool GetStr(const std::string& key, std::string* out) const;

  const GgufTensorInfo* tensor(const std::string& name) const;
  const std::vector<GgufTensorInfo>& tensors() const { return tensors_; }
  uint64_t data_offset() const { return data_offset_; }
  uint32_t version() const { return version_; }

 private:
  uint32_t version_ = 0;
  uint64_t data_offset_ = 0;
  std::unordered_map<std::string, uint32_t> u32_;
  std::unordered_map<std::string, float> f32_;
  std::unordered_map<std::string, std::string> str_;
  std::vector<GgufTensorInfo> tensors_;
  std::unordered_map<std::string, size_t> index_;
};

// The string arrays stored under `keys` in a GGUF file's metadata (the
// tensor infos are not read, so any tensor types are fine).  Keys that are
// absent or hold another type are left out of *out.  false on a missing
// file, a bad header or truncated metadata.
bool ReadGgufStringArrays(const std::string& path, const std::vector<std::string>& keys,
                          std::unordered_map<std::string, std::vector<std::string>>* out);

}  // namespace nuthatch

#endif  // NUTHATCH_B200_GGUF_FILE_H_

// Per-expert byte slices of the fused *_exps tensors in a GGUF file
// (reference: src/model/expert_reader.h:10-43).  Expert e of a 3-D tensor
// [ne0, ne1, n_expert] is the nb[2]-byte slice at data_offset + tensor_offset
// + e*nb[2].
#ifndef NUTHATCH_B200_EXPERT_READER_H_
#define NUTHATCH_B200_EXPERT_READER_H_

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>

#include "nuthatch/tensor_source.h"

namespace nuthatch {

class ExpertReader {
 public:
  static std::unique_ptr<ExpertReader> Open(const std::string& gguf_path);

  ExpertReader(const ExpertReader&) = delete;
  ExpertReader& operator=(const ExpertReader&) = delete;

  size_t ExpertBytes(const std::string& tensor_name) const;  // 0 if absent
  int NumExperts(const std::string& tensor_name) const;      // 0 if absent
  int32_t ExpertType(const std::string& tensor_name) const;  // -1 if absent
  // Reads expert `expert_idx` of `tensor_name` into out (>= ExpertBytes bytes).
  bool ReadExpert(const std::string& tensor_name, int expert_idx, void* out) const;

  // Host-side fault injection for tests (no reference counterpart): after n
  // more successful ReadExpert calls every read fails as a short read would;
  // n < 0 turns it off.  Lets the failure handling of the slot cache be tested
  // without a failing disk.
  void FailReadsAfter(int64_t n) const { fail_after_ = n; }

 private:
  struct Info {
    uint64_t file_offset;
    size_t expert_bytes;
    int n_experts;
    int32_t type;
  };
  ExpertReader(std::unique_ptr<TensorSource> src, std::unordered_map<std::string, Info> info)
      : src_(std::move(src)), info_(std::move(info)) {}
  std::unique_ptr<TensorSource> src_;
  std::unordered_map<std::string, Info> info_;
  mutable int64_t fail_after_ = -1;
};

}  // namespace nuthatch

#endif  // NUTHATCH_B200_EXPERT_READER_H_

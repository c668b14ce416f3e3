// Streaming model (reference: src/model/streaming_model.h:17-44): non-expert
// weights resident in HBM; expert tensors (names containing "_exps.weight")
// are not uploaded.  Their bytes are kept in pinned host memory (the expert
// store the slot caches fill from) and remain readable from disk through
// reader().
#ifndef NUTHATCH_B200_STREAMING_MODEL_H_
#define NUTHATCH_B200_STREAMING_MODEL_H_

#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "nuthatch/expert_reader.h"
#include "nuthatch/expert_slot_cache.h"
#include "nuthatch/olmoe_model.h"

namespace nuthatch {

class StreamingModel {
 public:
  // pinned_store: also read every expert into pinned host memory (the H2D
  // source of the slot fills); otherwise misses read from disk per fill.
  static std::unique_ptr<StreamingModel> Load(const std::string& path, bool pinned_store = true);
  ~StreamingModel();

  StreamingModel(const StreamingModel&) = delete;
  StreamingModel& operator=(const StreamingModel&) = delete;

  const OlmoeConfig& config() const { return cfg_; }
  const DTensor* tensor(const std::string& name) const;  // nullptr for expert tensors
  const DTensor* layer_tensor(int layer, const std::string& suffix) const;
  ExpertReader* reader() const { return reader_.get(); }
  // Host store of one layer's experts (null pointers when not pinned).
  const ExpertHostStore* host_store(int layer) const;
  size_t resident_bytes() const { return bytes_; }

  // Per-layer slot pools of the last StreamingGenerate call and what they
  // were built for.
  struct SlotSet {
    int capacity = 0;
    SlotPolicy policy = SlotPolicy::kLru;
    uint32_t pin_slots = 0;
    std::vector<std::vector<uint32_t>> pinned;
    std::vector<std::unique_ptr<ExpertSlotCache>> caches;
  };
  struct Workspace;
  Workspace* workspace() const { return ws_.get(); }

 private:
  StreamingModel() = default;
  OlmoeConfig cfg_;
  void* base_ = nullptr;
  size_t bytes_ = 0;
  void* host_ = nullptr;
  std::unordered_map<std::string, DTensor> tensors_;
  std::unique_ptr<ExpertReader> reader_;
  std::vector<ExpertHostStore> stores_;
  std::unique_ptr<Workspace> ws_;
};

}  // namespace nuthatch

#endif  // NUTHATCH_B200_STREAMING_MODEL_H_

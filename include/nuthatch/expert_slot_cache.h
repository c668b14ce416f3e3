// HBM expert slot pool of one MoE layer (reference:
// src/model/expert_slot_cache.h:16-64, where the slots are host ggml tensors).
//
// Each slot holds one expert's gate, up and down bytes in their native GGUF
// layout; the three slot tensors are [.., .., C + staging] and the expert
// kernels read them with slot indices.  Ensure(ids) counts one hit or miss per
// distinct id in order and returns id -> slot.  Misses are filled from the
// pinned host expert store with cudaMemcpyAsync on the copy stream; the slot
// decisions are made here on the host.
//
// Policies:
//  * kLru (default, the reference's semantics): C slots, an empty slot first,
//    else the least recently used one is evicted (expert_slot_cache.cc:59-72).
//    Bit-identical hit/miss counts to LruPolicy(n_layers, C).
//  * kLearnedPin: `pin` slots preloaded at Create with the layer's hottest
//    experts from a usage histogram (always hit), the other C - pin slots an
//    LRU; counts equal LearnedPinPolicy(pin, C - pin).
// When a token routes to more distinct non-pinned experts than there are LRU
// slots (possible only for learned pin, or capacity < k), missed experts are
// staged in k extra staging slots for the compute and copied into their LRU
// slot afterwards, so the compute always sees every selected expert.
#ifndef NUTHATCH_B200_EXPERT_SLOT_CACHE_H_
#define NUTHATCH_B200_EXPERT_SLOT_CACHE_H_

#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "nuthatch/cache_policy.h"
#include "nuthatch/olmoe_model.h"

namespace nuthatch {

class ExpertReader;

// Where missing experts come from: pinned host bytes of each layer's fused
// gate/up/down tensors (expert e at base + e * expert_bytes).
struct ExpertHostStore {
  const uint8_t* gate = nullptr;
  const uint8_t* up = nullptr;
  const uint8_t* down = nullptr;
  size_t gate_bytes = 0, up_bytes = 0, down_bytes = 0;
  int32_t gate_type = -1, up_type = -1, down_type = -1;
  int n_experts = 0;
};

enum class SlotPolicy { kLru = 0, kLearnedPin = 1 };

struct SlotCacheOptions {
  SlotPolicy policy = SlotPolicy::kLru;
  uint32_t pin_slots = 0;              // learned pin only
  const UsageHistogram* usage = nullptr;  // learned pin only
  int staging = 0;                     // extra staging slots (set to k by the streaming driver)
  void* copy_stream = nullptr;         // cudaStream_t for the fills (nullptr: the legacy stream)
};

class ExpertSlotCache {
 public:
  // nullptr on capacity <= 0, a missing expert tensor or an allocation failure
  // (expert_slot_cache.cc:7-31).  With `store` null, misses read through
  // `reader` (disk -> pinned bounce buffer -> HBM).
  static std::unique_ptr<ExpertSlotCache> Create(const OlmoeConfig& cfg, int layer, int capacity,
                                                 ExpertReader* reader,
                                                 const ExpertHostStore* store = nullptr,
                                                 const SlotCacheOptions& opt = SlotCacheOptions());
  ~ExpertSlotCache();

  ExpertSlotCache(const ExpertSlotCache&) = delete;
  ExpertSlotCache& operator=(const ExpertSlotCache&) = delete;

  // Makes every id resident for the coming compute; returns id -> slot.
  // Duplicates within the batch count once.  Fills are enqueued on the copy
  // stream; call fills_done_event() / Commit() around the compute.
  std::unordered_map<int, int> Ensure(const std::vector<int>& expert_ids);
  // Enqueues the deferred staging -> LRU slot copies on `stream` after the compute.
  int Commit(void* stream);
  // Starts a new generation with the same slots: empties the LRU part, keeps
  // the pinned experts (their slots still hold them) and zeroes the counters.
  // Waits for this cache's copies in flight first.
  void Restart();
  // Event recorded after the last fill of the latest Ensure (cudaEvent_t).
  void* fills_done_event() const { return fill_event_; }
  // false when a fill of the last Ensure failed (a read error or short read
  // of the expert reader, or a copy that could not be enqueued); the slot
  // involved is left empty and mapped to no expert, so a later Ensure of the
  // same id misses and fills it again.  The reference ignores a failed read
  // (expert_slot_cache.cc:96) and maps the slot regardless.
  bool ok() const { return ok_; }

  const DTensor* gate_slots() const { return &gate_; }  // [n_embd, n_ff, slots]
  const DTensor* up_slots() const { return &up_; }
  const DTensor* down_slots() const { return &down_; }

  int capacity() const { return capacity_; }
  // Slots of the LRU part (capacity minus the pinned experts): the most
  // distinct unpinned experts one Ensure can hold without staging.
  int lru_slots() const { return lru_slots_; }
  bool is_pinned(int expert) const { return pinned_.count(expert) != 0; }
  int64_t hits() const { return hits_; }
  int64_t misses() const { return misses_; }
  uint64_t h2d_bytes() const { return h2d_bytes_; }

 private:
  ExpertSlotCache() = default;
  bool Fill(int slot, int expert);
  int AcquireLru();

  ExpertReader* reader_ = nullptr;
  ExpertHostStore store_;
  bool has_store_ = false;
  std::string gate_name_, up_name_, down_name_;
  DTensor gate_, up_, down_;
  void* base_ = nullptr;
  // Reader fills: a ring of pinned bounce buffers, each reused only after the
  // event recorded behind its last copies has completed, so the disk read of
  // one fill overlaps the host-to-device copies of the previous ones.
  static constexpr int kBounce = 3;
  void* bounce_[kBounce] = {nullptr, nullptr, nullptr};
  void* bounce_done_[kBounce] = {nullptr, nullptr, nullptr};
  int bounce_next_ = 0;
  void* copy_stream_ = nullptr;
  void* fill_event_ = nullptr;
  int capacity_ = 0;
  int lru_slots_ = 0;       // slots [pin_count_, pin_count_ + lru_slots_) are the LRU part
  int pin_count_ = 0;
  int staging_ = 0;         // slots [capacity_, capacity_ + staging_) stage over-subscribed misses
  SlotPolicy policy_ = SlotPolicy::kLru;
  std::unordered_map<int, int> pinned_;     // expert -> pinned slot
  std::unordered_map<int, int> id_to_slot_; // LRU part
  std::vector<int> slot_to_id_;
  std::vector<uint64_t> slot_tick_;
  uint64_t tick_ = 0;
  std::vector<std::pair<int, int>> pending_;  // (staging slot, LRU slot) copies after compute
  int64_t hits_ = 0;
  int64_t misses_ = 0;
  uint64_t h2d_bytes_ = 0;
  bool ok_ = true;
};

}  // namespace nuthatch

#endif  // NUTHATCH_B200_EXPERT_SLOT_CACHE_H_

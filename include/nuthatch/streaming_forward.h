// Two-phase streaming greedy generation (reference:
// src/model/streaming_forward.h:11-21, streaming_forward.cc:196-253).
//
// Per token and layer: phase A (attention with KV cache, residual, router)
// runs on the device and the selected global expert ids are read back; the
// host slot cache Ensure()s them (fills on the copy stream) and remaps them to
// slot ids; phase B (gate/up, down, weighted combine, residual) runs on the
// slot tensors.  Prompt tokens are fed one at a time, as in the reference.
#ifndef NUTHATCH_B200_STREAMING_FORWARD_H_
#define NUTHATCH_B200_STREAMING_FORWARD_H_

#include <cstdint>
#include <vector>

#include "nuthatch/cache_policy.h"
#include "nuthatch/expert_slot_cache.h"
#include "nuthatch/routing_trace.h"
#include "nuthatch/streaming_model.h"

namespace nuthatch {

struct StreamingStats {
  std::vector<int64_t> hits;    // per layer
  std::vector<int64_t> misses;  // per layer
  uint64_t h2d_bytes = 0;
  double fill_ms = 0;           // host time between phase A readback and phase B launch, summed
  int status = 0;
};

struct StreamingOptions {
  SlotPolicy policy = SlotPolicy::kLru;
  const UsageHistogram* usage = nullptr;  // learned pin
  uint32_t pin_slots = 0;                 // learned pin; 0 = LearnedPinSlots(capacity)
  RoutingTrace* trace = nullptr;
  StreamingStats* stats = nullptr;
};

// capacity >= 1; returns the n_predict new ids (empty for an empty prompt or
// n_predict <= 0, streaming_forward.cc:233).
std::vector<int32_t> StreamingGenerate(const StreamingModel& model, std::vector<int32_t> ids,
                                       int n_predict, bool norm_topk, int capacity);

std::vector<int32_t> StreamingGenerateEx(const StreamingModel& model, const std::vector<int32_t>& ids,
                                         int n_predict, bool norm_topk, int capacity,
                                         const StreamingOptions& opt);

}  // namespace nuthatch

#endif  // NUTHATCH_B200_STREAMING_FORWARD_H_

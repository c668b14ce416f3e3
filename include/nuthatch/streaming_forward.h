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
#include "nuthatch/generate.h"
#include "nuthatch/routing_trace.h"
#include "nuthatch/streaming_model.h"

namespace nuthatch {

struct StreamingStats {
  std::vector<int64_t> hits;    // per layer
  std::vector<int64_t> misses;  // per layer
  uint64_t h2d_bytes = 0;
  double fill_ms = 0;           // host time between phase A readback and phase B launch, summed
  int64_t waves = 0;            // batched form: slot-pool waves over all layers and steps
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

// Batched streaming decode (no reference counterpart; the reference streams
// one sequence and requires distinct(ids) <= capacity per layer,
// expert_slot_cache.h:21).  B sequences of equal prompt length advance in
// lockstep through the batched kernels while each layer's experts stream
// through a slot pool of `capacity` slots (policy as in StreamingOptions).
// The prompt runs as GreedyGenerateCachedBatch's does (positions 0..P-2 of
// every sequence in chunks of up to 512 rows), each chunk's experts streamed
// like a decode step's.
// When the batch selects more distinct experts than the pool holds, the layer
// runs in waves: the distinct unpinned experts, in order of first selection,
// lru_slots at a time, each wave made resident by one Ensure and its
// (token, pick) products run before the next wave's fills; the top-k-order
// combine follows the last wave.  Every sequence's ids equal the resident
// batched decode.  Hits and misses count per Ensure of each wave (the
// reference defines none for this case).  opt.trace is not filled; bopt gives
// the decode device time (the host decides every layer's slots, so no CUDA
// graph is used).  With bopt->ep set, every rank of the group calls this at
// once with its own sequences (the same count and lengths everywhere): each
// rank streams only its expert shard (E/N experts) through its own
// `capacity` slots per layer, learned pin choosing among those experts, and
// serves every rank's picks of them; tokens and selections are all-gathered
// and pick rows return by all-to-all as in GreedyGenerateCachedBatch, so the
// ids equal the single-GPU batch.  Hits, misses and waves are this rank's.
std::vector<std::vector<int32_t>> StreamingGenerateBatch(const StreamingModel& model,
                                                         const std::vector<std::vector<int32_t>>& prompts,
                                                         int n_predict, bool norm_topk, int capacity,
                                                         const StreamingOptions& opt, BatchOptions* bopt = nullptr);

}  // namespace nuthatch

#endif  // NUTHATCH_B200_STREAMING_FORWARD_H_

// Greedy generation on one B200 (reference: src/model/generate.h:16-33).
//
// Each token runs the per-token forward on the device: embedding, n_layers x
// (QKV, fused QK-norm/RoPE/KV-append/attention, output projection + residual,
// router top-k, expert gate/up SwiGLU, expert down + weighted combine +
// residual), output norm + lm_head + argmax.  The decode cursor lives in
// device memory, so the whole generation is enqueued without host round
// trips (one CUDA graph replay per token when graphs are on) and the host
// reads the generated ids once at the end.
#ifndef NUTHATCH_B200_GENERATE_H_
#define NUTHATCH_B200_GENERATE_H_

#include <cstdint>
#include <vector>

#include "nuthatch/olmoe_model.h"
#include "nuthatch/routing_trace.h"

namespace nuthatch {

// Optional outputs and switches (no reference counterpart: debugging and
// parity hooks).
struct GenerateOptions {
  bool use_graph = true;          // replay a captured CUDA graph per token
  RoutingTrace* trace = nullptr;  // routing records, token-major (generate.cc:154-166)
  std::vector<float>* trace_gap = nullptr;  // per (token, layer): k-th minus (k+1)-th probability
  std::vector<float>* hidden = nullptr;     // per step, per layer h after the MoE residual [n_predict][L][d]
  std::vector<float>* logits = nullptr;     // per step logits [n_predict][V]
  int status = 0;                            // NH_OK or the first error code
  // Out, when timed: device time (CUDA events on the decode stream) of the
  // batched prompt prefill and of the batch-1 steps after it.
  bool timed = false;
  double prefill_ms = 0, decode_ms = 0;
};

// Full recompute of the sequence every step (generate.cc:10-53).
std::vector<int32_t> GreedyGenerate(const OlmoeModel& model, std::vector<int32_t> ids,
                                    int n_predict, bool norm_topk);

// KV-cached greedy decode (generate.cc:55-106).  Returns the n_predict new ids.
std::vector<int32_t> GreedyGenerateCached(const OlmoeModel& model, std::vector<int32_t> ids,
                                          int n_predict, bool norm_topk);

// Same, with the routing of every processed token appended to *trace
// (generate.cc:108-181).
std::vector<int32_t> GreedyGenerateCachedTrace(const OlmoeModel& model, std::vector<int32_t> ids,
                                               int n_predict, bool norm_topk, RoutingTrace* trace);

// The general form used by the three above.
std::vector<int32_t> GreedyGenerateCachedEx(const OlmoeModel& model, const std::vector<int32_t>& ids,
                                            int n_predict, bool norm_topk, GenerateOptions* opt);

// Batched greedy decode (no reference counterpart: the batched overload the
// boundary needs for many independent sequences).  All prompts must have the
// same length; positions 0..P-2 of every sequence are prefilled in chunks of
// up to 512 rows (NH_BATCH_PREFILL=0: one position per step instead), then
// each sequence advances one position per step in lockstep with its own KV
// cache, and its ids equal GreedyGenerateCached on it alone.
//
// Expert parallelism (ep set): every rank of the group calls this at once with
// its own share of the sequences (the same count on every rank) and a model
// holding the rank's expert shard (OlmoeModel::LoadExpertShard with
// ExpertShard::Of) or all experts; see nuthatch/expert_parallel.h.
class ExpertGroup;
struct BatchOptions {
  bool use_graph = true;            // replay a captured CUDA graph per step
  const ExpertGroup* ep = nullptr;  // expert-parallel group, or single GPU
  double decode_ms = 0;             // out: device time from the last prompt position to the end
  double prefill_ms = 0;            // out: device time of the chunked prompt prefill (0 without one)
  int status = 0;                   // out: NH_OK or the first error code
};
std::vector<std::vector<int32_t>> GreedyGenerateCachedBatch(const OlmoeModel& model,
                                                            const std::vector<std::vector<int32_t>>& prompts,
                                                            int n_predict, bool norm_topk,
                                                            BatchOptions* opt = nullptr);

}  // namespace nuthatch

#endif  // NUTHATCH_B200_GENERATE_H_

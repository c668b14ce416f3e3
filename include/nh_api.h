/* nh_api.h — C ABI of the host library (libnuthatch_b200.so) for FFI
 * callers (ctypes, cgo, JNI).  Each function wraps the C++ surface in
 * the headers of include/nuthatch/, which mirror the reference's C++ API (namespace
 * nuthatch); citations are to the reference function each one replaces.
 *
 * Conventions: objects are opaque pointers, NULL on failure (as the
 * reference's factories return nullptr); other calls return NH_OK (0) or a
 * negative NH_E_* code from nh_kernels.h.  All buffers are host memory.
 * Calls on one object are not thread-safe (the reference's are
 * single-threaded too).
 */
#ifndef NH_API_H_
#define NH_API_H_

#include <stdint.h>

#include "nh_kernels.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct NhConfig {
  uint32_t n_layers, n_embd, n_head, n_head_kv, n_ff, n_expert, n_expert_used, n_vocab, n_ctx_train;
  float rope_freq_base, rms_eps;
} NhConfig;

const char* nh_version(void);
/* cudaSetDevice; later loads and calls use that device. */
int nh_set_device(int device);
/* Text of the last error set on this thread ("" if none). */
const char* nh_last_error(void);

/* Host-only metadata read: ParseOlmoeConfig (olmoe_model.cc:31-54) on the
 * file's GGUF header; returns the tensor count or a negative code.  Touches no
 * GPU. */
int nh_gguf_probe(const char* path, NhConfig* out);

/* OlmoeModel::Load (olmoe_model.cc:56-71): the whole GGUF resident in HBM. */
void* nh_model_load(const char* path);
void nh_model_free(void* model);
int nh_model_config(const void* model, NhConfig* out);
/* Device tensor lookup (OlmoeModel::tensor, olmoe_model.cc:86-89). */
int nh_model_tensor(const void* model, const char* name, int64_t ne[4], int32_t* type, void** data,
                    uint64_t* nbytes);

/* Greedy generation.  mode 0: GreedyGenerateCached (generate.cc:55-106);
 * mode 1: GreedyGenerate, full recompute per step (generate.cc:10-53).
 * Writes n_predict ids to out_tokens.  Optional outputs (NULL to skip; mode
 * 0 only), token-major over the n_prompt + n_predict - 1 processed tokens:
 * trace_sel [n_tok][n_layers][n_expert_used] (GreedyGenerateCachedTrace,
 * generate.cc:108-181), trace_gap [n_tok][n_layers]; per generated step:
 * hidden [n_predict][n_layers][n_embd] (h after each layer's MoE residual),
 * logits [n_predict][n_vocab].  use_graph: replay one captured CUDA graph
 * per token. */
int nh_generate(void* model, int mode, const int32_t* prompt, int n_prompt, int n_predict, int norm_topk,
                int use_graph, int32_t* out_tokens, int32_t* trace_sel, float* trace_gap, float* hidden,
                float* logits);
/* GreedyGenerateCached (mode 0 of nh_generate) with the device time of its
 * two parts: the batched prefill of the prompt positions before the last
 * (prefill_ms; 0 when the prompt ran position by position) and the batch-1
 * steps from the last prompt position on (decode_ms).  Either may be NULL. */
int nh_generate_timed(void* model, const int32_t* prompt, int n_prompt, int n_predict, int norm_topk,
                      int32_t* out_tokens, double* prefill_ms, double* decode_ms);
/* Kernel launches per decode step of this model. */
int nh_generate_launches(const void* model);

/* Batched greedy decode (GreedyGenerateCachedBatch): n_seq prompts of
 * n_prompt ids each (prompts [n_seq][n_prompt]); writes out_tokens
 * [n_seq][n_predict] and, when decode_ms is not null, the device time of the
 * decode part (last prompt position onwards). */
int nh_generate_batch(void* model, const int32_t* prompts, int n_seq, int n_prompt, int n_predict, int norm_topk,
                      int use_graph, int32_t* out_tokens, double* decode_ms);

/* Expert parallelism over the GPUs of one node (no reference counterpart; the
 * EP configuration {world, rank, communicator} of the drop-in boundary, see
 * include/nuthatch/expert_parallel.h).  One process per GPU:
 *   rank 0: nh_ep_new_id(id) and hand the 128 id bytes to every rank;
 *   every rank: ep = nh_ep_create(id, world, rank) on its device (collective),
 *   model = nh_model_load_expert_shard(path, rank * E/world, E/world), then
 *   nh_generate_batch_ep(model, ep, its own n_seq prompts, ...) on all ranks
 *   at once (the same n_seq, n_prompt and n_predict everywhere); free the
 *   model and nh_ep_free(ep) before the process group that carried the id.
 * nh_ep_new_id returns NH_E_STATE when NCCL cannot be loaded; nh_ep_create
 * and the shard load return NULL on failure.  The shard model serves only
 * nh_generate_batch_ep; the single-GPU generate calls refuse it (NH_E_STATE). */
int nh_ep_new_id(uint8_t* id);
void* nh_ep_create(const uint8_t* id, int world, int rank);
void nh_ep_free(void* ep);
void* nh_model_load_expert_shard(const char* path, uint32_t first, uint32_t count);
int nh_generate_batch_ep(void* model, const void* ep, const int32_t* prompts, int n_seq, int n_prompt, int n_predict,
                         int norm_topk, int use_graph, int32_t* out_tokens, double* decode_ms);

/* Both batched forms with the device time split in two (ep NULL: one GPU):
 * the chunked prefill of the prompt positions before the last (prefill_ms, 0
 * when the prompt ran one position per step) and the steps from the last
 * prompt position on (decode_ms).  Either pointer may be NULL. */
int nh_generate_batch_timed(void* model, const void* ep, const int32_t* prompts, int n_seq, int n_prompt,
                            int n_predict, int norm_topk, int use_graph, int32_t* out_tokens, double* prefill_ms,
                            double* decode_ms);

/* Decode replay for timing (no reference counterpart; the reference times
 * whole generate calls).  prepare: runs the prompt's first n_prompt-1
 * positions and saves the cursor (synchronises).  run: restores the cursor
 * and enqueues the n_predict decode positions (the last prompt token first)
 * as CUDA graph replays on the model's stream; asynchronous.  result: waits
 * and copies the ids of the last run.  stream: the model's cudaStream_t.
 * kernel_loop: enqueues reps passes over all layers of one kernel (0 expert
 * gate/up, 1 expert down, 2 QKV, 3 the fused MoE block nh_moe_layer) on that
 * stream; returns launches. */
int nh_decode_prepare(void* model, const int32_t* prompt, int n_prompt, int n_predict);
int nh_decode_run(void* model, int n_predict);
int nh_decode_result(void* model, int n_predict, int32_t* out_tokens);
void* nh_model_stream(void* model);
int nh_decode_kernel_loop(void* model, int which, int reps);

/* StreamingModel::Load (streaming_model.cc:19-86); pinned_store: keep every
 * expert in pinned host memory as the fill source. */
void* nh_stream_model_load(const char* path, int pinned_store);
void nh_stream_model_free(void* model);
int nh_stream_model_config(const void* model, NhConfig* out);

/* StreamingGenerate (streaming_forward.cc:228-253) with a slot policy:
 * policy 0 LRU (the reference's ExpertSlotCache), 1 learned pin with
 * pin_slots pinned (0: ceil(3*capacity/4)) chosen from usage
 * [n_layers][n_expert] counts.  hits/misses: [n_layers]. */
int nh_stream_generate(void* model, const int32_t* prompt, int n_prompt, int n_predict, int norm_topk,
                       int capacity, int policy, int pin_slots, const uint64_t* usage, int32_t* out_tokens,
                       int64_t* hits, int64_t* misses, uint64_t* h2d_bytes, int32_t* trace_sel);

/* StreamingGenerateBatch (no reference counterpart): n_seq prompts of n_prompt
 * ids decoded in lockstep with every layer's experts streamed through a slot
 * pool of `capacity` (policy, pin_slots, usage as nh_stream_generate); layers
 * whose batch selects more distinct experts than the pool holds run in waves.
 * out_tokens [n_seq][n_predict]; hits/misses [n_layers] (per wave's Ensure);
 * waves: slot-pool waves over all layers and steps; decode_ms: device time
 * from the last prompt position on.  Optional outputs may be NULL. */
int nh_stream_generate_batch(void* model, const int32_t* prompts, int n_seq, int n_prompt, int n_predict,
                             int norm_topk, int capacity, int policy, int pin_slots, const uint64_t* usage,
                             int32_t* out_tokens, int64_t* hits, int64_t* misses, uint64_t* h2d_bytes, int64_t* waves,
                             double* decode_ms);

/* nh_stream_generate_batch with expert parallelism (ep from nh_ep_create, or
 * NULL for one GPU): every rank calls it at once with its own n_seq prompts
 * (the same n_seq, n_prompt and n_predict everywhere); each rank streams only
 * its expert shard (n_expert / world experts) through `capacity` slots per
 * layer, learned pin choosing among those experts.  hits, misses, h2d_bytes
 * and waves are this rank's. */
int nh_stream_generate_batch_ep(void* model, const void* ep, const int32_t* prompts, int n_seq, int n_prompt,
                                int n_predict, int norm_topk, int capacity, int policy, int pin_slots,
                                const uint64_t* usage, int32_t* out_tokens, int64_t* hits, int64_t* misses,
                                uint64_t* h2d_bytes, int64_t* waves, double* decode_ms);

/* The slot-pool waves of one layer of the batched streaming form (host only,
 * no GPU needed): over n_picks selections sel [token][k], the distinct
 * unpinned experts in [e_lo, e_hi) in order of first selection, `per` to a
 * wave, with the selected pinned experts (pinned[e] != 0) joining wave 0
 * after its unpinned ones.  wave_of [n_expert]: each expert's wave or -1;
 * wave_size [n_expert] and wave_experts [n_expert]: the waves' id lists, one
 * after the other.  Returns the wave count (>= 1), NH_E_STATE for a selection
 * outside [0, n_expert), NH_E_CAPACITY for an unpinned expert with per <= 0. */
int nh_plan_waves(const int32_t* sel, int n_picks, int n_expert, int e_lo, int e_hi, int per, const uint8_t* pinned,
                  int32_t* wave_of, int32_t* wave_size, int32_t* wave_experts);

/* The pairs of wave w grouped by slot (slot_of [n_expert]: each expert's slot
 * after that wave's Ensure): off/cnt [slots]; for pair i in slot order,
 * (token, pick) order within a slot, act[i] = j / k and out[i] = j (act and
 * out hold up to n_picks entries).  Returns the pair count, or NH_E_STATE
 * when an expert of the wave has no slot in [0, slots). */
int nh_group_wave_pairs(const int32_t* sel, int n_picks, int k, int n_expert, const int32_t* wave_of, int w,
                        const int32_t* slot_of, int slots, int32_t* off, int32_t* cnt, int32_t* act, int32_t* out);

/* Tokenizer (tokenizer.h; the reference's src/tokenizer/tokenizer.h).  Load
 * reads tokenizer.ggml.tokens / .merges of a GGUF (NULL without a
 * vocabulary); from_lists takes NUL-terminated strings (NULL if any is NULL).  encode / decode /
 * token return the full count of ids or bytes and write at most `cap` of
 * them; split returns the pre-split chunk count and writes [begin, end) byte
 * offsets of at most `cap` chunks (2 entries each).  Host only. */
void* nh_tokenizer_load(const char* path);
void* nh_tokenizer_from_lists(const char* const* vocab, int64_t n_vocab, const char* const* merges,
                              int64_t n_merges);
void nh_tokenizer_free(void* tok);
int64_t nh_tokenizer_vocab_size(const void* tok);
int64_t nh_tokenizer_encode(const void* tok, const char* text, int64_t len, int32_t* ids, int64_t cap);
int64_t nh_tokenizer_decode(const void* tok, const int32_t* ids, int64_t n, char* out, int64_t cap);
int64_t nh_tokenizer_token(const void* tok, int32_t id, char* out, int64_t cap);
int64_t nh_tokenizer_split(const char* text, int64_t len, int64_t* bounds, int64_t cap);

/* Cache policies over a flat trace: record r has layer[r] and experts
 * experts[offsets[r]..offsets[r+1]).  kind 0 LruPolicy(n_layers, a)
 * (lru_policy.cc), 1 OsPageCachePolicy(a) (os_page_cache_policy.cc), 2
 * LearnedPinPolicy(n_layers, pin=a, lru=b, usage) (learned_pin_policy.cc)
 * with usage [n_layers][n_expert] counts, or BuildUsage(trace) when usage is
 * NULL.  Returns hits; *accesses gets the access count. */
int64_t nh_replay(int kind, uint32_t n_layers, uint32_t n_expert, int64_t n_records, const uint32_t* layer,
                  const int64_t* offsets, const uint32_t* experts, uint32_t a, uint32_t b, const uint64_t* usage,
                  int64_t* accesses);
/* SweepBudgets (trace_sweep.cc:10-34): out[3*i..] = learned, lru, os hit rates. */
int nh_sweep_budgets(uint32_t n_layers, uint32_t n_expert, int64_t n_records, const uint32_t* layer,
                     const int64_t* offsets, const uint32_t* experts, const uint32_t* budgets, int n_budgets,
                     double* out);
/* SweepBudgetsCalibrated (no reference counterpart; the out-of-sample form):
 * learned pin's usage histogram from the calibration trace (cal_*), every
 * policy replaying the evaluation trace; out as nh_sweep_budgets. */
int nh_sweep_budgets_calibrated(uint32_t n_layers, uint32_t n_expert, int64_t cal_records, const uint32_t* cal_layer,
                                const int64_t* cal_offsets, const uint32_t* cal_experts, int64_t n_records,
                                const uint32_t* layer, const int64_t* offsets, const uint32_t* experts,
                                const uint32_t* budgets, int n_budgets, double* out);
/* SweepPinRatio (trace_sweep.cc:36-50): out[pin] = learned hit rate. */
int nh_sweep_pin_ratio(uint32_t n_layers, uint32_t n_expert, int64_t n_records, const uint32_t* layer,
                       const int64_t* offsets, const uint32_t* experts, uint32_t budget, double* out);

/* WriteRoutingTrace / ReadRoutingTrace / ReadRoutingTraceText
 * (routing_trace.cc:28-111).  Read: call with caps 0 to get the record count
 * (return) and *n_experts_total, then again with buffers. */
int nh_trace_write(const char* path, uint32_t n_layers, uint32_t n_expert, int64_t n_records,
                   const uint32_t* token, const uint32_t* layer, const int64_t* offsets, const uint32_t* experts);
int64_t nh_trace_read(const char* path, int text, uint32_t* n_layers, uint32_t* n_expert, int64_t* n_experts_total,
                      int64_t cap_records, int64_t cap_experts, uint32_t* token, uint32_t* layer, int64_t* offsets,
                      uint32_t* experts);

/* ExpertReader (expert_reader.cc:10-69). */
void* nh_expert_reader_open(const char* gguf_path);
void nh_expert_reader_free(void* reader);
uint64_t nh_expert_reader_bytes(const void* reader, const char* tensor);
int nh_expert_reader_read(const void* reader, const char* tensor, int expert, void* out);
/* Host-side fault injection for tests (no reference counterpart): after n more
 * successful expert reads every read of this reader fails as a short read
 * would; n < 0 turns it off (ExpertReader::FailReadsAfter). */
int nh_expert_reader_fail_after(void* reader, int64_t n);

/* ExpertSlotCache (expert_slot_cache.cc:7-104) over a reader; policy as in
 * nh_stream_generate.  ensure: writes the slot of each of the n ids. */
void* nh_slot_cache_create(const NhConfig* cfg, int layer, int capacity, void* reader, int policy, int pin_slots,
                           const uint64_t* usage_layer /* [n_expert] or NULL */);
void nh_slot_cache_free(void* cache);
int nh_slot_cache_ensure(void* cache, const int32_t* ids, int n, int32_t* slots);
int64_t nh_slot_cache_hits(const void* cache);
int64_t nh_slot_cache_misses(const void* cache);
/* Copies the device bytes of slot `slot` of tensor which (0 gate, 1 up,
 * 2 down) to host `out` (synchronises). */
int nh_slot_cache_read_slot(const void* cache, int which, int slot, void* out, uint64_t bytes);

#ifdef __cplusplus
}
#endif

#endif /* NH_API_H_ */

// Internal: the device workspace and per-token kernel sequence shared by the
// resident (generate.cc) and streaming (streaming_forward.cc) drivers.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <vector>

#include "../../../include/nh_kernels.h"
#include "nuthatch/kv_cache.h"
#include "nuthatch/olmoe_model.h"

namespace nuthatch {

struct LayerView {
  const float* attn_norm = nullptr;
  const void* wq = nullptr;
  const void* wk = nullptr;
  const void* wv = nullptr;
  const void* wo = nullptr;
  int32_t tq = 0, tk = 0, tv = 0, to = 0;
  const float* q_norm = nullptr;
  const float* k_norm = nullptr;
  const float* ffn_norm = nullptr;
  const float* router = nullptr;
  const void* gate = nullptr;
  const void* up = nullptr;
  const void* down = nullptr;
  int32_t tg = 0, tu = 0, td = 0;
  uint64_t gate_nb2 = 0, up_nb2 = 0, down_nb2 = 0;
};

struct ModelView {
  OlmoeConfig cfg;
  const void* embd = nullptr;
  int32_t te = 0;
  std::vector<LayerView> layers;
  const float* out_norm = nullptr;
  const void* out = nullptr;
  int32_t tout = 0;
};

// Builds the view over resident tensors (experts included when `experts`).
// Returns false when a required tensor is missing or has the wrong shape.
template <typename M>
bool BuildView(const M& m, bool experts, ModelView* v);

// Device buffers of a chunk of prefill rows (Engine::Prefill), sized for
// `rows` token positions.
struct PrefillBuffers {
  ~PrefillBuffers();
  int Reserve(const OlmoeConfig& c, int rows);
  void Release();
  int rows = 0;
  float *h = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *qr = nullptr, *att = nullptr, *xn = nullptr;
  float *wts = nullptr, *ff = nullptr, *y = nullptr;
  uint8_t *q8 = nullptr, *q8ff = nullptr;
  int32_t *sel = nullptr, *off = nullptr, *cnt = nullptr, *act_idx = nullptr, *out_idx = nullptr;
};

class Engine {
 public:
  explicit Engine(const OlmoeConfig& cfg);
  ~Engine();

  // Ensures buffers for sequences up to max_seq positions, prompts up to
  // max_prompt ids and n_predict up to max_predict; allocates the dump
  // buffers when `dumps`.  Returns NH_OK or an error code.
  int Reserve(int max_seq, int max_prompt, int max_predict, bool dumps);

  // Uploads the prompt and resets the decode cursor to start_pos (async on
  // stream()); start_pos > 0 when Prefill fills positions 0..start_pos-1.
  int Begin(const int32_t* prompt, int n_prompt, int n_predict, int start_pos = 0);

  // One-shot prompt prefill, the reference's first GreedyGenerateCached step
  // (generate.cc:63-91, forward.cc:45-79): positions 0..n_tok-1 of the
  // uploaded prompt run through the batched kernels in chunks of up to
  // kPrefillChunk positions (grouped expert products, causal prefill
  // attention), writing their K/V rows and, with `trace`, their routing.  Per
  // position the arithmetic is that of the batch-1 step, so the cache and the
  // ids that follow are identical.  No logits are formed for these positions
  // (only the last prompt position's are used, and the batch-1 step forms
  // them).
  static constexpr int kPrefillChunk = 512;
  int Prefill(const ModelView& m, int n_tok, bool norm_topk, bool trace);
  // Whether the batched kernels cover this model's shapes and weight types.
  // experts_resident false: the view has no expert tensors (they stream
  // through slot pools); only the other tensors are checked.
  static bool PrefillSupported(const ModelView& m, bool experts_resident = true);

  int EnqueueEmbed(const ModelView& m);
  // QKV, attention and the output projection of one layer.
  int EnqueueAttention(const ModelView& m, int layer);
  // EnqueueAttention plus the router (phase A of the two-phase form).
  int EnqueueAttnPhase(const ModelView& m, int layer, bool norm_topk, bool trace);
  // After a phase A: enqueues the hand-over of the router's selection to
  // mapped host memory, then waits on the host (spinning, at most timeout_s)
  // until it has arrived and copies it to sel_host().  No stream
  // synchronisation: work enqueued before the call keeps running.
  int AwaitSelection(double timeout_s);
  // The whole MoE block of a resident layer in one cooperative kernel;
  // NH_E_ARG / NH_E_TYPE (nothing enqueued) where that kernel does not cover
  // the shapes.
  int EnqueueFusedMoe(const ModelView& m, int layer, bool norm_topk, bool trace, bool dumps);
  // Phase B over expert weights at gate/up/down with per-slot selection
  // wsel (device memory) or, when slots_host is not null, the host's slots.
  int EnqueueMoePhase(const ModelView& m, int layer, const void* gate, int32_t tg, uint64_t gnb2,
                      const void* up, int32_t tu, uint64_t unb2, const void* down, int32_t td,
                      uint64_t dnb2, const int32_t* wsel, bool dumps, const int32_t* slots_host = nullptr);
  int EnqueueFinal(const ModelView& m, bool dumps);
  int EnqueueStep(const ModelView& m, bool norm_topk, bool trace, bool dumps);

  // Runs `steps` resident decode steps, via a captured CUDA graph when use_graph.
  int RunSteps(const ModelView& m, int steps, bool norm_topk, bool trace, bool dumps, bool use_graph);

  // Reads back the generated ids and the kernel error word (synchronises).
  int Finish(int n_predict, std::vector<int32_t>* out);

  // Decode-cursor snapshot: Save (synchronises) records the device cursor;
  // Restore enqueues its upload, so a decode can be replayed from that point.
  int SaveState();
  int RestoreState();
  // Enqueues `reps` passes over all layers of one kernel with the current
  // activations (0 expert gate/up, 1 expert down, 2 QKV, 3 the fused MoE
  // block, 4 the whole-layer kernel; 3 and 4 also update the residual);
  // returns launches.
  int KernelLoop(const ModelView& m, int which, int reps);
  void FillMoeLayer(const ModelView& m, int layer, bool norm_topk, bool trace, bool dumps, NhMoeLayer* out);
  // Kernels the last enqueued resident step launched (0 before the first).
  int step_launches() const { return step_launches_; }

  cudaStream_t stream() const { return stream_; }
  int32_t* sel_dev() const { return sel_; }
  int32_t* wsel_dev() const { return wsel_; }
  int32_t* sel_host() const { return sel_host_; }
  int32_t* wsel_host() const { return wsel_host_; }
  const int32_t* trace_sel_dev() const { return trace_sel_; }
  const float* trace_gap_dev() const { return trace_gap_; }
  const float* dump_hidden_dev() const { return dump_hidden_; }
  const float* dump_logits_dev() const { return dump_logits_; }
  int max_seq() const { return max_seq_; }
  int launches_per_step() const { return 2 + 6 * static_cast<int>(cfg_.n_layers); }

 private:
  void FreeAll();
  OlmoeConfig cfg_;
  std::unique_ptr<PrefillBuffers> pf_;
  cudaStream_t stream_ = nullptr;
  int max_seq_ = 0, max_prompt_ = 0, max_predict_ = 0;
  bool dumps_ = false;
  std::unique_ptr<KvCache> kv_;
  NhDecodeState* state_ = nullptr;
  NhDecodeState* state_host_ = nullptr;
  NhDecodeState* state_saved_ = nullptr;
  int32_t* prompt_ = nullptr;
  int32_t* prompt_host_ = nullptr;
  int32_t* out_ = nullptr;
  int32_t* out_host_ = nullptr;
  float* h_ = nullptr;
  float* q_ = nullptr;
  float* k_ = nullptr;
  float* v_ = nullptr;
  float* attn_ = nullptr;
  int32_t* sel_ = nullptr;
  int32_t* wsel_ = nullptr;
  int32_t* sel_host_ = nullptr;
  int32_t* wsel_host_ = nullptr;
  // Mapped pinned host memory the selection is published into: ids, then a
  // sequence number (host and device addresses), and the last number used.
  int32_t* pub_sel_ = nullptr;
  uint32_t* pub_seq_ = nullptr;
  int32_t* pub_sel_dev_ = nullptr;
  uint32_t* pub_seq_dev_ = nullptr;
  uint32_t pub_count_ = 0;
  float* wts_ = nullptr;
  float* ff_ = nullptr;
  float* rope_cs_ = nullptr;
  void* attn_scratch_ = nullptr;
  void* router_scratch_ = nullptr;
  void* moe_scratch_ = nullptr;
  void* argmax_scratch_ = nullptr;
  int32_t* trace_sel_ = nullptr;
  float* trace_gap_ = nullptr;
  float* dump_hidden_ = nullptr;
  float* dump_logits_ = nullptr;
  cudaGraphExec_t graph_ = nullptr;
  uint64_t graph_key_ = ~0ull;
  uint64_t alloc_gen_ = 0;
  int step_launches_ = 0;
};

}  // namespace nuthatch

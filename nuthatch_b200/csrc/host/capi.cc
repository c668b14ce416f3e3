// extern "C" wrappers over the C++ surface (include/nh_api.h).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>

#include "../../../include/nh_api.h"
#include "nuthatch/cache_policy.h"
#include "nuthatch/expert_parallel.h"
#include "nuthatch/expert_reader.h"
#include "nuthatch/expert_slot_cache.h"
#include "nuthatch/generate.h"
#include "nuthatch/gguf_file.h"
#include "nuthatch/olmoe_model.h"
#include "nuthatch/routing_trace.h"
#include "nuthatch/streaming_forward.h"
#include "nuthatch/streaming_model.h"
#include "nuthatch/tokenizer.h"
#include "wave_plan.h"
#include "workspace.h"

using namespace nuthatch;

namespace {

thread_local std::string g_err;

void SetErr(const std::string& s) { g_err = s; }

void FillConfig(const OlmoeConfig& c, NhConfig* o) {
  *o = NhConfig{c.n_layers, c.n_embd,   c.n_head,        c.n_head_kv, c.n_ff, c.n_expert, c.n_expert_used,
                c.n_vocab,  c.n_ctx_train, c.rope_freq_base, c.rms_eps};
}

RoutingTrace MakeTrace(uint32_t n_layers, uint32_t n_expert, int64_t n_records, const uint32_t* token,
                       const uint32_t* layer, const int64_t* offsets, const uint32_t* experts) {
  RoutingTrace t;
  t.n_layers = n_layers;
  t.n_expert = n_expert;
  t.records.reserve(static_cast<size_t>(n_records));
  for (int64_t r = 0; r < n_records; ++r) {
    RoutingRecord rec;
    rec.token = token != nullptr ? token[r] : static_cast<uint32_t>(r);
    rec.layer = layer[r];
    rec.experts.assign(experts + offsets[r], experts + offsets[r + 1]);
    t.records.push_back(std::move(rec));
  }
  return t;
}

UsageHistogram DenseUsage(const uint64_t* usage, uint32_t n_layers, uint32_t n_expert) {
  UsageHistogram u;
  u.per_layer.resize(n_layers);
  if (usage == nullptr) return u;
  for (uint32_t l = 0; l < n_layers; ++l)
    for (uint32_t e = 0; e < n_expert; ++e)
      if (usage[static_cast<size_t>(l) * n_expert + e] > 0) u.per_layer[l][e] = usage[static_cast<size_t>(l) * n_expert + e];
  return u;
}

struct SlotCacheHandle {
  std::unique_ptr<ExpertSlotCache> cache;
  UsageHistogram usage;
  cudaStream_t stream = nullptr;
};

}  // namespace

extern "C" {

const char* nh_version(void) { return "nuthatch-b200 0.1.0"; }

int nh_set_device(int device) { return cudaSetDevice(device) == cudaSuccess ? NH_OK : NH_E_CUDA; }

const char* nh_last_error(void) { return g_err.c_str(); }

int nh_gguf_probe(const char* path, NhConfig* out) {
  if (path == nullptr || out == nullptr) return NH_E_ARG;
  auto g = GgufFile::Open(path);
  if (g == nullptr) return NH_E_IO;
  FillConfig(ParseOlmoeConfig(*g), out);
  return static_cast<int>(g->tensors().size());
}

void* nh_model_load(const char* path) {
  if (path == nullptr) return nullptr;
  auto m = OlmoeModel::Load(path);
  if (m == nullptr) SetErr(std::string("OlmoeModel::Load failed: ") + path);
  return m.release();
}

void nh_model_free(void* model) { delete static_cast<OlmoeModel*>(model); }

int nh_model_config(const void* model, NhConfig* out) {
  if (model == nullptr || out == nullptr) return NH_E_ARG;
  FillConfig(static_cast<const OlmoeModel*>(model)->config(), out);
  return NH_OK;
}

int nh_model_tensor(const void* model, const char* name, int64_t ne[4], int32_t* type, void** data, uint64_t* nbytes) {
  if (model == nullptr || name == nullptr) return NH_E_ARG;
  const DTensor* t = static_cast<const OlmoeModel*>(model)->tensor(name);
  if (t == nullptr) return NH_E_ARG;
  for (int i = 0; i < 4; ++i) ne[i] = t->ne[i];
  *type = t->type;
  *data = t->data;
  *nbytes = t->nbytes;
  return NH_OK;
}

int nh_generate(void* model, int mode, const int32_t* prompt, int n_prompt, int n_predict, int norm_topk,
                int use_graph, int32_t* out_tokens, int32_t* trace_sel, float* trace_gap, float* hidden,
                float* logits) {
  if (model == nullptr || (n_prompt > 0 && prompt == nullptr) || (n_predict > 0 && out_tokens == nullptr))
    return NH_E_ARG;
  const OlmoeModel& m = *static_cast<OlmoeModel*>(model);
  std::vector<int32_t> ids(prompt, prompt + (n_prompt > 0 ? n_prompt : 0));
  if (n_prompt <= 0 || n_predict <= 0) return NH_OK;
  std::vector<int32_t> out;
  if (mode == 1) {
    out = GreedyGenerate(m, ids, n_predict, norm_topk != 0);
    if (static_cast<int>(out.size()) != n_predict) return NH_E_CUDA;
  } else {
    GenerateOptions o;
    o.use_graph = use_graph != 0;
    RoutingTrace tr;
    std::vector<float> gap, hid, lg;
    if (trace_sel != nullptr) o.trace = &tr;
    if (trace_gap != nullptr) o.trace_gap = &gap;
    if (hidden != nullptr) o.hidden = &hid;
    if (logits != nullptr) o.logits = &lg;
    out = GreedyGenerateCachedEx(m, ids, n_predict, norm_topk != 0, &o);
    if (o.status != NH_OK) {
      SetErr("GreedyGenerateCached failed");
      return o.status;
    }
    if (trace_sel != nullptr) {
      size_t k = 0;
      for (const RoutingRecord& r : tr.records)
        for (uint32_t e : r.experts) trace_sel[k++] = static_cast<int32_t>(e);
    }
    if (trace_gap != nullptr) std::memcpy(trace_gap, gap.data(), gap.size() * 4);
    if (hidden != nullptr) std::memcpy(hidden, hid.data(), hid.size() * 4);
    if (logits != nullptr) std::memcpy(logits, lg.data(), lg.size() * 4);
  }
  std::memcpy(out_tokens, out.data(), out.size() * 4);
  return NH_OK;
}

int nh_generate_timed(void* model, const int32_t* prompt, int n_prompt, int n_predict, int norm_topk,
                      int32_t* out_tokens, double* prefill_ms, double* decode_ms) {
  if (model == nullptr || prompt == nullptr || out_tokens == nullptr || n_prompt <= 0 || n_predict <= 0)
    return NH_E_ARG;
  GenerateOptions o;
  o.timed = true;
  std::vector<int32_t> ids(prompt, prompt + n_prompt);
  const std::vector<int32_t> out =
      GreedyGenerateCachedEx(*static_cast<OlmoeModel*>(model), ids, n_predict, norm_topk != 0, &o);
  if (o.status != NH_OK) {
    SetErr("GreedyGenerateCached failed");
    return o.status;
  }
  std::memcpy(out_tokens, out.data(), out.size() * 4);
  if (prefill_ms != nullptr) *prefill_ms = o.prefill_ms;
  if (decode_ms != nullptr) *decode_ms = o.decode_ms;
  return NH_OK;
}

int nh_generate_launches(const void* model) {
  if (model == nullptr) return NH_E_ARG;
  // The count the last resident step enqueued (four or six kernels per
  // layer, with or without the fused MoE block); before any step, the
  // six-kernel form's count.
  const auto* m = static_cast<const OlmoeModel*>(model);
  const int n = m->workspace() != nullptr ? m->workspace()->engine.step_launches() : 0;
  return n > 0 ? n : 2 + 6 * static_cast<int>(m->config().n_layers);
}

int nh_generate_batch_timed(void* model, const void* ep, const int32_t* prompts, int n_seq, int n_prompt,
                            int n_predict, int norm_topk, int use_graph, int32_t* out_tokens, double* prefill_ms,
                            double* decode_ms) {
  if (model == nullptr || prompts == nullptr || out_tokens == nullptr || n_seq <= 0 || n_prompt <= 0 ||
      n_predict <= 0) {
    SetErr("nh_generate_batch: bad argument");
    return NH_E_ARG;
  }
  std::vector<std::vector<int32_t>> p(n_seq);
  for (int b = 0; b < n_seq; ++b)
    p[b].assign(prompts + static_cast<size_t>(b) * n_prompt, prompts + static_cast<size_t>(b + 1) * n_prompt);
  BatchOptions o;
  o.use_graph = use_graph != 0;
  o.ep = static_cast<const ExpertGroup*>(ep);
  const auto ids = GreedyGenerateCachedBatch(*static_cast<const OlmoeModel*>(model), p, n_predict, norm_topk != 0, &o);
  if (o.status != NH_OK) {
    SetErr("nh_generate_batch: failed with code " + std::to_string(o.status));
    return o.status;
  }
  for (int b = 0; b < n_seq; ++b)
    std::memcpy(out_tokens + static_cast<size_t>(b) * n_predict, ids[b].data(), static_cast<size_t>(n_predict) * 4);
  if (prefill_ms != nullptr) *prefill_ms = o.prefill_ms;
  if (decode_ms != nullptr) *decode_ms = o.decode_ms;
  return NH_OK;
}

int nh_generate_batch(void* model, const int32_t* prompts, int n_seq, int n_prompt, int n_predict, int norm_topk,
                      int use_graph, int32_t* out_tokens, double* decode_ms) {
  return nh_generate_batch_timed(model, nullptr, prompts, n_seq, n_prompt, n_predict, norm_topk, use_graph,
                                 out_tokens, nullptr, decode_ms);
}

void* nh_model_load_expert_shard(const char* path, uint32_t first, uint32_t count) {
  if (path == nullptr) {
    SetErr("nh_model_load_expert_shard: null path");
    return nullptr;
  }
  auto m = OlmoeModel::LoadExpertShard(path, first, count);
  if (m == nullptr) SetErr(std::string("nh_model_load_expert_shard: failed to load ") + path);
  return m.release();
}

int nh_ep_new_id(uint8_t* id) { return ExpertGroup::NewId(id) ? NH_OK : NH_E_STATE; }

void* nh_ep_create(const uint8_t* id, int world, int rank) {
  auto g = ExpertGroup::Create(id, world, rank);
  if (g == nullptr) SetErr("nh_ep_create: NCCL communicator could not be created");
  return g.release();
}

void nh_ep_free(void* ep) { delete static_cast<ExpertGroup*>(ep); }

int nh_generate_batch_ep(void* model, const void* ep, const int32_t* prompts, int n_seq, int n_prompt, int n_predict,
                         int norm_topk, int use_graph, int32_t* out_tokens, double* decode_ms) {
  if (ep == nullptr) {
    SetErr("nh_generate_batch_ep: null group");
    return NH_E_ARG;
  }
  return nh_generate_batch_timed(model, ep, prompts, n_seq, n_prompt, n_predict, norm_topk, use_graph, out_tokens,
                                 nullptr, decode_ms);
}

int nh_decode_prepare(void* model, const int32_t* prompt, int n_prompt, int n_predict) {
  if (model == nullptr || prompt == nullptr || n_prompt <= 0 || n_predict <= 0) return NH_E_ARG;
  OlmoeModel::Workspace* ws = static_cast<OlmoeModel*>(model)->workspace();
  if (ws == nullptr || !ws->view_ok || !static_cast<OlmoeModel*>(model)->holds_all_experts()) return NH_E_STATE;
  Engine& e = ws->engine;
  int rc = e.Reserve(n_prompt + n_predict + 1, n_prompt, n_predict, false);
  if (rc == NH_OK) rc = e.Begin(prompt, n_prompt, n_predict);
  if (rc == NH_OK) rc = e.RunSteps(ws->view, n_prompt - 1, false, false, false, true);
  if (rc == NH_OK) rc = e.SaveState();
  return rc;
}

int nh_decode_run(void* model, int n_predict) {
  if (model == nullptr || n_predict <= 0) return NH_E_ARG;
  OlmoeModel::Workspace* ws = static_cast<OlmoeModel*>(model)->workspace();
  Engine& e = ws->engine;
  int rc = e.RestoreState();
  if (rc == NH_OK) rc = e.RunSteps(ws->view, n_predict, false, false, false, true);
  return rc;
}

int nh_decode_result(void* model, int n_predict, int32_t* out_tokens) {
  if (model == nullptr || out_tokens == nullptr) return NH_E_ARG;
  std::vector<int32_t> out;
  const int rc = static_cast<OlmoeModel*>(model)->workspace()->engine.Finish(n_predict, &out);
  if (rc == NH_OK) std::memcpy(out_tokens, out.data(), out.size() * 4);
  return rc;
}

void* nh_model_stream(void* model) {
  if (model == nullptr) return nullptr;
  return static_cast<OlmoeModel*>(model)->workspace()->engine.stream();
}

int nh_decode_kernel_loop(void* model, int which, int reps) {
  if (model == nullptr || reps <= 0) return NH_E_ARG;
  OlmoeModel::Workspace* ws = static_cast<OlmoeModel*>(model)->workspace();
  return ws->engine.KernelLoop(ws->view, which, reps);
}

void* nh_stream_model_load(const char* path, int pinned_store) {
  if (path == nullptr) return nullptr;
  auto m = StreamingModel::Load(path, pinned_store != 0);
  if (m == nullptr) SetErr(std::string("StreamingModel::Load failed: ") + path);
  return m.release();
}

void nh_stream_model_free(void* model) { delete static_cast<StreamingModel*>(model); }

int nh_stream_model_config(const void* model, NhConfig* out) {
  if (model == nullptr || out == nullptr) return NH_E_ARG;
  FillConfig(static_cast<const StreamingModel*>(model)->config(), out);
  return NH_OK;
}

int nh_stream_generate(void* model, const int32_t* prompt, int n_prompt, int n_predict, int norm_topk, int capacity,
                       int policy, int pin_slots, const uint64_t* usage, int32_t* out_tokens, int64_t* hits,
                       int64_t* misses, uint64_t* h2d_bytes, int32_t* trace_sel) {
  if (model == nullptr || (n_prompt > 0 && prompt == nullptr)) return NH_E_ARG;
  const StreamingModel& m = *static_cast<StreamingModel*>(model);
  const OlmoeConfig& c = m.config();
  std::vector<int32_t> ids(prompt, prompt + (n_prompt > 0 ? n_prompt : 0));
  StreamingOptions o;
  StreamingStats st;
  o.stats = &st;
  UsageHistogram u;
  if (policy == 1) {
    u = DenseUsage(usage, c.n_layers, c.n_expert);
    o.policy = SlotPolicy::kLearnedPin;
    o.usage = &u;
    o.pin_slots = pin_slots > 0 ? static_cast<uint32_t>(pin_slots) : 0;
  }
  RoutingTrace tr;
  if (trace_sel != nullptr) o.trace = &tr;
  std::vector<int32_t> out = StreamingGenerateEx(m, ids, n_predict, norm_topk != 0, capacity, o);
  if (st.status != NH_OK) {
    SetErr("StreamingGenerate failed");
    return st.status;
  }
  if (out_tokens != nullptr) std::memcpy(out_tokens, out.data(), out.size() * 4);
  for (uint32_t l = 0; l < c.n_layers && l < st.hits.size(); ++l) {
    if (hits != nullptr) hits[l] = st.hits[l];
    if (misses != nullptr) misses[l] = st.misses[l];
  }
  if (h2d_bytes != nullptr) *h2d_bytes = st.h2d_bytes;
  if (trace_sel != nullptr) {
    size_t k = 0;
    for (const RoutingRecord& r : tr.records)
      for (uint32_t e : r.experts) trace_sel[k++] = static_cast<int32_t>(e);
  }
  return NH_OK;
}

int nh_stream_generate_batch_ep(void* model, const void* ep, const int32_t* prompts, int n_seq, int n_prompt,
                                int n_predict, int norm_topk, int capacity, int policy, int pin_slots,
                                const uint64_t* usage, int32_t* out_tokens, int64_t* hits, int64_t* misses,
                                uint64_t* h2d_bytes, int64_t* waves, double* decode_ms) {
  if (model == nullptr || prompts == nullptr || out_tokens == nullptr || n_seq <= 0 || n_prompt <= 0 ||
      n_predict <= 0 || (policy == 1 && usage == nullptr)) {
    SetErr("nh_stream_generate_batch: bad argument");
    return NH_E_ARG;
  }
  const StreamingModel& m = *static_cast<StreamingModel*>(model);
  const OlmoeConfig& c = m.config();
  std::vector<std::vector<int32_t>> p(n_seq);
  for (int b = 0; b < n_seq; ++b)
    p[b].assign(prompts + static_cast<size_t>(b) * n_prompt, prompts + static_cast<size_t>(b + 1) * n_prompt);
  StreamingOptions o;
  StreamingStats st;
  o.stats = &st;
  UsageHistogram u;
  if (policy == 1) {
    u = DenseUsage(usage, c.n_layers, c.n_expert);
    o.policy = SlotPolicy::kLearnedPin;
    o.usage = &u;
    o.pin_slots = pin_slots > 0 ? static_cast<uint32_t>(pin_slots) : 0;
  }
  BatchOptions bo;
  bo.ep = static_cast<const ExpertGroup*>(ep);
  const auto ids = StreamingGenerateBatch(m, p, n_predict, norm_topk != 0, capacity, o, &bo);
  if (st.status != NH_OK) {
    SetErr("StreamingGenerateBatch failed with code " + std::to_string(st.status));
    return st.status;
  }
  for (int b = 0; b < n_seq; ++b)
    std::memcpy(out_tokens + static_cast<size_t>(b) * n_predict, ids[b].data(), static_cast<size_t>(n_predict) * 4);
  for (uint32_t l = 0; l < c.n_layers && l < st.hits.size(); ++l) {
    if (hits != nullptr) hits[l] = st.hits[l];
    if (misses != nullptr) misses[l] = st.misses[l];
  }
  if (h2d_bytes != nullptr) *h2d_bytes = st.h2d_bytes;
  if (waves != nullptr) *waves = st.waves;
  if (decode_ms != nullptr) *decode_ms = bo.decode_ms;
  return NH_OK;
}

int nh_stream_generate_batch(void* model, const int32_t* prompts, int n_seq, int n_prompt, int n_predict,
                             int norm_topk, int capacity, int policy, int pin_slots, const uint64_t* usage,
                             int32_t* out_tokens, int64_t* hits, int64_t* misses, uint64_t* h2d_bytes, int64_t* waves,
                             double* decode_ms) {
  return nh_stream_generate_batch_ep(model, nullptr, prompts, n_seq, n_prompt, n_predict, norm_topk, capacity, policy,
                                     pin_slots, usage, out_tokens, hits, misses, h2d_bytes, waves, decode_ms);
}

int64_t nh_replay(int kind, uint32_t n_layers, uint32_t n_expert, int64_t n_records, const uint32_t* layer,
                  const int64_t* offsets, const uint32_t* experts, uint32_t a, uint32_t b, const uint64_t* usage,
                  int64_t* accesses) {
  const RoutingTrace t = MakeTrace(n_layers, n_expert, n_records, nullptr, layer, offsets, experts);
  ReplayStats s;
  if (kind == 0) {
    LruPolicy p(n_layers, a);
    s = Replay(t, &p);
  } else if (kind == 1) {
    OsPageCachePolicy p(a);
    s = Replay(t, &p);
  } else {
    LearnedPinPolicy p(n_layers, a, b, usage != nullptr ? DenseUsage(usage, n_layers, n_expert) : BuildUsage(t));
    s = Replay(t, &p);
  }
  if (accesses != nullptr) *accesses = static_cast<int64_t>(s.accesses);
  return static_cast<int64_t>(s.hits);
}

int nh_sweep_budgets(uint32_t n_layers, uint32_t n_expert, int64_t n_records, const uint32_t* layer,
                     const int64_t* offsets, const uint32_t* experts, const uint32_t* budgets, int n_budgets,
                     double* out) {
  const RoutingTrace t = MakeTrace(n_layers, n_expert, n_records, nullptr, layer, offsets, experts);
  const auto rows = SweepBudgets(t, std::vector<uint32_t>(budgets, budgets + n_budgets));
  for (size_t i = 0; i < rows.size(); ++i) {
    out[3 * i] = rows[i].learned;
    out[3 * i + 1] = rows[i].lru;
    out[3 * i + 2] = rows[i].os;
  }
  return static_cast<int>(rows.size());
}

int nh_sweep_budgets_calibrated(uint32_t n_layers, uint32_t n_expert, int64_t cal_records, const uint32_t* cal_layer,
                                const int64_t* cal_offsets, const uint32_t* cal_experts, int64_t n_records,
                                const uint32_t* layer, const int64_t* offsets, const uint32_t* experts,
                                const uint32_t* budgets, int n_budgets, double* out) {
  if ((cal_records > 0 && (cal_layer == nullptr || cal_offsets == nullptr)) ||
      (n_records > 0 && (layer == nullptr || offsets == nullptr)) || (n_budgets > 0 && budgets == nullptr) ||
      out == nullptr)
    return NH_E_ARG;
  const RoutingTrace cal = MakeTrace(n_layers, n_expert, cal_records, nullptr, cal_layer, cal_offsets, cal_experts);
  const RoutingTrace t = MakeTrace(n_layers, n_expert, n_records, nullptr, layer, offsets, experts);
  const auto rows = SweepBudgetsCalibrated(cal, t, std::vector<uint32_t>(budgets, budgets + n_budgets));
  for (size_t i = 0; i < rows.size(); ++i) {
    out[3 * i] = rows[i].learned;
    out[3 * i + 1] = rows[i].lru;
    out[3 * i + 2] = rows[i].os;
  }
  return static_cast<int>(rows.size());
}

int nh_sweep_pin_ratio(uint32_t n_layers, uint32_t n_expert, int64_t n_records, const uint32_t* layer,
                       const int64_t* offsets, const uint32_t* experts, uint32_t budget, double* out) {
  const RoutingTrace t = MakeTrace(n_layers, n_expert, n_records, nullptr, layer, offsets, experts);
  const auto rows = SweepPinRatio(t, budget);
  for (size_t i = 0; i < rows.size(); ++i) out[i] = rows[i].learned;
  return static_cast<int>(rows.size());
}

int nh_trace_write(const char* path, uint32_t n_layers, uint32_t n_expert, int64_t n_records, const uint32_t* token,
                   const uint32_t* layer, const int64_t* offsets, const uint32_t* experts) {
  if (path == nullptr) return NH_E_ARG;
  return WriteRoutingTrace(MakeTrace(n_layers, n_expert, n_records, token, layer, offsets, experts), path) ? NH_OK
                                                                                                           : NH_E_IO;
}

int64_t nh_trace_read(const char* path, int text, uint32_t* n_layers, uint32_t* n_expert, int64_t* n_experts_total,
                      int64_t cap_records, int64_t cap_experts, uint32_t* token, uint32_t* layer, int64_t* offsets,
                      uint32_t* experts) {
  if (path == nullptr) return NH_E_ARG;
  RoutingTrace t;
  if (!(text ? ReadRoutingTraceText(path, &t) : ReadRoutingTrace(path, &t))) return NH_E_IO;
  *n_layers = t.n_layers;
  *n_expert = t.n_expert;
  int64_t total = 0;
  for (const auto& r : t.records) total += static_cast<int64_t>(r.experts.size());
  *n_experts_total = total;
  const int64_t n = static_cast<int64_t>(t.records.size());
  if (cap_records >= n && cap_experts >= total) {
    int64_t off = 0;
    for (int64_t i = 0; i < n; ++i) {
      token[i] = t.records[i].token;
      layer[i] = t.records[i].layer;
      offsets[i] = off;
      for (uint32_t e : t.records[i].experts) experts[off++] = e;
    }
    offsets[n] = off;
  }
  return n;
}

void* nh_expert_reader_open(const char* gguf_path) {
  if (gguf_path == nullptr) return nullptr;
  return ExpertReader::Open(gguf_path).release();
}
void nh_expert_reader_free(void* reader) { delete static_cast<ExpertReader*>(reader); }
uint64_t nh_expert_reader_bytes(const void* reader, const char* tensor) {
  return static_cast<const ExpertReader*>(reader)->ExpertBytes(tensor);
}
int nh_expert_reader_read(const void* reader, const char* tensor, int expert, void* out) {
  return static_cast<const ExpertReader*>(reader)->ReadExpert(tensor, expert, out) ? NH_OK : NH_E_IO;
}

void* nh_slot_cache_create(const NhConfig* cfg, int layer, int capacity, void* reader, int policy, int pin_slots,
                           const uint64_t* usage_layer) {
  if (cfg == nullptr || reader == nullptr) return nullptr;
  OlmoeConfig c;
  c.n_layers = cfg->n_layers;
  c.n_embd = cfg->n_embd;
  c.n_ff = cfg->n_ff;
  c.n_expert = cfg->n_expert;
  std::unique_ptr<SlotCacheHandle> h(new SlotCacheHandle());
  SlotCacheOptions o;
  if (policy == 1) {
    o.policy = SlotPolicy::kLearnedPin;
    o.pin_slots = static_cast<uint32_t>(pin_slots);
    h->usage.per_layer.resize(static_cast<size_t>(layer) + 1);
    if (usage_layer != nullptr)
      for (uint32_t e = 0; e < cfg->n_expert; ++e)
        if (usage_layer[e] > 0) h->usage.per_layer[layer][e] = usage_layer[e];
    o.usage = &h->usage;
    o.staging = static_cast<int>(cfg->n_expert_used > 0 ? cfg->n_expert_used : cfg->n_expert);
  }
  cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking);
  o.copy_stream = h->stream;
  h->cache = ExpertSlotCache::Create(c, layer, capacity, static_cast<ExpertReader*>(reader), nullptr, o);
  if (h->cache == nullptr) {
    cudaStreamDestroy(h->stream);
    return nullptr;
  }
  return h.release();
}

void nh_slot_cache_free(void* cache) {
  auto* h = static_cast<SlotCacheHandle*>(cache);
  if (h == nullptr) return;
  h->cache.reset();
  if (h->stream != nullptr) cudaStreamDestroy(h->stream);
  delete h;
}

int nh_slot_cache_ensure(void* cache, const int32_t* ids, int n, int32_t* slots) {
  auto* h = static_cast<SlotCacheHandle*>(cache);
  if (h == nullptr || (n > 0 && ids == nullptr)) return NH_E_ARG;
  std::vector<int> v(ids, ids + n);
  auto m = h->cache->Ensure(v);
  if (cudaStreamSynchronize(h->stream) != cudaSuccess || !h->cache->ok()) return NH_E_IO;
  if (h->cache->Commit(h->stream) != NH_OK || cudaStreamSynchronize(h->stream) != cudaSuccess) return NH_E_CUDA;
  if (slots != nullptr)
    for (int i = 0; i < n; ++i) slots[i] = m[ids[i]];
  return NH_OK;
}

int nh_expert_reader_fail_after(void* reader, int64_t n) {
  if (reader == nullptr) return NH_E_ARG;
  static_cast<ExpertReader*>(reader)->FailReadsAfter(n);
  return NH_OK;
}

int64_t nh_slot_cache_hits(const void* cache) { return static_cast<const SlotCacheHandle*>(cache)->cache->hits(); }
int64_t nh_slot_cache_misses(const void* cache) {
  return static_cast<const SlotCacheHandle*>(cache)->cache->misses();
}

int nh_slot_cache_read_slot(const void* cache, int which, int slot, void* out, uint64_t bytes) {
  const auto* h = static_cast<const SlotCacheHandle*>(cache);
  if (h == nullptr || out == nullptr || which < 0 || which > 2) return NH_E_ARG;
  const DTensor* t = which == 0 ? h->cache->gate_slots() : which == 1 ? h->cache->up_slots() : h->cache->down_slots();
  if (slot < 0 || slot >= t->ne[2] || bytes > t->nb[2]) return NH_E_ARG;
  return cudaMemcpy(out, static_cast<const uint8_t*>(t->data) + t->nb[2] * slot, bytes, cudaMemcpyDeviceToHost) ==
                 cudaSuccess
             ? NH_OK
             : NH_E_CUDA;
}

int nh_plan_waves(const int32_t* sel, int n_picks, int n_expert, int e_lo, int e_hi, int per, const uint8_t* pinned,
                  int32_t* wave_of, int32_t* wave_size, int32_t* wave_experts) {
  if (n_expert <= 0 || pinned == nullptr || wave_of == nullptr || wave_size == nullptr || wave_experts == nullptr)
    return NH_E_ARG;
  std::vector<char> pin(pinned, pinned + n_expert);
  std::vector<std::vector<int>> waves;
  std::vector<int> of;
  const int n = PlanWaves(sel, n_picks, n_expert, e_lo, e_hi, per, pin, &waves, &of);
  if (n < 0) return n;
  size_t k = 0;
  for (int w = 0; w < n; ++w) {
    wave_size[w] = static_cast<int32_t>(waves[w].size());
    for (int e : waves[w]) wave_experts[k++] = e;
  }
  for (int e = 0; e < n_expert; ++e) wave_of[e] = of[e];
  return n;
}

int nh_group_wave_pairs(const int32_t* sel, int n_picks, int k, int n_expert, const int32_t* wave_of, int w,
                        const int32_t* slot_of, int slots, int32_t* off, int32_t* cnt, int32_t* act, int32_t* out) {
  if (n_expert <= 0 || wave_of == nullptr || slot_of == nullptr) return NH_E_ARG;
  return GroupWavePairs(sel, n_picks, k, std::vector<int>(wave_of, wave_of + n_expert), w,
                        std::vector<int>(slot_of, slot_of + n_expert), slots, off, cnt, act, out);
}

void* nh_tokenizer_load(const char* path) {
  if (path == nullptr) return nullptr;
  auto t = Tokenizer::Load(path);
  if (t == nullptr) SetErr(std::string("nh_tokenizer_load: no vocabulary in ") + path);
  return t.release();
}

void* nh_tokenizer_from_lists(const char* const* vocab, int64_t n_vocab, const char* const* merges,
                              int64_t n_merges) {
  if ((vocab == nullptr && n_vocab > 0) || (merges == nullptr && n_merges > 0) || n_vocab < 0 || n_merges < 0)
    return nullptr;
  for (int64_t i = 0; i < n_vocab; ++i)
    if (vocab[i] == nullptr) return nullptr;
  for (int64_t i = 0; i < n_merges; ++i)
    if (merges[i] == nullptr) return nullptr;
  std::vector<std::string> v(vocab, vocab + n_vocab), m(merges, merges + n_merges);
  return Tokenizer::FromLists(std::move(v), std::move(m)).release();
}

void nh_tokenizer_free(void* tok) { delete static_cast<Tokenizer*>(tok); }

int64_t nh_tokenizer_vocab_size(const void* tok) {
  return tok != nullptr ? static_cast<const Tokenizer*>(tok)->vocab_size() : NH_E_ARG;
}

int64_t nh_tokenizer_encode(const void* tok, const char* text, int64_t len, int32_t* ids, int64_t cap) {
  if (tok == nullptr || (text == nullptr && len > 0) || len < 0 || (ids == nullptr && cap > 0)) return NH_E_ARG;
  const auto v = static_cast<const Tokenizer*>(tok)->Encode(std::string(text != nullptr ? text : "", len));
  const int64_t n = static_cast<int64_t>(v.size());
  if (n > 0 && cap > 0) std::memcpy(ids, v.data(), static_cast<size_t>(std::min(n, cap)) * 4);
  return n;
}

int64_t nh_tokenizer_decode(const void* tok, const int32_t* ids, int64_t n, char* out, int64_t cap) {
  if (tok == nullptr || (ids == nullptr && n > 0) || n < 0 || (out == nullptr && cap > 0)) return NH_E_ARG;
  const std::string s = static_cast<const Tokenizer*>(tok)->Decode(std::vector<int32_t>(ids, ids + n));
  const int64_t len = static_cast<int64_t>(s.size());
  if (len > 0 && cap > 0) std::memcpy(out, s.data(), static_cast<size_t>(std::min(len, cap)));
  return len;
}

int64_t nh_tokenizer_token(const void* tok, int32_t id, char* out, int64_t cap) {
  if (tok == nullptr || (out == nullptr && cap > 0)) return NH_E_ARG;
  const std::string& s = static_cast<const Tokenizer*>(tok)->token(id);
  const int64_t len = static_cast<int64_t>(s.size());
  if (len > 0 && cap > 0) std::memcpy(out, s.data(), static_cast<size_t>(std::min(len, cap)));
  return len;
}

int64_t nh_tokenizer_split(const char* text, int64_t len, int64_t* bounds, int64_t cap) {
  if ((text == nullptr && len > 0) || len < 0 || (bounds == nullptr && cap > 0)) return NH_E_ARG;
  const auto ch = Tokenizer::Split(std::string(text != nullptr ? text : "", len));
  const int64_t n = static_cast<int64_t>(ch.size());
  for (int64_t i = 0; i < n && i < cap; ++i) {
    bounds[2 * i] = static_cast<int64_t>(ch[i].first);
    bounds[2 * i + 1] = static_cast<int64_t>(ch[i].second);
  }
  return n;
}

}  // extern "C"

// Resident greedy generation (reference: src/model/generate.cc:10-181).
#include "nuthatch/generate.h"

#include <cuda_runtime.h>

#include "workspace.h"

namespace nuthatch {

namespace {

// The batched prompt prefill is on unless NH_PREFILL=0 (read once).
bool PrefillEnabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("NH_PREFILL");
    v = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return v != 0;
}

}  // namespace

std::vector<int32_t> GreedyGenerateCachedEx(const OlmoeModel& model, const std::vector<int32_t>& ids,
                                            int n_predict, bool norm_topk, GenerateOptions* opt) {
  GenerateOptions local;
  GenerateOptions& o = opt != nullptr ? *opt : local;
  o.status = NH_OK;
  std::vector<int32_t> out;
  if (ids.empty() || n_predict <= 0) return out;
  OlmoeModel::Workspace* ws = model.workspace();
  if (ws == nullptr || !ws->view_ok || !model.holds_all_experts()) {
    o.status = NH_E_STATE;
    return out;
  }
  const OlmoeConfig& c = model.config();
  for (int32_t t : ids) {
    if (t < 0 || static_cast<uint32_t>(t) >= c.n_vocab) {
      o.status = NH_E_ARG;
      return out;
    }
  }
  Engine& e = ws->engine;
  const int P = static_cast<int>(ids.size());
  const bool dumps = o.hidden != nullptr || o.logits != nullptr;
  const bool trace = o.trace != nullptr || o.trace_gap != nullptr;
  int rc = e.Reserve(P + n_predict + 1, P, n_predict, dumps);
  // The prompt is forwarded at once, as the reference's first step does
  // (generate.cc:63-91): positions 0..P-2 through the batched prefill, then
  // the last prompt position as the first batch-1 step.  Models outside the
  // batched kernels' shapes (and NH_PREFILL=0) take the prompt one position
  // per step; the ids are the same either way.
  const int start = P > 1 && PrefillEnabled() && Engine::PrefillSupported(ws->view) ? P - 1 : 0;
  if (rc == NH_OK) rc = e.Begin(ids.data(), P, n_predict, start);
  cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
  if (o.timed)
    for (cudaEvent_t& x : ev) cudaEventCreate(&x);
  if (o.timed) cudaEventRecord(ev[0], e.stream());
  if (rc == NH_OK && start > 0) rc = e.Prefill(ws->view, start, norm_topk, trace);
  if (o.timed) cudaEventRecord(ev[1], e.stream());
  const int steps = P + n_predict - 1;
  if (rc == NH_OK) rc = e.RunSteps(ws->view, steps - start, norm_topk, trace, dumps, o.use_graph);
  if (o.timed) {
    cudaEventRecord(ev[2], e.stream());
    float a = 0.f, b = 0.f;
    if (cudaEventSynchronize(ev[2]) == cudaSuccess && cudaEventElapsedTime(&a, ev[0], ev[1]) == cudaSuccess &&
        cudaEventElapsedTime(&b, ev[1], ev[2]) == cudaSuccess) {
      o.prefill_ms = a;
      o.decode_ms = b;
    }
    for (cudaEvent_t x : ev) cudaEventDestroy(x);
  }
  if (rc == NH_OK) rc = e.Finish(n_predict, &out);
  if (rc != NH_OK) {
    o.status = rc;
    cudaStreamSynchronize(e.stream());
    out.clear();
    return out;
  }
  const int64_t L = c.n_layers, K = c.n_expert_used, d = c.n_embd, V = c.n_vocab;
  if (trace) {
    std::vector<int32_t> sel(static_cast<size_t>(steps) * L * K);
    std::vector<float> gap(static_cast<size_t>(steps) * L);
    cudaMemcpy(sel.data(), e.trace_sel_dev(), sel.size() * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(gap.data(), e.trace_gap_dev(), gap.size() * 4, cudaMemcpyDeviceToHost);
    if (o.trace != nullptr) {
      // Token-major records of every processed token (generate.cc:154-166).
      o.trace->n_layers = c.n_layers;
      o.trace->n_expert = c.n_expert;
      o.trace->records.clear();
      for (int t = 0; t < steps; ++t) {
        for (int64_t l = 0; l < L; ++l) {
          RoutingRecord r;
          r.token = static_cast<uint32_t>(t);
          r.layer = static_cast<uint32_t>(l);
          for (int64_t i = 0; i < K; ++i) r.experts.push_back(static_cast<uint32_t>(sel[(t * L + l) * K + i]));
          o.trace->records.push_back(std::move(r));
        }
      }
    }
    if (o.trace_gap != nullptr) *o.trace_gap = gap;
  }
  if (o.hidden != nullptr) {
    o.hidden->resize(static_cast<size_t>(n_predict) * L * d);
    cudaMemcpy(o.hidden->data(), e.dump_hidden_dev(), o.hidden->size() * 4, cudaMemcpyDeviceToHost);
  }
  if (o.logits != nullptr) {
    o.logits->resize(static_cast<size_t>(n_predict) * V);
    cudaMemcpy(o.logits->data(), e.dump_logits_dev(), o.logits->size() * 4, cudaMemcpyDeviceToHost);
  }
  return out;
}

std::vector<int32_t> GreedyGenerateCached(const OlmoeModel& model, std::vector<int32_t> ids, int n_predict,
                                          bool norm_topk) {
  return GreedyGenerateCachedEx(model, ids, n_predict, norm_topk, nullptr);
}

std::vector<int32_t> GreedyGenerateCachedTrace(const OlmoeModel& model, std::vector<int32_t> ids, int n_predict,
                                               bool norm_topk, RoutingTrace* trace) {
  GenerateOptions o;
  o.trace = trace;
  return GreedyGenerateCachedEx(model, ids, n_predict, norm_topk, &o);
}

std::vector<int32_t> GreedyGenerate(const OlmoeModel& model, std::vector<int32_t> ids, int n_predict,
                                    bool norm_topk) {
  // Every step recomputes the whole sequence from an empty cache and keeps
  // only the argmax of the last position.
  std::vector<int32_t> out;
  if (ids.empty() || n_predict <= 0) return out;
  for (int step = 0; step < n_predict; ++step) {
    std::vector<int32_t> one = GreedyGenerateCachedEx(model, ids, 1, norm_topk, nullptr);
    if (one.size() != 1) return {};
    out.push_back(one[0]);
    ids.push_back(one[0]);
  }
  return out;
}

}  // namespace nuthatch

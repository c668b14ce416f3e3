// ORACLE — test infrastructure only (checker, never product).
//
// C ABI over the reference's own, unmodified src/cache, src/trace and src/io
// sources, compiled from the reference tree into oracle/_ref by
// oracle/Makefile.  Used to pin the oracle's and the product's cache-policy,
// trace-format and positioned-read behaviour to the reference's compiled code.
#include <cstdint>
#include <string>
#include <vector>

#include "src/cache/cache_policy.h"
#include "src/cache/learned_pin_policy.h"
#include "src/cache/lru_policy.h"
#include "src/cache/os_page_cache_policy.h"
#include "src/cache/trace_sweep.h"
#include "src/io/tensor_source.h"
#include "src/trace/routing_trace.h"

namespace {

nuthatch::RoutingTrace MakeTrace(uint32_t n_layers, uint32_t n_expert, int64_t n_records,
                                 const uint32_t* token, const uint32_t* layer,
                                 const int64_t* offsets, const uint32_t* experts) {
  nuthatch::RoutingTrace t;
  t.n_layers = n_layers;
  t.n_expert = n_expert;
  t.records.reserve(n_records);
  for (int64_t r = 0; r < n_records; ++r) {
    nuthatch::RoutingRecord rec;
    rec.token = token != nullptr ? token[r] : static_cast<uint32_t>(r);
    rec.layer = layer[r];
    rec.experts.assign(experts + offsets[r], experts + offsets[r + 1]);
    t.records.push_back(std::move(rec));
  }
  return t;
}

}  // namespace

extern "C" {

// kind 0: LruPolicy(n_layers, a); 1: OsPageCachePolicy(a); 2: LearnedPinPolicy
// (n_layers, pin=a, lru=b, BuildUsage(trace)).  Returns hits, *accesses set.
int64_t ref_replay(int kind, uint32_t n_layers, uint32_t n_expert, int64_t n_records,
                   const uint32_t* layer, const int64_t* offsets, const uint32_t* experts,
                   uint32_t a, uint32_t b, int64_t* accesses) {
  const nuthatch::RoutingTrace t =
      MakeTrace(n_layers, n_expert, n_records, nullptr, layer, offsets, experts);
  nuthatch::ReplayStats s;
  if (kind == 0) {
    nuthatch::LruPolicy p(n_layers, a);
    s = nuthatch::Replay(t, &p);
  } else if (kind == 1) {
    nuthatch::OsPageCachePolicy p(a);
    s = nuthatch::Replay(t, &p);
  } else {
    nuthatch::LearnedPinPolicy p(n_layers, a, b, nuthatch::BuildUsage(t));
    s = nuthatch::Replay(t, &p);
  }
  *accesses = static_cast<int64_t>(s.accesses);
  return static_cast<int64_t>(s.hits);
}

// LearnedPinPolicy(n_layers, pin, lru, usage) with the usage histogram given
// as dense counts usage[n_layers][n_expert] (a calibration run's, not the
// replayed trace's).  Returns hits, *accesses set.
int64_t ref_replay_pin_usage(uint32_t n_layers, uint32_t n_expert, int64_t n_records, const uint32_t* layer,
                             const int64_t* offsets, const uint32_t* experts, uint32_t pin, uint32_t lru,
                             const uint64_t* usage, int64_t* accesses) {
  const nuthatch::RoutingTrace t =
      MakeTrace(n_layers, n_expert, n_records, nullptr, layer, offsets, experts);
  nuthatch::UsageHistogram u;
  u.per_layer.resize(n_layers);
  for (uint32_t l = 0; l < n_layers; ++l)
    for (uint32_t e = 0; e < n_expert; ++e)
      if (usage[static_cast<size_t>(l) * n_expert + e] != 0) u.per_layer[l][e] = usage[static_cast<size_t>(l) * n_expert + e];
  nuthatch::LearnedPinPolicy p(n_layers, pin, lru, u);
  const nuthatch::ReplayStats s = nuthatch::Replay(t, &p);
  *accesses = static_cast<int64_t>(s.accesses);
  return static_cast<int64_t>(s.hits);
}

// SweepBudgets: out rows of (learned, lru, os) hit rates, one per budget.
int ref_sweep_budgets(uint32_t n_layers, uint32_t n_expert, int64_t n_records,
                      const uint32_t* layer, const int64_t* offsets, const uint32_t* experts,
                      const uint32_t* budgets, int n_budgets, double* out) {
  const nuthatch::RoutingTrace t =
      MakeTrace(n_layers, n_expert, n_records, nullptr, layer, offsets, experts);
  std::vector<uint32_t> b(budgets, budgets + n_budgets);
  const auto rows = nuthatch::SweepBudgets(t, b);
  for (size_t i = 0; i < rows.size(); ++i) {
    out[3 * i + 0] = rows[i].learned;
    out[3 * i + 1] = rows[i].lru;
    out[3 * i + 2] = rows[i].os;
  }
  return static_cast<int>(rows.size());
}

int ref_sweep_pin_ratio(uint32_t n_layers, uint32_t n_expert, int64_t n_records,
                        const uint32_t* layer, const int64_t* offsets, const uint32_t* experts,
                        uint32_t budget, double* out) {
  const nuthatch::RoutingTrace t =
      MakeTrace(n_layers, n_expert, n_records, nullptr, layer, offsets, experts);
  const auto rows = nuthatch::SweepPinRatio(t, budget);
  for (size_t i = 0; i < rows.size(); ++i) out[i] = rows[i].learned;
  return static_cast<int>(rows.size());
}

int ref_write_trace(const char* path, uint32_t n_layers, uint32_t n_expert, int64_t n_records,
                    const uint32_t* token, const uint32_t* layer, const int64_t* offsets,
                    const uint32_t* experts) {
  const nuthatch::RoutingTrace t =
      MakeTrace(n_layers, n_expert, n_records, token, layer, offsets, experts);
  return nuthatch::WriteRoutingTrace(t, path) ? 0 : -1;
}

// Reads a binary (text=0) or text (text=1) trace.  First call with cap=0 to
// learn the sizes: returns record count; *n_experts_total gets the flat size.
int64_t ref_read_trace(const char* path, int text, uint32_t* n_layers, uint32_t* n_expert,
                       int64_t* n_experts_total, int64_t cap_records, int64_t cap_experts,
                       uint32_t* token, uint32_t* layer, int64_t* offsets, uint32_t* experts) {
  nuthatch::RoutingTrace t;
  const bool ok = text ? nuthatch::ReadRoutingTraceText(path, &t)
                       : nuthatch::ReadRoutingTrace(path, &t);
  if (!ok) return -1;
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

// TensorSource::ReadAt through the reference's own POSIX pread loop.
int ref_read_at(const char* path, uint64_t offset, uint64_t size, void* out) {
  auto src = nuthatch::TensorSource::Open(path);
  if (src == nullptr) return -1;
  return src->ReadAt(offset, size, out) ? 0 : -2;
}

}  // extern "C"

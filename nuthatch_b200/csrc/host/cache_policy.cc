// Expert cache policies, trace replay and the budget sweeps.  Behaviour
// follows the reference's src/cache (cache_policy.cc:5-18, lru_policy.cc:5-30,
// os_page_cache_policy.cc:5-25, learned_pin_policy.cc:8-59,
// trace_sweep.cc:10-50); the structure here is one recency primitive
// (RecencySet) that all three policies compose.
#include <algorithm>

#include "nuthatch/cache_policy.h"

namespace nuthatch {

bool RecencySet::Touch(uint64_t key) {
  const uint64_t now = ++clock_;
  auto found = stamp_of_.find(key);
  if (found != stamp_of_.end()) {
    // Present: move its index entry from the old stamp to the new one.
    by_stamp_.erase(found->second);
    by_stamp_.emplace(now, key);
    found->second = now;
    return true;
  }
  if (capacity_ == 0) return false;
  stamp_of_.emplace(key, now);
  by_stamp_.emplace(now, key);
  if (stamp_of_.size() > capacity_) {
    // The new key holds the largest stamp, so the victim is always another.
    const auto oldest = by_stamp_.begin();
    stamp_of_.erase(oldest->second);
    by_stamp_.erase(oldest);
  }
  return false;
}

ReplayStats Replay(const RoutingTrace& trace, CachePolicy* policy) {
  ReplayStats stats;
  for (const RoutingRecord& rec : trace.records) {
    stats.accesses += rec.experts.size();
    for (uint32_t e : rec.experts) stats.hits += policy->Access(rec.layer, e) ? 1 : 0;
  }
  stats.misses = stats.accesses - stats.hits;
  return stats;
}

LruPolicy::LruPolicy(uint32_t n_layers, uint32_t slots_per_layer)
    : per_layer_(n_layers, RecencySet(slots_per_layer)) {}

bool LruPolicy::Access(uint32_t layer, uint32_t expert) {
  return layer < per_layer_.size() && per_layer_[layer].Touch(expert);
}

OsPageCachePolicy::OsPageCachePolicy(uint64_t capacity) : resident_(capacity) {}

bool OsPageCachePolicy::Access(uint32_t layer, uint32_t expert) {
  return resident_.Touch((static_cast<uint64_t>(layer) << 32) | expert);
}

UsageHistogram BuildUsage(const RoutingTrace& trace) {
  UsageHistogram usage;
  usage.per_layer.resize(trace.n_layers);
  for (const RoutingRecord& rec : trace.records) {
    if (rec.layer < trace.n_layers) {
      auto& counts = usage.per_layer[rec.layer];
      for (uint32_t e : rec.experts) counts[e] += 1;
    }
  }
  return usage;
}

std::vector<uint32_t> PinnedExperts(const UsageHistogram& usage, uint32_t layer, uint32_t pin_slots) {
  if (layer >= usage.per_layer.size() || pin_slots == 0) return {};
  // Rank by (count descending, id ascending): a strict total order, so the
  // chosen set does not depend on the hash map's iteration order.
  struct Ranked {
    uint64_t count;
    uint32_t id;
  };
  std::vector<Ranked> all;
  all.reserve(usage.per_layer[layer].size());
  for (const auto& kv : usage.per_layer[layer]) all.push_back({kv.second, kv.first});
  const auto before = [](const Ranked& a, const Ranked& b) {
    return a.count > b.count || (a.count == b.count && a.id < b.id);
  };
  const size_t take = std::min<size_t>(pin_slots, all.size());
  std::nth_element(all.begin(), all.begin() + take - (take > 0 ? 1 : 0), all.end(), before);
  std::sort(all.begin(), all.begin() + take, before);
  std::vector<uint32_t> ids(take);
  for (size_t i = 0; i < take; ++i) ids[i] = all[i].id;
  return ids;
}

LearnedPinPolicy::LearnedPinPolicy(uint32_t n_layers, uint32_t pin_slots, uint32_t lru_slots,
                                   const UsageHistogram& usage)
    : pinned_(n_layers), rest_(n_layers, RecencySet(lru_slots)) {
  for (uint32_t l = 0; l < n_layers; ++l) {
    pinned_[l] = PinnedExperts(usage, l, pin_slots);
    std::sort(pinned_[l].begin(), pinned_[l].end());
  }
}

bool LearnedPinPolicy::Access(uint32_t layer, uint32_t expert) {
  if (layer >= pinned_.size()) return false;
  const std::vector<uint32_t>& pins = pinned_[layer];
  if (std::binary_search(pins.begin(), pins.end(), expert)) return true;
  return rest_[layer].Touch(expert);
}

std::vector<SweepRow> SweepBudgets(const RoutingTrace& trace, const std::vector<uint32_t>& budgets) {
  return SweepBudgetsCalibrated(trace, trace, budgets);
}

std::vector<SweepRow> SweepBudgetsCalibrated(const RoutingTrace& calibration, const RoutingTrace& trace,
                                             const std::vector<uint32_t>& budgets) {
  UsageHistogram usage = BuildUsage(calibration);
  usage.per_layer.resize(std::max<size_t>(usage.per_layer.size(), trace.n_layers));
  const auto rate = [&trace](CachePolicy&& p) { return Replay(trace, &p).hit_rate(); };
  std::vector<SweepRow> rows;
  for (uint32_t budget : budgets) {
    if (budget == 0) continue;
    const uint32_t pin = LearnedPinSlots(budget);
    SweepRow row;
    row.budget = budget;
    row.learned = rate(LearnedPinPolicy(trace.n_layers, pin, budget - std::min(pin, budget), usage));
    row.lru = rate(LruPolicy(trace.n_layers, budget));
    row.os = rate(OsPageCachePolicy(static_cast<uint64_t>(budget) * trace.n_layers));
    rows.push_back(row);
  }
  return rows;
}

std::vector<PinRatioRow> SweepPinRatio(const RoutingTrace& trace, uint32_t budget) {
  const UsageHistogram usage = BuildUsage(trace);
  std::vector<PinRatioRow> rows(static_cast<size_t>(budget) + 1);
  for (uint32_t pin = 0; pin <= budget; ++pin) {
    LearnedPinPolicy p(trace.n_layers, pin, budget - pin, usage);
    rows[pin] = {pin, budget - pin, Replay(trace, &p).hit_rate()};
  }
  return rows;
}

}  // namespace nuthatch

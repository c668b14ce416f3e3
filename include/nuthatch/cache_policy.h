// Expert cache policies and trace replay (reference: src/cache/cache_policy.h,
// lru_policy.h, learned_pin_policy.h, os_page_cache_policy.h, trace_sweep.h).
//
// Learned pin picks, per layer, the `pin_slots` experts with the highest
// usage count; equal counts go to the lower expert id (the reference orders
// equal counts by unordered_map iteration order, which depends on the
// standard library).
#ifndef NUTHATCH_B200_CACHE_POLICY_H_
#define NUTHATCH_B200_CACHE_POLICY_H_

#include <cstdint>
#include <map>
#include <unordered_map>
#include <vector>

#include "nuthatch/routing_trace.h"

namespace nuthatch {

struct ReplayStats {
  uint64_t accesses = 0;
  uint64_t hits = 0;
  uint64_t misses = 0;
  double hit_rate() const { return accesses ? static_cast<double>(hits) / accesses : 0.0; }
};

class CachePolicy {
 public:
  virtual ~CachePolicy() = default;
  // true = hit (resident), false = miss; updates the policy state.
  virtual bool Access(uint32_t layer, uint32_t expert) = 0;
};

// Replays every access of the trace, in record order (cache_policy.cc:5-18).
ReplayStats Replay(const RoutingTrace& trace, CachePolicy* policy);

// The building block of every policy below: a set of at most `capacity` keys
// ordered by last use.  Touch(key) reports whether the key was present and
// makes it the most recent; a key that is not present is inserted, and when
// that overfills the set the key touched longest ago leaves.  Each touch
// stamps the key with the next value of a use clock; `by_stamp_` indexes the
// keys by stamp, so the oldest is its first entry.  Capacity 0 holds nothing.
class RecencySet {
 public:
  explicit RecencySet(uint64_t capacity = 0) : capacity_(capacity) {}
  bool Touch(uint64_t key);
  uint64_t size() const { return stamp_of_.size(); }

 private:
  uint64_t capacity_;
  uint64_t clock_ = 0;
  std::unordered_map<uint64_t, uint64_t> stamp_of_;  // key -> stamp of its last use
  std::map<uint64_t, uint64_t> by_stamp_;            // stamp -> key
};

// Per-layer LRU of slots_per_layer experts (lru_policy.cc:5-30).
class LruPolicy : public CachePolicy {
 public:
  LruPolicy(uint32_t n_layers, uint32_t slots_per_layer);
  bool Access(uint32_t layer, uint32_t expert) override;

 private:
  std::vector<RecencySet> per_layer_;
};

// One global LRU over (layer, expert) of `capacity` entries: the OS page
// cache model (os_page_cache_policy.cc:5-25).
class OsPageCachePolicy : public CachePolicy {
 public:
  explicit OsPageCachePolicy(uint64_t capacity);
  bool Access(uint32_t layer, uint32_t expert) override;

 private:
  RecencySet resident_;  // keys (layer << 32) | expert
};

// Per-layer usage counts (learned_pin_policy.h:14-17).
struct UsageHistogram {
  std::vector<std::unordered_map<uint32_t, uint64_t>> per_layer;
};
UsageHistogram BuildUsage(const RoutingTrace& trace);

// The experts pinned in one layer: top `pin_slots` by count, ties to the lower id.
std::vector<uint32_t> PinnedExperts(const UsageHistogram& usage, uint32_t layer, uint32_t pin_slots);

// Pinned experts always hit; the rest go through a per-layer LRU of
// lru_slots (learned_pin_policy.cc:19-59).
class LearnedPinPolicy : public CachePolicy {
 public:
  LearnedPinPolicy(uint32_t n_layers, uint32_t pin_slots, uint32_t lru_slots,
                   const UsageHistogram& usage);
  bool Access(uint32_t layer, uint32_t expert) override;

 private:
  std::vector<std::vector<uint32_t>> pinned_;  // per layer, sorted ascending
  std::vector<RecencySet> rest_;               // per layer, lru_slots each
};

// Budget and pin-ratio sweeps (trace_sweep.cc:10-50): learned uses
// pin = ceil(3*budget/4) (1 when budget is 1), lru = budget - pin; OS
// capacity = budget * n_layers; budget 0 is skipped.
struct SweepRow {
  uint32_t budget;
  double learned;
  double lru;
  double os;
};
std::vector<SweepRow> SweepBudgets(const RoutingTrace& trace, const std::vector<uint32_t>& budgets);

// The out-of-sample form of SweepBudgets (no reference counterpart; the
// cross-input evaluation the reference's analysis calls for): learned pin
// takes its usage histogram from `calibration` (e.g. a routing trace written
// by an earlier run with WriteRoutingTrace and read back), and every policy
// replays `eval`.  With calibration == eval it equals SweepBudgets.
std::vector<SweepRow> SweepBudgetsCalibrated(const RoutingTrace& calibration, const RoutingTrace& eval,
                                             const std::vector<uint32_t>& budgets);

struct PinRatioRow {
  uint32_t pin;
  uint32_t lru;
  double learned;
};
std::vector<PinRatioRow> SweepPinRatio(const RoutingTrace& trace, uint32_t budget);

// pin share used by the sweeps and by the learned-pin slot cache.
inline uint32_t LearnedPinSlots(uint32_t budget) {
  return budget > 1 ? (budget * 3 + 3) / 4 : budget;
}

}  // namespace nuthatch

#endif  // NUTHATCH_B200_CACHE_POLICY_H_

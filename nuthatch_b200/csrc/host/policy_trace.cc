// Cache policies, replay and sweeps (reference: src/cache/*.cc) and the
// routing trace formats (reference: src/trace/routing_trace.cc).
#include <algorithm>
#include <cstring>
#include <fstream>
#include <sstream>

#include "nuthatch/cache_policy.h"
#include "nuthatch/routing_trace.h"

namespace nuthatch {

ReplayStats Replay(const RoutingTrace& trace, CachePolicy* policy) {
  ReplayStats s;
  for (const RoutingRecord& rec : trace.records) {
    for (uint32_t e : rec.experts) {
      ++s.accesses;
      if (policy->Access(rec.layer, e)) ++s.hits;
      else ++s.misses;
    }
  }
  return s;
}

LruPolicy::LruPolicy(uint32_t n_layers, uint32_t slots_per_layer) : slots_(slots_per_layer), layers_(n_layers) {}

bool LruPolicy::Access(uint32_t layer, uint32_t expert) {
  if (layer >= layers_.size()) return false;
  Layer& L = layers_[layer];
  auto it = L.pos.find(expert);
  if (it != L.pos.end()) {
    L.order.splice(L.order.begin(), L.order, it->second);
    return true;
  }
  if (slots_ == 0) return false;
  L.order.push_front(expert);
  L.pos[expert] = L.order.begin();
  if (L.order.size() > slots_) {
    L.pos.erase(L.order.back());
    L.order.pop_back();
  }
  return false;
}

OsPageCachePolicy::OsPageCachePolicy(uint64_t capacity) : cap_(capacity) {}

bool OsPageCachePolicy::Access(uint32_t layer, uint32_t expert) {
  const uint64_t k = (static_cast<uint64_t>(layer) << 32) | expert;
  auto it = pos_.find(k);
  if (it != pos_.end()) {
    order_.splice(order_.begin(), order_, it->second);
    return true;
  }
  if (cap_ == 0) return false;
  order_.push_front(k);
  pos_[k] = order_.begin();
  if (order_.size() > cap_) {
    pos_.erase(order_.back());
    order_.pop_back();
  }
  return false;
}

UsageHistogram BuildUsage(const RoutingTrace& trace) {
  UsageHistogram u;
  u.per_layer.resize(trace.n_layers);
  for (const RoutingRecord& rec : trace.records) {
    if (rec.layer >= trace.n_layers) continue;
    for (uint32_t e : rec.experts) ++u.per_layer[rec.layer][e];
  }
  return u;
}

std::vector<uint32_t> PinnedExperts(const UsageHistogram& usage, uint32_t layer, uint32_t pin_slots) {
  std::vector<uint32_t> out;
  if (layer >= usage.per_layer.size()) return out;
  std::vector<std::pair<uint32_t, uint64_t>> v(usage.per_layer[layer].begin(), usage.per_layer[layer].end());
  std::sort(v.begin(), v.end(), [](const auto& a, const auto& b) {
    return a.second != b.second ? a.second > b.second : a.first < b.first;
  });
  for (size_t i = 0; i < std::min<size_t>(pin_slots, v.size()); ++i) out.push_back(v[i].first);
  return out;
}

LearnedPinPolicy::LearnedPinPolicy(uint32_t n_layers, uint32_t pin_slots, uint32_t lru_slots,
                                   const UsageHistogram& usage)
    : lru_slots_(lru_slots), layers_(n_layers) {
  for (uint32_t l = 0; l < n_layers; ++l) {
    for (uint32_t e : PinnedExperts(usage, l, pin_slots)) layers_[l].pinned.insert(e);
  }
}

bool LearnedPinPolicy::Access(uint32_t layer, uint32_t expert) {
  if (layer >= layers_.size()) return false;
  Layer& L = layers_[layer];
  if (L.pinned.count(expert)) return true;
  auto it = L.pos.find(expert);
  if (it != L.pos.end()) {
    L.order.splice(L.order.begin(), L.order, it->second);
    return true;
  }
  if (lru_slots_ == 0) return false;
  L.order.push_front(expert);
  L.pos[expert] = L.order.begin();
  if (L.order.size() > lru_slots_) {
    L.pos.erase(L.order.back());
    L.order.pop_back();
  }
  return false;
}

std::vector<SweepRow> SweepBudgets(const RoutingTrace& trace, const std::vector<uint32_t>& budgets) {
  const UsageHistogram usage = BuildUsage(trace);
  std::vector<SweepRow> rows;
  for (uint32_t b : budgets) {
    if (b == 0) continue;
    const uint32_t pin = LearnedPinSlots(b);
    LearnedPinPolicy learned(trace.n_layers, pin, b > pin ? b - pin : 0, usage);
    LruPolicy lru(trace.n_layers, b);
    OsPageCachePolicy os(static_cast<uint64_t>(b) * trace.n_layers);
    rows.push_back({b, Replay(trace, &learned).hit_rate(), Replay(trace, &lru).hit_rate(),
                    Replay(trace, &os).hit_rate()});
  }
  return rows;
}

std::vector<PinRatioRow> SweepPinRatio(const RoutingTrace& trace, uint32_t budget) {
  const UsageHistogram usage = BuildUsage(trace);
  std::vector<PinRatioRow> rows;
  for (uint32_t pin = 0; pin <= budget; ++pin) {
    LearnedPinPolicy learned(trace.n_layers, pin, budget - pin, usage);
    rows.push_back({pin, budget - pin, Replay(trace, &learned).hit_rate()});
  }
  return rows;
}

// ------------------------------------------------------------------ trace files
namespace {
constexpr char kMagic[8] = {'N', 'U', 'T', 'H', 'T', 'R', 'C', '1'};
constexpr uint32_t kVersion = 1;

template <typename T>
void Put(std::ostream& os, T v) {
  os.write(reinterpret_cast<const char*>(&v), sizeof(v));
}
template <typename T>
bool Get(std::istream& is, T* v) {
  return static_cast<bool>(is.read(reinterpret_cast<char*>(v), sizeof(*v)));
}
}  // namespace

bool WriteRoutingTrace(const RoutingTrace& trace, const std::string& path) {
  std::ofstream os(path, std::ios::binary);
  if (!os) return false;
  os.write(kMagic, sizeof(kMagic));
  Put<uint32_t>(os, kVersion);
  Put<uint32_t>(os, trace.n_layers);
  Put<uint32_t>(os, trace.n_expert);
  Put<uint64_t>(os, trace.records.size());
  for (const RoutingRecord& r : trace.records) {
    Put<uint32_t>(os, r.token);
    Put<uint32_t>(os, r.layer);
    Put<uint32_t>(os, static_cast<uint32_t>(r.experts.size()));
    for (uint32_t e : r.experts) Put<uint32_t>(os, e);
  }
  return static_cast<bool>(os);
}

bool ReadRoutingTrace(const std::string& path, RoutingTrace* out) {
  std::ifstream is(path, std::ios::binary);
  if (!is) return false;
  char magic[8];
  if (!is.read(magic, 8) || std::memcmp(magic, kMagic, 8) != 0) return false;
  uint32_t version = 0, n_layers = 0, n_expert = 0;
  uint64_t n = 0;
  if (!Get(is, &version) || version != kVersion || !Get(is, &n_layers) || !Get(is, &n_expert) || !Get(is, &n))
    return false;
  RoutingTrace t;
  t.n_layers = n_layers;
  t.n_expert = n_expert;
  if (n < 1000000) t.records.reserve(n);
  for (uint64_t i = 0; i < n; ++i) {
    RoutingRecord r;
    uint32_t k = 0;
    if (!Get(is, &r.token) || !Get(is, &r.layer) || !Get(is, &k)) return false;
    if (n_expert != 0 && k > n_expert) return false;
    r.experts.resize(k);
    for (uint32_t j = 0; j < k; ++j)
      if (!Get(is, &r.experts[j])) return false;
    t.records.push_back(std::move(r));
  }
  *out = std::move(t);
  return true;
}

bool ReadRoutingTraceText(const std::string& path, RoutingTrace* out) {
  std::ifstream is(path);
  if (!is) return false;
  RoutingTrace t;
  uint32_t max_layer = 0, max_expert = 0, token = 0;
  std::string line;
  while (std::getline(is, line)) {
    std::istringstream ls(line);
    RoutingRecord r;
    if (!(ls >> r.layer)) continue;
    r.token = token++;
    uint32_t e = 0;
    while (ls >> e) {
      r.experts.push_back(e);
      max_expert = std::max(max_expert, e);
    }
    if (r.experts.empty()) continue;
    max_layer = std::max(max_layer, r.layer);
    t.records.push_back(std::move(r));
  }
  if (t.records.empty()) return false;
  t.n_layers = max_layer + 1;
  t.n_expert = max_expert + 1;
  *out = std::move(t);
  return true;
}

}  // namespace nuthatch

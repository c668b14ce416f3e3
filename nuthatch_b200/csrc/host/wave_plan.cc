// Slot-pool waves of the batched streaming form (host only).
#include "wave_plan.h"

#include "nh_kernels.h"

namespace nuthatch {

int PlanWaves(const int32_t* sel, int n_picks, int n_expert, int e_lo, int e_hi, int per,
              const std::vector<char>& pinned, std::vector<std::vector<int>>* waves, std::vector<int>* wave_of) {
  if ((sel == nullptr && n_picks > 0) || n_picks < 0 || n_expert <= 0 || e_lo < 0 || e_hi > n_expert ||
      e_lo > e_hi || static_cast<int>(pinned.size()) != n_expert || waves == nullptr || wave_of == nullptr)
    return NH_E_ARG;
  waves->clear();
  wave_of->assign(n_expert, -1);
  std::vector<int> pinned_seen;
  for (int j = 0; j < n_picks; ++j) {
    const int e = sel[j];
    if (e < 0 || e >= n_expert) return NH_E_STATE;
    if (e < e_lo || e >= e_hi || (*wave_of)[e] >= 0) continue;
    if (pinned[e]) {
      (*wave_of)[e] = 0;
      pinned_seen.push_back(e);
      continue;
    }
    if (per <= 0) return NH_E_CAPACITY;
    // The waves hold unpinned experts only until the loop ends.
    if (waves->empty() || static_cast<int>(waves->back().size()) == per) waves->emplace_back();
    waves->back().push_back(e);
    (*wave_of)[e] = static_cast<int>(waves->size()) - 1;
  }
  if (waves->empty()) waves->emplace_back();
  // Pinned experts join wave 0 after its unpinned ones, in order of first
  // selection (their Ensure hits change no LRU state).
  for (int e : pinned_seen) (*waves)[0].push_back(e);
  return static_cast<int>(waves->size());
}

int GroupWavePairs(const int32_t* sel, int n_picks, int k, const std::vector<int>& wave_of, int w,
                   const std::vector<int>& slot_of, int slots, int32_t* off, int32_t* cnt, int32_t* act,
                   int32_t* out) {
  if ((sel == nullptr && n_picks > 0) || n_picks < 0 || k <= 0 || slots <= 0 || off == nullptr || cnt == nullptr ||
      (n_picks > 0 && (act == nullptr || out == nullptr)) || wave_of.size() != slot_of.size())
    return NH_E_ARG;
  const int n_expert = static_cast<int>(wave_of.size());
  for (int g = 0; g < slots; ++g) cnt[g] = 0;
  for (int j = 0; j < n_picks; ++j) {
    const int e = sel[j];
    if (e < 0 || e >= n_expert) return NH_E_STATE;
    if (wave_of[e] != w) continue;
    const int g = slot_of[e];
    if (g < 0 || g >= slots) return NH_E_STATE;
    ++cnt[g];
  }
  int n = 0;
  for (int g = 0; g < slots; ++g) {
    off[g] = n;
    n += cnt[g];
  }
  std::vector<int32_t> cursor(off, off + slots);
  for (int j = 0; j < n_picks; ++j) {
    const int e = sel[j];
    if (wave_of[e] != w) continue;
    const int pos = cursor[slot_of[e]]++;
    act[pos] = j / k;
    out[pos] = j;
  }
  return n;
}

}  // namespace nuthatch

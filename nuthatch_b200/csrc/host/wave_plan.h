// Slot-pool waves of the batched streaming form (host only, no CUDA): which
// experts of one MoE layer are made resident together, and the (token, pick)
// pairs each wave's grouped products take.  No reference counterpart: the
// reference streams one sequence and requires distinct(ids) <= capacity per
// layer (expert_slot_cache.h:21).
#ifndef NUTHATCH_B200_HOST_WAVE_PLAN_H_
#define NUTHATCH_B200_HOST_WAVE_PLAN_H_

#include <cstdint>
#include <vector>

namespace nuthatch {

// The waves of one layer over n_picks selections `sel` (row-major
// [token][k]).  The distinct unpinned experts served here (ids in
// [e_lo, e_hi)) are taken in order of first selection, `per` to a wave; the
// pinned experts the batch selects (pinned[e] != 0, served ones only) join
// wave 0 after its unpinned experts, in order of first selection.  waves[w]
// is the id list one Ensure makes resident; wave_of[e] is expert e's wave, or
// -1 when the batch does not select it or it is served elsewhere.  There is
// always at least one wave.  Returns the number of waves, or NH_E_STATE for a
// selection outside [0, n_expert), NH_E_CAPACITY for an unpinned served
// expert with per <= 0, NH_E_ARG for bad sizes.
int PlanWaves(const int32_t* sel, int n_picks, int n_expert, int e_lo, int e_hi, int per,
              const std::vector<char>& pinned, std::vector<std::vector<int>>* waves, std::vector<int>* wave_of);

// The pairs of wave w grouped by slot: off[g], cnt[g] for the `slots` slots,
// then for pair i in slot order ((token, pick) order within a slot)
// act[i] = j / k (the token row) and out[i] = j (the pick index).
// slot_of[e] is the slot holding expert e (from that wave's Ensure).
// Returns the pair count, or NH_E_STATE when an expert of the wave has no
// slot in [0, slots), NH_E_ARG for bad sizes.
int GroupWavePairs(const int32_t* sel, int n_picks, int k, const std::vector<int>& wave_of, int w,
                   const std::vector<int>& slot_of, int slots, int32_t* off, int32_t* cnt, int32_t* act,
                   int32_t* out);

}  // namespace nuthatch

#endif  // NUTHATCH_B200_HOST_WAVE_PLAN_H_

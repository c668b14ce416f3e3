// Single-sequence KV cache in HBM (reference: src/model/kv_cache.h:14-35).
// Per layer, f32 K and V of [max_seq][n_embd_kv]; K holds post-RoPE keys.
#ifndef NUTHATCH_B200_KV_CACHE_H_
#define NUTHATCH_B200_KV_CACHE_H_

#include <vector>

#include "nuthatch/olmoe_model.h"

namespace nuthatch {

class KvCache {
 public:
  // Allocates 2 * n_layers * max_seq * n_embd_kv floats on the current device.
  KvCache(const OlmoeConfig& cfg, int max_seq);
  ~KvCache();

  KvCache(const KvCache&) = delete;
  KvCache& operator=(const KvCache&) = delete;

  bool ok() const { return base_ != nullptr; }
  float* k(int layer) const { return k_[layer]; }
  float* v(int layer) const { return v_[layer]; }

  int n_past() const { return n_past_; }
  void advance(int n) { n_past_ += n; }
  void reset() { n_past_ = 0; }
  int max_seq() const { return max_seq_; }

 private:
  void* base_ = nullptr;
  std::vector<float*> k_;
  std::vector<float*> v_;
  int n_past_ = 0;
  int max_seq_ = 0;
};

}  // namespace nuthatch

#endif  // NUTHATCH_B200_KV_CACHE_H_

// OLMoE model resident in HBM (reference: src/model/olmoe_model.h:18-68).
//
// OlmoeModel::Load reads every tensor of the GGUF into one device allocation
// in its native GGUF layout (each tensor 256-byte aligned, 256 bytes of tail
// padding).  tensor()/layer_tensor() return device tensor handles where the
// reference returns ggml_tensor*.
#ifndef NUTHATCH_B200_OLMOE_MODEL_H_
#define NUTHATCH_B200_OLMOE_MODEL_H_

#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>

namespace nuthatch {

class GgufFile;

// Hyper-parameters read from GGUF metadata (olmoe_model.h:18-32).
struct OlmoeConfig {
  uint32_t n_layers = 0;
  uint32_t n_embd = 0;
  uint32_t n_head = 0;
  uint32_t n_head_kv = 0;
  uint32_t n_ff = 0;
  uint32_t n_expert = 0;
  uint32_t n_expert_used = 0;
  uint32_t n_vocab = 0;
  uint32_t n_ctx_train = 0;
  float rope_freq_base = 10000.0f;
  float rms_eps = 1e-5f;

  uint32_t head_dim() const { return n_head ? n_embd / n_head : 0; }
};

// ParseOlmoeConfig (olmoe_model.cc:31-54): keys prefixed by
// general.architecture ("olmoe" when absent); head_count_kv defaults to
// head_count; n_vocab from output.weight ne[1], else token_embd.weight ne[1].
OlmoeConfig ParseOlmoeConfig(const GgufFile& g);

// A tensor in device memory (the ggml_tensor* of the reference API).
struct DTensor {
  std::string name;
  int32_t type = -1;
  int64_t ne[4] = {1, 1, 1, 1};
  size_t nb[4] = {0, 0, 0, 0};
  void* data = nullptr;  // device pointer
  size_t nbytes = 0;
};

class OlmoeModel {
 public:
  // nullptr on a missing/invalid GGUF, an unsupported tensor type, or a
  // device allocation/copy failure (olmoe_model.h:43-44).  Uses the current
  // CUDA device.
  static std::unique_ptr<OlmoeModel> Load(const std::string& path);
  // Expert-parallel load (no reference counterpart): every non-expert tensor,
  // and of each ffn_{gate,up,down}_exps tensor only experts [first, first +
  // count), whose DTensor then has ne[2] == count and starts at expert
  // `first`.  Such a model serves GreedyGenerateCachedBatch with an
  // ExpertGroup; the single-GPU entry points refuse it.
  static std::unique_ptr<OlmoeModel> LoadExpertShard(const std::string& path, uint32_t first, uint32_t count);
  ~OlmoeModel();

  OlmoeModel(const OlmoeModel&) = delete;
  OlmoeModel& operator=(const OlmoeModel&) = delete;

  const OlmoeConfig& config() const { return cfg_; }
  const DTensor* tensor(const std::string& name) const;
  const DTensor* layer_tensor(int layer, const std::string& suffix) const;

  int device() const { return device_; }
  size_t device_bytes() const { return bytes_; }
  // The experts held in device memory: [expert_first, expert_first +
  // expert_count); all of them (0, n_expert) after Load.
  uint32_t expert_first() const { return expert_first_; }
  uint32_t expert_count() const { return expert_count_; }
  bool holds_all_experts() const { return expert_first_ == 0 && expert_count_ == cfg_.n_expert; }

  // Reusable device workspace of the decode engine (KV cache, activations,
  // captured step graph); owned here so repeated generate calls do not
  // reallocate.  Internal.
  struct Workspace;
  Workspace* workspace() const { return ws_.get(); }

 private:
  OlmoeModel() = default;
  OlmoeConfig cfg_;
  int device_ = 0;
  uint32_t expert_first_ = 0, expert_count_ = 0;
  void* base_ = nullptr;
  size_t bytes_ = 0;
  std::unordered_map<std::string, DTensor> tensors_;
  std::unique_ptr<Workspace> ws_;
};

}  // namespace nuthatch

#endif  // NUTHATCH_B200_OLMOE_MODEL_H_

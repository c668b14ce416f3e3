// Expert parallelism across the GPUs of one node (no counterpart in the
// reference, which runs on one CPU; the EP configuration {world, rank,
// communicator} its drop-in boundary adds).
//
// One process per GPU.  Every rank holds the non-expert weights and a
// contiguous shard of each layer's experts (ExpertShard), and owns a
// contiguous share of the batch's sequences (attention is data-parallel).
// Per MoE layer the ranks all-gather the tokens' Q8_K activation rows and
// their top-k selections, each rank runs its own experts over every token
// that selected them, and an all-to-all returns each pick's output row to the
// token's rank, which adds the k products in top-k order (moe.cc:51-60), so
// every sequence's ids equal its single-GPU decode.
#ifndef NUTHATCH_B200_EXPERT_PARALLEL_H_
#define NUTHATCH_B200_EXPERT_PARALLEL_H_

#include <cstdint>
#include <memory>

namespace nuthatch {

// Experts [first, first + count) of n_expert belong to `rank` of `world`:
// equal contiguous shares (n_expert % world == 0 is required by callers).
struct ExpertShard {
  uint32_t first = 0;
  uint32_t count = 0;
  static ExpertShard Of(uint32_t n_expert, int world, int rank) {
    const uint32_t per = world > 0 ? n_expert / static_cast<uint32_t>(world) : n_expert;
    return {per * static_cast<uint32_t>(rank), per};
  }
};

// A communicator over the ranks of one expert-parallel job (NCCL underneath,
// loaded at run time).  Non-copyable; destroy it before the process group
// that exchanged its id.
class ExpertGroup {
 public:
  static constexpr int kIdBytes = 128;
  // Writes a new group id into id[kIdBytes] (one rank makes it and hands it
  // to the others, e.g. over torch.distributed).  False when NCCL is missing.
  static bool NewId(uint8_t* id);
  // Joins the group on the current CUDA device; collective over all ranks.
  // nullptr on failure (NCCL missing, bad arguments, or NCCL init failure).
  static std::unique_ptr<ExpertGroup> Create(const uint8_t* id, int world, int rank);
  ~ExpertGroup();
  ExpertGroup(const ExpertGroup&) = delete;
  ExpertGroup& operator=(const ExpertGroup&) = delete;

  int world() const { return world_; }
  int rank() const { return rank_; }
  void* comm() const { return comm_; }  // ncclComm_t

 private:
  ExpertGroup() = default;
  int world_ = 1, rank_ = 0;
  void* comm_ = nullptr;
};

}  // namespace nuthatch

#endif  // NUTHATCH_B200_EXPERT_PARALLEL_H_

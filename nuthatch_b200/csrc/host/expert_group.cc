// ExpertGroup: the NCCL communicator of an expert-parallel job.
#include <cstring>

#include "nccl_api.h"
#include "nuthatch/expert_parallel.h"

namespace nuthatch {

static_assert(sizeof(ncclUniqueId) == ExpertGroup::kIdBytes, "NCCL unique id size");

bool ExpertGroup::NewId(uint8_t* id) {
  const NcclApi& n = Nccl();
  if (!n.ok || id == nullptr) return false;
  ncclUniqueId u;
  if (n.GetUniqueId(&u) != ncclSuccess) return false;
  std::memcpy(id, &u, sizeof(u));
  return true;
}

std::unique_ptr<ExpertGroup> ExpertGroup::Create(const uint8_t* id, int world, int rank) {
  const NcclApi& n = Nccl();
  if (!n.ok || id == nullptr || world <= 0 || rank < 0 || rank >= world) return nullptr;
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  ncclComm_t comm = nullptr;
  if (n.CommInitRank(&comm, world, u, rank) != ncclSuccess || comm == nullptr) return nullptr;
  std::unique_ptr<ExpertGroup> g(new ExpertGroup());
  g->world_ = world;
  g->rank_ = rank;
  g->comm_ = comm;
  return g;
}

ExpertGroup::~ExpertGroup() {
  if (comm_ != nullptr) Nccl().CommDestroy(static_cast<ncclComm_t>(comm_));
}

}  // namespace nuthatch

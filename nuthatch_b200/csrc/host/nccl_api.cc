// NCCL entry points resolved at run time (see nccl_api.h).
#include "nccl_api.h"

#include <dlfcn.h>

#include <mutex>

namespace nuthatch {

namespace {

template <typename F>
bool Bind(void* h, const char* name, F* out) {
  *out = reinterpret_cast<F>(dlsym(h, name));
  return *out != nullptr;
}

NcclApi Resolve() {
  NcclApi a;
  // An NCCL the process already holds (e.g. torch's) first, so both users
  // share one copy; otherwise the loader's search path.
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (h == nullptr) return a;
  a.ok = Bind(h, "ncclGetUniqueId", &a.GetUniqueId) && Bind(h, "ncclCommInitRank", &a.CommInitRank) &&
         Bind(h, "ncclCommDestroy", &a.CommDestroy) && Bind(h, "ncclCommGetAsyncError", &a.CommGetAsyncError) &&
         Bind(h, "ncclAllGather", &a.AllGather) && Bind(h, "ncclSend", &a.Send) && Bind(h, "ncclRecv", &a.Recv) &&
         Bind(h, "ncclGroupStart", &a.GroupStart) && Bind(h, "ncclGroupEnd", &a.GroupEnd) &&
         Bind(h, "ncclGetErrorString", &a.GetErrorString);
  return a;
}

}  // namespace

const NcclApi& Nccl() {
  static std::once_flag once;
  static NcclApi api;
  std::call_once(once, [] { api = Resolve(); });
  return api;
}

}  // namespace nuthatch

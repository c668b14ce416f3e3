// Host-side launch helpers shared by the kernel files.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>
#include <mutex>
#include <utility>

#include "../../../include/nh_kernels.h"
#include "phase_trace.cuh"

namespace nh {

// SM count of the current device (cached per device).
inline int device_sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// Programmatic dependent launch is on unless NH_PDL=0 is set in the
// environment (read once).
inline int pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("NH_PDL");
    v = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return v;
}

// The lane-per-super-block row-dot engine is used where it covers the shape
// unless NH_ROWDOT=2 selects the lane-per-chunk engine everywhere (read once;
// both give identical results).
inline bool engine_v3() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("NH_ROWDOT");
    v = (e != nullptr && e[0] == '2') ? 0 : 1;
  }
  return v != 0;
}

// Upper bound on resident CTAs per SM for the row-dot kernels (NH_CTAS_PER_SM,
// default 2, read once).  One CTA per SM leaves room for the next kernel's
// CTAs to become resident early under programmatic dependent launch.
inline int ctas_per_sm_cap() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("NH_CTAS_PER_SM");
    v = (e != nullptr && e[0] >= '1' && e[0] <= '4') ? e[0] - '0' : 2;
  }
  return v;
}

// Batched Q4_K/Q6_K products run on the tensor cores unless NH_BATCH_MMA=0 (read
// once; both forms give identical results).
inline bool batch_mma_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("NH_BATCH_MMA");
    v = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return v != 0;
}

// The dynamic shared-memory limit one kernel has been given on each device.
// cudaFuncSetAttribute acts on the current device only, so a process that
// drives several GPUs needs one record per device.  Reads are lock-free; the
// rare raise is serialised so the attribute only ever grows and the record
// never claims more than was set.
struct SmemLimit {
  static constexpr int kMaxDevices = 64;
  std::atomic<size_t> limit[kMaxDevices];
  std::mutex raise;
  SmemLimit() {
    for (auto& l : limit) l.store(48 * 1024, std::memory_order_relaxed);
  }
};

template <typename Kern>
bool ensure_smem(Kern k, size_t bytes, SmemLimit& rec) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= SmemLimit::kMaxDevices) return false;
  std::atomic<size_t>& cur = rec.limit[dev];
  if (bytes <= cur.load(std::memory_order_acquire)) return true;
  std::lock_guard<std::mutex> hold(rec.raise);
  if (bytes <= cur.load(std::memory_order_relaxed)) return true;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)) != cudaSuccess)
    return false;
  cur.store(bytes, std::memory_order_release);
  return true;
}

// Launches with the programmatic-stream-serialisation attribute, so the
// kernel may begin while its predecessor in the stream finishes; kernels
// launched this way call griddepcontrol.wait before reading any result of
// the preceding kernel.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl_enabled();
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...) == cudaSuccess ? NH_OK : NH_E_CUDA;
}

// Cooperative launch: the runtime admits the grid only if every CTA can be
// resident at once, so CTAs may wait for one another.  Programmatic dependent
// launch is requested too; should the runtime refuse the pair, the launch is
// repeated without it and the pair is not tried again.
template <typename... KArgs, typename... Args>
int launch_coop(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  static std::atomic<bool> pair_ok{true};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = pdl_enabled();
  cfg.attrs = at;
  const bool pair = pair_ok.load(std::memory_order_relaxed);
  cfg.numAttrs = pair ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, kern, args...) == cudaSuccess) return NH_OK;
  if (!pair) return NH_E_CUDA;
  (void)cudaGetLastError();
  pair_ok.store(false, std::memory_order_relaxed);
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...) == cudaSuccess ? NH_OK : NH_E_CUDA;
}

}  // namespace nh

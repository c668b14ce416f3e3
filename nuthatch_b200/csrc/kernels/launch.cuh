// Host-side launch helpers shared by the kernel files.
#pragma once

#include <cuda_runtime.h>

#include <cstdlib>
#include <utility>

#include "../../../include/nh_kernels.h"

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

// Thread-block clusters that share the activation preparation are used only
// when NH_CLUSTER=1 (read once).  Measured on B200 they cost more in cluster
// barriers and scheduling than the shared preparation saves, so the default
// is one CTA per cluster.
inline bool clusters_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("NH_CLUSTER");
    v = (e != nullptr && e[0] == '1') ? 1 : 0;
  }
  return v != 0;
}

// Largest cluster size C <= 8 (a power of two) with K % (4*C) == 0 and, when
// the activation is quantised, (K/256) % C == 0; 1 when clusters are off.
inline int prep_cluster_size(int K, bool quant) {
  if (!clusters_enabled()) return 1;
  int c = 8;
  while (c > 1 && (K % (4 * c) != 0 || (quant && (K / 256) % c != 0))) c >>= 1;
  return c;
}

template <typename Kern>
bool ensure_smem(Kern k, size_t bytes, size_t& configured) {
  if (bytes <= configured) return true;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)) != cudaSuccess)
    return false;
  configured = bytes;
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

// launch_pdl with a 1-D thread-block cluster of `cluster` CTAs (grid.x must
// be a multiple of it).
template <typename... KArgs, typename... Args>
int launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, int cluster,
                       Args&&... args) {
  if (cluster <= 1) return launch_pdl(kern, grid, block, smem, s, std::forward<Args>(args)...);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl_enabled();
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = static_cast<unsigned>(cluster);
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...) == cudaSuccess ? NH_OK : NH_E_CUDA;
}

// Cooperative launch: the runtime admits the grid only if every CTA can be
// resident at once, so CTAs may wait for one another.  Programmatic dependent
// launch is requested too; should the runtime refuse the pair, the launch is
// repeated without it and the pair is not tried again.
template <typename... KArgs, typename... Args>
int launch_coop(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  static bool pair_ok = true;
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
  cfg.numAttrs = pair_ok ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, kern, args...) == cudaSuccess) return NH_OK;
  if (!pair_ok) return NH_E_CUDA;
  (void)cudaGetLastError();
  pair_ok = false;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...) == cudaSuccess ? NH_OK : NH_E_CUDA;
}

// Rounds a grid down to a multiple of the cluster size (at least one cluster).
inline int round_grid(int grid, int cluster) {
  if (cluster <= 1) return grid;
  const int g = grid / cluster * cluster;
  return g < cluster ? cluster : g;
}

}  // namespace nh

// Per-CTA phase timestamps of the decode kernels, for diagnosing latency
// chains (no reference counterpart).  Compiled in only with -DNH_PHASE_TRACE
// (`python -m nuthatch_b200.build --phase-trace` builds a separate library);
// in the product build every function below is empty.
//
// A traced CTA takes a ring slot at entry (its atomic's latency overlaps the
// kernel), keeps up to 12 %globaltimer stamps in shared memory (thread 0
// only, no atomics on the path), and writes one 128-byte record at its end:
// w[0] = kernel id << 32 | linear CTA index, w[1] = SM id, w[2 + i] = stamp i
// (0 = not reached; stamp 9 = end).  The ring has kPhaseTraceCap records; the
// host gives its buffer and counter with nh_phase_trace_set_<unit>().
#ifndef NUTHATCH_B200_PHASE_TRACE_CUH_
#define NUTHATCH_B200_PHASE_TRACE_CUH_

#include <cuda_runtime.h>

namespace nh {

#ifdef NH_PHASE_TRACE

struct PhaseRecord {
  unsigned long long w[16];
};
constexpr unsigned kPhaseTraceCap = 1u << 20;
static __device__ PhaseRecord* g_phase_ring = nullptr;
static __device__ unsigned* g_phase_count = nullptr;
static __shared__ unsigned long long g_phase_st[12];

__device__ __forceinline__ unsigned long long phase_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned phase_begin() {
  unsigned i = 0;
  if (threadIdx.x == 0 && g_phase_ring != nullptr) {
    for (int k = 1; k < 12; ++k) g_phase_st[k] = 0;
    g_phase_st[0] = phase_now();
    i = atomicAdd(g_phase_count, 1u);
  }
  return i;
}
__device__ __forceinline__ void phase_stamp(int ph) {
  if (threadIdx.x == 0 && g_phase_ring != nullptr) g_phase_st[ph] = phase_now();
}
__device__ __forceinline__ void phase_value(int slot, unsigned long long v) {
  if (threadIdx.x == 0 && g_phase_ring != nullptr) g_phase_st[slot] = v;
}
__device__ __forceinline__ void phase_end(int kid, unsigned i) {
  if (threadIdx.x != 0 || g_phase_ring == nullptr) return;
  g_phase_st[9] = phase_now();
  unsigned sm;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
  PhaseRecord* r = g_phase_ring + (i & (kPhaseTraceCap - 1));
  r->w[0] = (static_cast<unsigned long long>(kid) << 32) | (blockIdx.x + blockIdx.y * gridDim.x);
  r->w[1] = sm;
  for (int k = 0; k < 12; ++k) r->w[2 + k] = g_phase_st[k];
}
// phase_end after a CTA barrier (every thread of the CTA must call it).
__device__ __forceinline__ void phase_end_sync(int kid, unsigned i) {
  __syncthreads();
  phase_end(kid, i);
}
// Time spent in up to four recurring phases of a loop (thread 0's view).
struct PhaseAcc {
  unsigned long long acc[4] = {0, 0, 0, 0};
  unsigned long long prev = 0;
  __device__ __forceinline__ void start() { prev = phase_now(); }
  __device__ __forceinline__ void mark(int k) {
    const unsigned long long n = phase_now();
    acc[k] += n - prev;
    prev = n;
  }
  // Records the four totals as stamps 2..5.
  __device__ __forceinline__ void store() const {
    for (int k = 0; k < 4; ++k) phase_value(2 + k, acc[k]);
  }
};
static inline void phase_trace_set(void* ring, void* count) {
  cudaMemcpyToSymbol(g_phase_ring, &ring, sizeof(void*));
  cudaMemcpyToSymbol(g_phase_count, &count, sizeof(void*));
}
#define NH_PHASE_TRACE_SETTER(unit) \
  extern "C" void nh_phase_trace_set_##unit(void* ring, void* count) { nh::phase_trace_set(ring, count); }

#else  // product build: nothing is recorded

__device__ __forceinline__ unsigned phase_begin() { return 0; }
__device__ __forceinline__ void phase_stamp(int) {}
__device__ __forceinline__ void phase_value(int, unsigned long long) {}
__device__ __forceinline__ void phase_end(int, unsigned) {}
__device__ __forceinline__ void phase_end_sync(int, unsigned) {}
struct PhaseAcc {
  __device__ __forceinline__ void start() {}
  __device__ __forceinline__ void mark(int) {}
  __device__ __forceinline__ void store() const {}
};
#define NH_PHASE_TRACE_SETTER(unit)

#endif

// Kernel ids of the records.
enum PhaseKernel : int {
  kPhQkvOrOut = 1,  // gemv3 (QKV, output projection)
  kPhAttention = 2,
  kPhMoeFused = 3,
  kPhEmbed = 4,
  kPhLmHead = 5,
  kPhGroupedTc = 6,
  kPhRouter = 7,
  kPhGateUp = 8,
  kPhDown = 9,
  kPhBatchMma = 10,
  kPhBatchMmaStaged = 11,
  kPhBatchAttention = 12,
};

}  // namespace nh

#endif  // NUTHATCH_B200_PHASE_TRACE_CUH_

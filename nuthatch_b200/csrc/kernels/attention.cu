// Decode-step attention over the f32 KV cache, fused with QK-norm, NEOX RoPE
// and the KV append.
//
// Grid (n_head, n_split): CTA (h, s) owns positions [s*kAttnSplit,
// (s+1)*kAttnSplit) of query head h.  The cached K/V rows of its range were
// written by earlier tokens, so the CTA starts their cp.async.bulk copies into
// shared memory before griddepcontrol.wait.  Every CTA re-derives the
// normalised, rotated query of its head (the QK-norm spans the full width, so
// each CTA reduces the whole q row; a few KB of L2 reads).  The CTA whose
// range holds the current position also forms the current K/V row itself, and
// the first query head of each KV head appends it to the cache, so no CTA
// reads a cache row that is being written.  Partial (max, sum, weighted V)
// triples are combined by the last CTA of each head in split order, so the
// result does not depend on CTA scheduling.
#include <cmath>
#include <mutex>

#include "launch.cuh"
#include "attention.cuh"

namespace nh {

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnArgs p) {
  const int h = blockIdx.x, sp = blockIdx.y;
  // The cursor was last written by the previous token's argmax, completed
  // before this kernel could launch.
  const int pos = *reinterpret_cast<volatile const int*>(&p.state->pos);
  const int n_active = (pos + 1 + kAttnSplit - 1) / kAttnSplit;
  if (sp >= n_active) return;
  const unsigned ph_idx = phase_begin();
  extern __shared__ __align__(128) float sm[];
  __shared__ AttnShared sh;
  const AttnSmem m = carve_attn(sm, p.hd, p.n_head);
  // Cached K/V rows and norm weights do not depend on the preceding kernel.
  attn_begin(p, h, sp, pos, m, sh);
  pdl_wait();
  phase_stamp(1);
  pdl_trigger();
  attn_finish(p, h, sp, pos, m, sh);
  phase_end_sync(kPhAttention, ph_idx);
}


}  // namespace nh

using namespace nh;

extern "C" int64_t nh_attention_scratch_bytes(int n_head, int head_dim, int max_seq) {
  const int64_t S = attn_splits(max_seq);
  return 256 + n_head * S * (8 + 4 + 4 * static_cast<int64_t>(head_dim)) + 512;
}

extern "C" void nh_rope_table(float base, int head_dim, int max_seq, float* cs) {
  const int half = head_dim / 2;
  const float theta_scale = std::pow(base, -2.0f / static_cast<float>(head_dim));
  for (int p = 0; p < max_seq; ++p) {
    float theta = static_cast<float>(p);
    for (int i = 0; i < half; ++i) {
      cs[(static_cast<int64_t>(p) * half + i) * 2 + 0] = std::cos(theta);
      cs[(static_cast<int64_t>(p) * half + i) * 2 + 1] = std::sin(theta);
      theta *= theta_scale;
    }
  }
}

namespace {

// The host-side checks shared by both attention entries (everything but the
// scratch buffer); NH_OK when a launch may go ahead.
int attention_args_ok(const NhDecodeState* state, const float* q, const float* k, const float* v,
                      const float* q_norm, const float* k_norm, int n_head, int n_head_kv, int head_dim,
                      const float* rope_cs, const float* k_cache, const float* v_cache, int max_seq,
                      const float* attn_out) {
  if (state == nullptr || q == nullptr || k == nullptr || v == nullptr || q_norm == nullptr || k_norm == nullptr ||
      rope_cs == nullptr || k_cache == nullptr || v_cache == nullptr || attn_out == nullptr) {
    return NH_E_ARG;
  }
  // Cache rows are copied whole with 16-byte bulk copies: head_dim*4 must be
  // a multiple of 16 and the cache 16-byte aligned.
  if (n_head <= 0 || n_head_kv <= 0 || n_head % n_head_kv != 0 || head_dim <= 0 || head_dim % 4 != 0 ||
      head_dim > 256 || max_seq <= 0 || (reinterpret_cast<uintptr_t>(k_cache) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(v_cache) & 15) != 0) {
    return NH_E_ARG;
  }
  if (attn_smem_floats(head_dim, n_head, n_head_kv) * sizeof(float) > 220 * 1024) return NH_E_ARG;
  return NH_OK;
}

}  // namespace

extern "C" int nh_attention_step(const NhDecodeState* state, const float* q, const float* k, const float* v,
                                 const float* q_norm, const float* k_norm, float eps, int n_head, int n_head_kv,
                                 int head_dim, const float* rope_cs, float kq_scale, float* k_cache, float* v_cache,
                                 int max_seq, void* scratch, float* attn_out, void* stream) {
  const int rc = attention_args_ok(state, q, k, v, q_norm, k_norm, n_head, n_head_kv, head_dim, rope_cs, k_cache,
                                   v_cache, max_seq, attn_out);
  if (rc != NH_OK) return rc;
  if (scratch == nullptr) return NH_E_ARG;
  AttnArgs p;
  p.state = const_cast<NhDecodeState*>(state);
  p.q = q;
  p.k = k;
  p.v = v;
  p.q_norm = q_norm;
  p.k_norm = k_norm;
  p.eps = eps;
  p.n_head = n_head;
  p.n_head_kv = n_head_kv;
  p.hd = head_dim;
  p.rope_cs = rope_cs;
  p.kq_scale = kq_scale;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.n_split = attn_splits(max_seq);
  uint8_t* sc = static_cast<uint8_t*>(scratch);
  p.tickets = reinterpret_cast<unsigned*>(sc);
  const int64_t slots = static_cast<int64_t>(n_head) * p.n_split;
  int64_t off = 256;
  p.part_l = reinterpret_cast<double*>(sc + off);
  off += slots * 8;
  p.part_m = reinterpret_cast<float*>(sc + off);
  off += slots * 4;
  off = (off + 15) & ~15ll;
  p.part_acc = reinterpret_cast<float*>(sc + off);
  p.out = attn_out;
  const size_t smem = attn_smem_floats(head_dim, n_head, n_head_kv) * sizeof(float);
  static SmemLimit configured;
  if (!ensure_smem(attention_kernel, smem, configured)) return NH_E_CUDA;
  return launch_pdl(attention_kernel, dim3(n_head, p.n_split), dim3(kAttnThreads), smem,
                    static_cast<cudaStream_t>(stream), p);
}

// ---------------------------------------------------------------- no-alloc form
// nh_attention_step_static: the same attention step for callers that cannot
// allocate device memory themselves (code running inside a host-side
// allocator hook or a memory-pool callback, plugin hosts that own all device
// allocations, or a process whose allocator is already at its limit), so they
// cannot provide the split-combine scratch.  Its scratch is a file-scope
// device array of NH_ATTN_STATIC_SCRATCH_BYTES, which every GPU that loads
// this library holds until the process exits.
//
// In host code `g_attn_static_scratch` names a host-side stand-in, not device
// memory; the device address comes from cudaGetSymbolAddress, looked up once
// per device (with that device current) on the first call made there and kept
// for the life of the process.  cudaDeviceReset on a device destroys the
// context that address belongs to, so after a reset the kept address is stale:
// a process that resets a device must not call this entry on it again.
namespace {

__device__ __align__(256) uint8_t g_attn_static_scratch[NH_ATTN_STATIC_SCRATCH_BYTES];

constexpr int kStaticMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_addr[kStaticMaxDevices] = {};

// Device address of the array on the current device, or nullptr.
void* static_scratch_address() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kStaticMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (g_static_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_attn_static_scratch) != cudaSuccess) return nullptr;
    g_static_addr[dev] = p;
  }
  return g_static_addr[dev];
}

}  // namespace

extern "C" int nh_attention_step_static(const NhDecodeState* state, const float* q, const float* k, const float* v,
                                        const float* q_norm, const float* k_norm, float eps, int n_head,
                                        int n_head_kv, int head_dim, const float* rope_cs, float kq_scale,
                                        float* k_cache, float* v_cache, int max_seq, float* attn_out,
                                        void* stream) {
  // Every check runs before anything is enqueued: a rejected call launches
  // nothing and leaves the array untouched.  Capacity first (shapes only),
  // then the arguments nh_attention_step itself checks.
  if (n_head <= 0 || n_head_kv <= 0 || head_dim <= 0 || max_seq <= 0) return NH_E_ARG;
  // The per-head split counters occupy the first 256 bytes: 4 bytes per head.
  if (n_head > 64) return NH_E_CAPACITY;
  if (nh_attention_scratch_bytes(n_head, head_dim, max_seq) > NH_ATTN_STATIC_SCRATCH_BYTES) return NH_E_CAPACITY;
  const int rc = attention_args_ok(state, q, k, v, q_norm, k_norm, n_head, n_head_kv, head_dim, rope_cs, k_cache,
                                   v_cache, max_seq, attn_out);
  if (rc != NH_OK) return rc;
  void* scratch = static_scratch_address();
  if (scratch == nullptr) return NH_E_CUDA;
  // The array keeps whatever the previous call left; the counters must start
  // at zero (the split partials are always written before they are read).
  if (cudaMemsetAsync(scratch, 0, 256, static_cast<cudaStream_t>(stream)) != cudaSuccess) return NH_E_CUDA;
  return nh_attention_step(state, q, k, v, q_norm, k_norm, eps, n_head, n_head_kv, head_dim, rope_cs, kq_scale,
                           k_cache, v_cache, max_seq, scratch, attn_out, stream);
}

NH_PHASE_TRACE_SETTER(attention)

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
#include "rowdot.cuh"

namespace nh {

constexpr int kAttnThreads = 128;
constexpr int kAttnSplit = 64;

struct AttnArgs {
  NhDecodeState* state;
  const float* q;
  const float* k;
  const float* v;
  const float* q_norm;
  const float* k_norm;
  float eps;
  int n_head, n_head_kv, hd;
  const float* rope_cs;
  float kq_scale;
  float* k_cache;
  float* v_cache;
  int n_split;
  unsigned* tickets;
  double* part_l;
  float* part_m;
  float* part_acc;
  float* out;
};

__device__ void rope_inplace(float* x, int hd, const float* cs) {
  const int half = hd / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float c = cs[2 * i], s = cs[2 * i + 1];
    const float x0 = x[i], x1 = x[i + half];
    x[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    x[i + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
  }
}

// Score of one cached position as one thread computes it: the lane-strided
// partial sums of the 32 lanes (element i goes to lane i % 32, in order) and
// the same butterfly tree a warp reduction forms, so the value equals the
// warp-per-position form bit for bit.  hd is a multiple of 32; kr and q are
// 16-byte aligned shared rows.
__device__ __forceinline__ float score_thread(const float* kr, const float* q, int hd) {
  float part[32];
#pragma unroll
  for (int l = 0; l < 32; ++l) part[l] = 0.f;
  for (int base = 0; base < hd; base += 32) {
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float4 kv = *reinterpret_cast<const float4*>(kr + base + 4 * t);
      const float4 qv = *reinterpret_cast<const float4*>(q + base + 4 * t);
      part[4 * t + 0] = __fadd_rn(part[4 * t + 0], __fmul_rn(kv.x, qv.x));
      part[4 * t + 1] = __fadd_rn(part[4 * t + 1], __fmul_rn(kv.y, qv.y));
      part[4 * t + 2] = __fadd_rn(part[4 * t + 2], __fmul_rn(kv.z, qv.z));
      part[4 * t + 3] = __fadd_rn(part[4 * t + 3], __fmul_rn(kv.w, qv.w));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
    for (int l = 0; l < o; ++l) part[l] = __fadd_rn(part[l], part[l + o]);
  }
  return part[0];
}

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnArgs p) {
  const int h = blockIdx.x, sp = blockIdx.y;
  // The cursor was last written by the previous token's argmax, completed
  // before this kernel could launch.
  const int pos = *reinterpret_cast<volatile const int*>(&p.state->pos);
  const int n_kv = pos + 1;
  const int n_active = (n_kv + kAttnSplit - 1) / kAttnSplit;
  if (sp >= n_active) return;
  extern __shared__ __align__(128) float sm[];
  const int hd = p.hd;
  const int kst = hd + 4;              // padded K row stride: conflict-free 16-byte reads per position
  float* Ks = sm;                      // [kAttnSplit][kst]
  float* Vs = Ks + kAttnSplit * kst;   // [kAttnSplit][hd]
  float* qh = Vs + kAttnSplit * hd;
  float* kc = qh + hd;
  float* vc = kc + hd;
  float* qn = vc + hd;                 // this head's q_norm slice
  float* kn = qn + hd;                 // this KV head's k_norm slice
  float* sc = kn + hd;                 // [kAttnSplit]
  float* qfull = sc + kAttnSplit;      // [n_head*hd]
  float* kfull = qfull + p.n_head * hd;  // [n_head_kv*hd]
  __shared__ __align__(8) uint64_t bar;
  __shared__ double red[40];
  __shared__ float s_max[4];
  __shared__ bool s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
  const int group = p.n_head / p.n_head_kv;
  const int kh = h / group;
  const int dq = p.n_head * hd, dkv = p.n_head_kv * hd;
  const int half = hd / 2;
  const int p0 = sp * kAttnSplit;
  const int p1 = min(n_kv, p0 + kAttnSplit);
  const int n = p1 - p0;
  const int n_cached = max(0, min(p1, pos) - p0);
  const bool covers_cur = (p1 == n_kv);
  // Cached K/V rows of this range were written by earlier tokens: copy them
  // before waiting.  Thread j < n_cached copies K row j, thread 64 + j V row j.
  const uint32_t row = static_cast<uint32_t>(hd) * 4;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    mbar_expect_tx(&bar, 2u * row * static_cast<uint32_t>(n_cached));
  }
  __syncthreads();
  {
    const int j = tid & (kAttnSplit - 1);
    if (j < n_cached) {
      const int64_t g = static_cast<int64_t>(p0 + j) * dkv + kh * hd;
      if (tid < kAttnSplit) bulk_g2s(Ks + j * kst, p.k_cache + g, row, &bar);
      else bulk_g2s(Vs + j * hd, p.v_cache + g, row, &bar);
    }
  }
  // Norm weights are static: stage them before waiting.
  copy_to_smem(qn, p.q_norm + h * hd, hd);
  if (covers_cur) copy_to_smem(kn, p.k_norm + kh * hd, hd);
  pdl_wait();
  pdl_trigger();

  // q (and, for the CTA holding the current position, k and v) as one batch
  // of vector loads into shared memory.
  copy_to_smem(qfull, p.q, dq);
  if (covers_cur) {
    copy_to_smem(kfull, p.k, dkv);
    copy_to_smem(vc, p.v + kh * hd, hd);
  }
  __syncthreads();
  // RMS of the full q (and k) rows, sums of squares in double: per thread,
  // per warp, then the warp partials in order.
  {
    double sq = 0.0, sk = 0.0;
    for (int i = tid; i < dq; i += blockDim.x) sq += static_cast<double>(__fmul_rn(qfull[i], qfull[i]));
    if (covers_cur)
      for (int i = tid; i < dkv; i += blockDim.x) sk += static_cast<double>(__fmul_rn(kfull[i], kfull[i]));
    sq = warp_sum_d(sq);
    sk = warp_sum_d(sk);
    if (lane == 0) {
      red[warp] = sq;
      red[8 + warp] = sk;
    }
  }
  __syncthreads();
  const float* cs = p.rope_cs + static_cast<int64_t>(pos) * hd;
  {
    double tq = 0.0, tk = 0.0;
    for (int w = 0; w < nw; ++w) {
      tq += red[w];
      tk += red[8 + w];
    }
    const float scq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(tq / static_cast<double>(dq)), p.eps)));
    // Normalise and rotate (NEOX pairs i, i + hd/2) in one step.
    for (int i = tid; i < half; i += blockDim.x) {
      const float c = cs[2 * i], s = cs[2 * i + 1];
      const float x0 = __fmul_rn(__fmul_rn(qfull[h * hd + i], scq), qn[i]);
      const float x1 = __fmul_rn(__fmul_rn(qfull[h * hd + i + half], scq), qn[i + half]);
      qh[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
      qh[i + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
    if (covers_cur) {
      const float sck =
          __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(tk / static_cast<double>(dkv)), p.eps)));
      for (int i = tid; i < half; i += blockDim.x) {
        const float c = cs[2 * i], s = cs[2 * i + 1];
        const float x0 = __fmul_rn(__fmul_rn(kfull[kh * hd + i], sck), kn[i]);
        const float x1 = __fmul_rn(__fmul_rn(kfull[kh * hd + i + half], sck), kn[i + half]);
        const float r0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        const float r1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        kc[i] = r0;
        kc[i + half] = r1;
        if (h % group == 0) {
          // The first query head of each KV head appends the new row.
          float* kd = p.k_cache + static_cast<int64_t>(pos) * dkv + kh * hd;
          kd[i] = r0;
          kd[i + half] = r1;
        }
      }
      if (h % group == 0) {
        float* vd = p.v_cache + static_cast<int64_t>(pos) * dkv + kh * hd;
        for (int i = tid; i < hd; i += blockDim.x) vd[i] = vc[i];
      }
    }
  }
  const bool ok = mbar_wait(&bar, 0);
  if (!ok && tid == 0) atomicCAS(&p.state->error, 0, NH_E_TIMEOUT);
  __syncthreads();

  // Scores kq = K.q * kq_scale.
  float my = -INFINITY;  // this thread's score (thread j: position p0 + j)
  if ((hd & 31) == 0) {
    if (tid < n) {
      const float* kr = (p0 + tid == pos) ? kc : Ks + tid * kst;
      const float d = score_thread(kr, qh, hd);
      my = ok ? __fmul_rn(d, p.kq_scale) : 0.f;
    }
  } else {
    for (int j = warp; j < n; j += nw) {
      const float* kr = (p0 + j == pos) ? kc : Ks + j * kst;
      float d = 0.f;
      for (int i = lane; i < hd; i += 32) d = __fadd_rn(d, __fmul_rn(kr[i], qh[i]));
      d = warp_sum(d);
      if (lane == 0) sc[j] = ok ? __fmul_rn(d, p.kq_scale) : 0.f;
    }
    __syncthreads();
    if (tid < n) my = sc[tid];
  }
  // n <= kAttnSplit (64) < blockDim.x: thread j holds position j.
  float m = warp_max(my);
  if (lane == 0) s_max[warp] = m;
  __syncthreads();
  m = s_max[0];
  for (int w = 1; w < nw; ++w) m = fmaxf(m, s_max[w]);
  const float e = tid < n ? exp_cw(__fsub_rn(my, m)) : 0.f;
  double l = warp_sum_d(tid < n ? static_cast<double>(e) : 0.0);
  if (lane == 0) red[16 + warp] = l;
  __syncthreads();
  l = 0.0;
  for (int w = 0; w < nw; ++w) l += red[16 + w];
  if (tid < n) sc[tid] = n_active == 1 ? __fmul_rn(e, static_cast<float>(1.0 / l)) : e;
  __syncthreads();

  float* out = p.out + h * hd;
  if (n_active == 1) {
    // ggml_soft_max scaled the exponentials by 1/sum before the V product (above).
    for (int i = tid; i < hd; i += blockDim.x) {
      float acc = 0.f;
      for (int j = 0; j < n; ++j) {
        const float vv = (p0 + j == pos) ? vc[i] : Vs[j * hd + i];
        acc = __fadd_rn(acc, __fmul_rn(vv, sc[j]));
      }
      out[i] = acc;
    }
    return;
  }
  const int slot = h * p.n_split + sp;
  for (int i = tid; i < hd; i += blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < n; ++j) {
      const float vv = (p0 + j == pos) ? vc[i] : Vs[j * hd + i];
      acc = __fadd_rn(acc, __fmul_rn(vv, sc[j]));
    }
    p.part_acc[static_cast<int64_t>(slot) * hd + i] = acc;
  }
  if (tid == 0) {
    p.part_m[slot] = m;
    p.part_l[slot] = l;
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned t = atomicAdd(&p.tickets[h], 1u);
    s_last = (t == static_cast<unsigned>(n_active - 1));
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // Combine the splits in order: weights exp(m_s - M) staged in shared memory.
  const volatile float* pm = p.part_m;
  const volatile double* pl = p.part_l;
  float M = -INFINITY;
  for (int s = 0; s < n_active; ++s) M = fmaxf(M, pm[h * p.n_split + s]);
  float* wsplit = sc;  // reuse: n_active <= n_split; sized kAttnSplit, so combine in chunks
  double L = 0.0;
  for (int s0 = 0; s0 < n_active; s0 += kAttnSplit) {
    const int cnt = min(kAttnSplit, n_active - s0);
    __syncthreads();
    for (int s = tid; s < cnt; s += blockDim.x) wsplit[s] = exp_cw(__fsub_rn(pm[h * p.n_split + s0 + s], M));
    __syncthreads();
    for (int s = 0; s < cnt; ++s) L += pl[h * p.n_split + s0 + s] * static_cast<double>(wsplit[s]);
  }
  const float inv = static_cast<float>(1.0 / L);
  for (int i = tid; i < hd; i += blockDim.x) {
    float acc = 0.f;
    for (int s0 = 0; s0 < n_active; s0 += kAttnSplit) {
      const int cnt = min(kAttnSplit, n_active - s0);
      for (int s = 0; s < cnt; ++s) {
        const float w = exp_cw(__fsub_rn(pm[h * p.n_split + s0 + s], M));
        acc = __fadd_rn(acc, __fmul_rn(__ldcg(&p.part_acc[static_cast<int64_t>(h * p.n_split + s0 + s) * hd + i]), w));
      }
    }
    out[i] = __fmul_rn(acc, inv);
  }
  if (tid == 0) p.tickets[h] = 0u;
}

int attn_splits(int max_seq) { return (max_seq + kAttnSplit - 1) / kAttnSplit; }

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

extern "C" int nh_attention_step(const NhDecodeState* state, const float* q, const float* k, const float* v,
                                 const float* q_norm, const float* k_norm, float eps, int n_head, int n_head_kv,
                                 int head_dim, const float* rope_cs, float kq_scale, float* k_cache, float* v_cache,
                                 int max_seq, void* scratch, float* attn_out, void* stream) {
  if (state == nullptr || q == nullptr || k == nullptr || v == nullptr || q_norm == nullptr || k_norm == nullptr ||
      rope_cs == nullptr || k_cache == nullptr || v_cache == nullptr || scratch == nullptr || attn_out == nullptr) {
    return NH_E_ARG;
  }
  // Cache rows are copied whole with 16-byte bulk copies: head_dim*4 must be
  // a multiple of 16 and the cache 16-byte aligned.
  if (n_head <= 0 || n_head_kv <= 0 || n_head % n_head_kv != 0 || head_dim <= 0 || head_dim % 4 != 0 ||
      head_dim > 256 || max_seq <= 0 || (reinterpret_cast<uintptr_t>(k_cache) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(v_cache) & 15) != 0) {
    return NH_E_ARG;
  }
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
  const size_t smem = static_cast<size_t>(kAttnSplit * (head_dim + 4) + kAttnSplit * head_dim + 5 * head_dim +
                                          kAttnSplit + (n_head + n_head_kv) * head_dim) *
                      sizeof(float);
  if (smem > 220 * 1024) return NH_E_ARG;
  static size_t configured = 48 * 1024;
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
// per device (with that device current) on the first call made there and kept.
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
  if (n_head <= 0 || n_head_kv <= 0 || head_dim <= 0 || max_seq <= 0) return NH_E_ARG;
  // The per-head split counters occupy the first 256 bytes: 4 bytes per head.
  if (n_head > 64) return NH_E_CAPACITY;
  if (nh_attention_scratch_bytes(n_head, head_dim, max_seq) > NH_ATTN_STATIC_SCRATCH_BYTES) return NH_E_CAPACITY;
  void* scratch = static_scratch_address();
  if (scratch == nullptr) return NH_E_CUDA;
  // The array keeps whatever the previous call left; the counters must start
  // at zero (the split partials are always written before they are read).
  if (cudaMemsetAsync(scratch, 0, 256, static_cast<cudaStream_t>(stream)) != cudaSuccess) return NH_E_CUDA;
  return nh_attention_step(state, q, k, v, q_norm, k_norm, eps, n_head, n_head_kv, head_dim, rope_cs, kq_scale,
                           k_cache, v_cache, max_seq, scratch, attn_out, stream);
}
